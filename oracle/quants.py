"""GGUF block decoders restated in numpy (test infrastructure: the CUDA path's checker, never the product).

Each decoder maps blocks `(n, block_bytes)` uint8 to weights `(n, per_block)` float32, evaluated in float32 in
the operation order of gguf-py 0.19.0's `dequantize_blocks` (the decoder the reference's tests hold its
kernels to, `tests/test_blocks.py:18-24`) so that every weight is bit-equal to it. The layout of every field
is written as per-weight position tables (byte, shift) built once from the formulas, rather than by reshapes.

Sources followed, per type (reference = yibie/strata-mlx; gguf-py = gguf 0.19.0 `gguf/quants.py`):
  Q8_0     gguf-py Q8_0.dequantize_blocks (quants.py:378);   reference strata_mlx/gguf.py:203-206
  Q2_K     gguf-py Q2_K.dequantize_blocks (quants.py:404-428); absent from the reference
  Q3_K     reference strata_mlx/blocks.py:164-175 (_UNPACK) and 45-50 (q3k_scale); gguf-py quants.py:431
  Q4_K     reference strata_mlx/gguf.py:174-179, 207-216; gguf-py quants.py:475
  Q5_K     reference strata_mlx/gguf.py:207-218;               gguf-py quants.py:525
  Q6_K     reference strata_mlx/gguf.py:135-165 (to_float, q6k_parts); gguf-py quants.py:552
  IQ3_XXS  reference strata_mlx/blocks.py:103-116;             gguf-py quants.py:1005
  IQ3_S    reference strata_mlx/blocks.py:89-102;              gguf-py quants.py:1057
  IQ4_XS   reference strata_mlx/blocks.py:78-88;               gguf-py quants.py:1351
  IQ4_NL   reference strata_mlx/blocks.py:69-77
  IQ2_XXS  reference strata_mlx/blocks.py:148-161
  IQ2_XS   reference strata_mlx/blocks.py:133-147
  IQ2_S    reference strata_mlx/blocks.py:117-132
  IQ1_M    reference strata_mlx/blocks.py:177-193
  Q2_0     reference strata_mlx/blocks.py:58-68, tests/test_gguf.py:34-38
The codebook grids and sign table are ggml's, read from gguf-py at import (as the reference reads them,
`strata_mlx/blocks.py:275-289`).
"""

import numpy as np

# name -> (GGML type id, weights per block, bytes per block); ids as strata_mlx/gguf.py:25-33
TYPES = {
    "Q8_0": (8, 32, 34), "Q2_K": (10, 256, 84), "Q3_K": (11, 256, 110), "Q4_K": (12, 256, 144),
    "Q5_K": (13, 256, 176), "Q6_K": (14, 256, 210), "IQ2_XXS": (16, 256, 66), "IQ2_XS": (17, 256, 74),
    "IQ3_XXS": (18, 256, 98), "IQ4_NL": (20, 32, 18), "IQ3_S": (21, 256, 110), "IQ2_S": (22, 256, 82),
    "IQ4_XS": (23, 256, 136), "IQ1_M": (29, 256, 56), "Q2_0": (42, 64, 18),
}
# where each block keeps its 16-bit float scales (as the reference's fixtures, tests/test_gguf.py:12-14,
# plus Q2_K's d and dmin at 80 and 82)
SCALE_BYTES = {"Q2_0": [0], "Q8_0": [0], "IQ4_NL": [0], "IQ4_XS": [0], "Q4_K": [0, 2], "Q5_K": [0, 2],
               "Q3_K": [108], "Q6_K": [208], "Q2_K": [80, 82], "IQ3_S": [0], "IQ3_XXS": [0], "IQ2_S": [0],
               "IQ2_XS": [0], "IQ2_XXS": [0], "IQ1_M": []}
KVALUES = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], dtype=np.int8)

f32 = np.float32
_J = np.arange(256)
_J32 = np.arange(32)


def _grid(name):
    from gguf import quants

    cls = getattr(quants, name)
    cls.init_grid()
    return cls.grid.reshape(cls.grid_shape).astype(np.float32)


def _ksigns():
    from gguf import quants

    return np.frombuffer(quants.IQ2_XXS.ksigns, dtype=np.uint8)


def _half(b, at):
    """The little-endian float16 at byte `at` of every block, as float32."""
    bits = b[:, at].astype(np.uint16) | (b[:, at + 1].astype(np.uint16) << 8)
    return bits.view(np.float16).astype(f32)


def _u16(b, at):
    return b[:, at].astype(np.uint32) | (b[:, at + 1].astype(np.uint32) << 8)


def _u32(b, at):
    return _u16(b, at) | (_u16(b, at + 2) << 16)


def _bits(b, byte, shift, width):
    """Field of `width` bits at per-weight (byte, shift) tables, for every block: (n, len(byte))."""
    return (b[:, byte] >> np.asarray(shift, dtype=np.uint8)) & np.uint8((1 << width) - 1)


# ---- one function per type: blocks (n, bytes) -> (n, per_block) float32

def q8_0(b):
    d = _half(b, 0)
    return d[:, None] * b[:, 2:34].view(np.int8).astype(f32)


def q2_k(b):
    sub = _J // 16
    q = _bits(b, 16 + 32 * (_J // 128) + _J % 32, 2 * ((_J % 128) // 32), 2).astype(f32)
    sc = b[:, sub]
    dl = _half(b, 80)[:, None] * (sc & 15).astype(f32)
    ml = _half(b, 82)[:, None] * (sc >> 4).astype(f32)
    return dl * q - ml


def _q3k_scales(b):
    """The sixteen 6-bit scales of a Q3_K block less 32, (n, 16) float32 (strata_mlx/blocks.py:45-50)."""
    k = np.arange(16)
    low = np.where(k < 8, b[:, 96 + k % 8] & 15, b[:, 96 + k % 8] >> 4)
    high = (b[:, 104 + k % 4] >> (2 * (k // 4)).astype(np.uint8)) & 3
    return ((low | (high << 4)).astype(np.int16) - 32).astype(f32)


def q3_k(b):
    two = _bits(b, 32 + 32 * (_J // 128) + _J % 32, 2 * ((_J % 128) // 32), 2).astype(np.int16)
    hm = _bits(b, _J % 32, _J // 32, 1)
    q = (two - np.where(hm == 1, 0, 4)).astype(f32)
    dl = _half(b, 108)[:, None] * _q3k_scales(b)
    return dl[:, _J // 16] * q


def _k4_scale_min(b):
    """Eight 6-bit (scale, min) pairs of a Q4_K/Q5_K block from bytes 4..15 (strata_mlx/gguf.py:174-179)."""
    t = np.arange(8)
    lo = t < 4
    s = lambda i: b[:, 4 + i]  # noqa: E731
    sc = np.where(lo, s(t % 4) & 63, (s(8 + t % 4) & 15) | ((s(t % 4) >> 6) << 4))
    mn = np.where(lo, s(4 + t % 4) & 63, (s(8 + t % 4) >> 4) | ((s(4 + t % 4) >> 6) << 4))
    return sc.astype(f32), mn.astype(f32)


def q4_k(b):
    t = _J // 32
    q = _bits(b, 16 + 32 * (t // 2) + _J % 32, 4 * (t % 2), 4).astype(f32)
    sc, mn = _k4_scale_min(b)
    dl = (_half(b, 0)[:, None] * sc)[:, t]
    ml = (_half(b, 2)[:, None] * mn)[:, t]
    return dl * q - ml


def q5_k(b):
    t = _J // 32
    low = _bits(b, 48 + 32 * (t // 2) + _J % 32, 4 * (t % 2), 4)
    high = _bits(b, 16 + _J % 32, t, 1)
    q = (low | (high << 4)).astype(f32)
    sc, mn = _k4_scale_min(b)
    dl = (_half(b, 0)[:, None] * sc)[:, t]
    ml = (_half(b, 2)[:, None] * mn)[:, t]
    return dl * q - ml


def q6_k(b):
    h, r = _J // 128, _J % 128
    low = _bits(b, 64 * h + r % 64, 4 * (r // 64), 4)
    high = _bits(b, 128 + 32 * h + r % 32, 2 * (r // 32), 2)
    q = ((low | (high << 4)).astype(np.int16) - 32).astype(f32)
    sc = b[:, 192:208].view(np.int8).astype(f32)
    dsc = _half(b, 208)[:, None] * sc  # (d * scale) first, then * q: the product can need 25 bits
    return dsc[:, _J // 16] * q


def iq3_xxs(b):
    grid, ksigns = _grid("IQ3_XXS"), _ksigns()
    ib, l = _J // 32, (_J % 32) // 4
    aux = np.stack([_u32(b, 66 + 4 * i) for i in range(8)], axis=1)  # (n, 8)
    db = _half(b, 0)[:, None] * (f32(0.5) + (aux >> 28).astype(f32)) * f32(0.5)
    g = grid[b[:, 2 + 8 * ib + l], _J % 4]
    m = (_J % 32) // 8
    sign_byte = ksigns[(aux[:, ib] >> (7 * m).astype(np.uint32)) & 127]
    neg = (sign_byte >> (_J % 8).astype(np.uint8)) & 1
    return db[:, ib] * g * np.where(neg == 1, f32(-1), f32(1))


def iq3_s(b):
    grid = _grid("IQ3_S")
    ib, l = _J // 32, (_J % 32) // 4
    sc = _bits(b, 106 + np.arange(8) // 2, 4 * (np.arange(8) % 2), 4)
    db = _half(b, 0)[:, None] * (1 + 2 * sc.astype(np.int32)).astype(f32)
    index = b[:, 2 + 8 * ib + l].astype(np.int32) | (_bits(b, 66 + ib, l, 1).astype(np.int32) << 8)
    g = grid[index, _J % 4]
    neg = _bits(b, 74 + _J // 8, _J % 8, 1)
    return db[:, ib] * g * np.where(neg == 1, f32(-1), f32(1))


def iq4_xs(b):
    i8 = np.arange(8)
    low = _bits(b, 4 + i8 // 2, 4 * (i8 % 2), 4).astype(np.uint32)
    high = (_u16(b, 2)[:, None] >> (2 * i8).astype(np.uint32)) & 3
    ls = (low | (high << 4)).astype(np.int32) - 32
    dl = _half(b, 0)[:, None] * ls.astype(f32)
    ib = _J // 32
    q = _bits(b, 8 + 16 * ib + _J % 16, 4 * ((_J % 32) // 16), 4)
    return dl[:, ib] * KVALUES[q].astype(f32)


def iq4_nl(b):
    q = _bits(b, 2 + _J32 % 16, 4 * (_J32 // 16), 4)
    return _half(b, 0)[:, None] * KVALUES[q].astype(f32)


def q2_0(b):
    j = np.arange(64)
    q = _bits(b, 2 + j // 4, 2 * (j % 4), 2).astype(f32)
    return _half(b, 0)[:, None] * (q - f32(1))


def iq2_xxs(b):
    grid, ksigns = _grid("IQ2_XXS"), _ksigns()
    ib, l = _J // 32, (_J % 32) // 8
    aux = np.stack([_u32(b, 2 + 8 * i + 4) for i in range(8)], axis=1)
    db = _half(b, 0)[:, None] * (f32(0.5) + (aux >> 28).astype(f32)) * f32(0.25)
    g = grid[b[:, 2 + 8 * ib + l], _J % 8]
    sign_byte = ksigns[(aux[:, ib] >> (7 * l).astype(np.uint32)) & 127]
    neg = (sign_byte >> (_J % 8).astype(np.uint8)) & 1
    return db[:, ib] * g * np.where(neg == 1, f32(-1), f32(1))


def iq2_xs(b):
    grid, ksigns = _grid("IQ2_XS"), _ksigns()
    ib, l = _J // 32, (_J % 32) // 8
    q16 = np.stack([_u16(b, 2 + 2 * i) for i in range(32)], axis=1)[:, 4 * ib + l]
    sc = _bits(b, 66 + ib, 4 * (l // 2), 4).astype(f32)
    dl = _half(b, 0)[:, None] * f32(0.25) * (f32(0.5) + sc)
    g = grid[q16 & 511, _J % 8]
    neg = (ksigns[q16 >> 9] >> (_J % 8).astype(np.uint8)) & 1
    return dl * g * np.where(neg == 1, f32(-1), f32(1))


def iq2_s(b):
    grid = _grid("IQ2_S")
    ib, l = _J // 32, (_J % 32) // 8
    index = b[:, 2 + 4 * ib + l].astype(np.int32) | (_bits(b, 66 + ib, 2 * l, 2).astype(np.int32) << 8)
    sc = _bits(b, 74 + ib, 4 * (l // 2), 4).astype(f32)
    dl = _half(b, 0)[:, None] * f32(0.25) * (f32(0.5) + sc)
    g = grid[index, _J % 8]
    neg = _bits(b, 34 + 4 * ib + l, _J % 8, 1)
    return dl * g * np.where(neg == 1, f32(-1), f32(1))


def iq1_m(b):
    grid = _grid("IQ1_M")  # values -1, 0, 1
    words = np.stack([_u16(b, 48 + 2 * i) for i in range(4)], axis=1)
    packed = ((words[:, 0] >> 12) | ((words[:, 1] >> 8) & 0x00F0) | ((words[:, 2] >> 4) & 0x0F00)
              | (words[:, 3] & 0xF000)).astype(np.uint16)
    d = packed.view(np.float16).astype(f32)
    ib, l = _J // 32, (_J % 32) // 8
    scales = words[:, ib // 2] >> (6 * (ib % 2)).astype(np.uint32)
    s3 = (scales >> (3 * (l // 2)).astype(np.uint32)) & 7
    dl = d[:, None] * (2 * s3 + 1).astype(f32)
    high = _bits(b, 32 + 2 * ib + l // 2, 4 * (l % 2), 4).astype(np.int32)
    index = b[:, 4 * ib + l].astype(np.int32) | ((high & 7) << 8)
    delta = np.where(high & 8, f32(-0.125), f32(0.125))
    return dl * (grid[index, _J % 8] + delta)


DECODERS = {"Q8_0": q8_0, "Q2_K": q2_k, "Q3_K": q3_k, "Q4_K": q4_k, "Q5_K": q5_k, "Q6_K": q6_k,
            "IQ3_XXS": iq3_xxs, "IQ3_S": iq3_s, "IQ4_XS": iq4_xs, "IQ4_NL": iq4_nl, "Q2_0": q2_0,
            "IQ2_XXS": iq2_xxs, "IQ2_XS": iq2_xs, "IQ2_S": iq2_s, "IQ1_M": iq1_m}


def row_bytes(kind: str, cols: int) -> int:
    _, per_block, block_bytes = TYPES[kind]
    if cols % per_block:
        raise ValueError(f"{kind}: rows of {cols} weights do not end on a block of {per_block}")
    return cols // per_block * block_bytes


def dequantize(blocks: np.ndarray, kind: str, shape: tuple) -> np.ndarray:
    """Every weight of a stack of `shape` (rows run along the last axis) as float32.

    Restates `strata_mlx/blocks.py:515-522` (`dequantize`): one call of the type's decoder per block.
    """
    _, per_block, block_bytes = TYPES[kind]
    row_bytes(kind, shape[-1])
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1, block_bytes)
    if b.shape[0] * per_block != int(np.prod(shape)):
        raise ValueError(f"{kind}: {b.shape[0]} blocks do not hold a tensor of {shape}")
    out = np.empty((b.shape[0], per_block), dtype=f32)
    step = 1 << 15
    for i in range(0, b.shape[0], step):  # bounded temporaries for large stacks
        out[i : i + step] = DECODERS[kind](b[i : i + step])
    return out.reshape(shape)


def random_blocks(kind: str, n_blocks: int, rng: np.random.Generator, scale=(-0.05, 0.05), normal=None):
    """Uniform random block bytes with the float16 scale fields overwritten (tests/test_gguf.py:17-30).

    `scale` draws the scales uniformly from an interval; `normal=sigma` draws |N(0, sigma)| instead (the
    benchmark's blocks: a positive super-scale around sigma).
    """
    _, _, block_bytes = TYPES[kind]
    b = rng.integers(0, 256, (n_blocks, block_bytes), dtype=np.uint8)

    def draw(n):
        if normal is not None:
            return np.abs(rng.normal(0.0, normal, n))
        return rng.uniform(scale[0], scale[1], n)

    for at in SCALE_BYTES[kind]:
        b[:, at : at + 2] = draw(n_blocks).astype("<f2").reshape(-1, 1).view(np.uint8)
    if kind == "IQ1_M":  # its scale is spread over the top nibbles of the four words at byte 48
        d = draw(n_blocks).astype("<f2").view("<u2")
        words = b[:, 48:56].copy().view("<u2")
        for i in range(4):
            words[:, i] = (words[:, i] & 0x0FFF) | (((d >> (4 * i)) & 15) << 12)
        b[:, 48:56] = words.view(np.uint8)
    return b
