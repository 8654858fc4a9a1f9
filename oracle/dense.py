"""The dense steps around the MoE block restated in numpy (test infrastructure: the CUDA path's checker, never the
product). Each function names the reference code it restates (yibie/strata-mlx, paths within that project).

    q6k_parts             Q6_K blocks -> (codes, scales, d)              strata_mlx/gguf.py:150-165
    scaled_floats/window  ScaledLinear's weights and its window product  strata_mlx/dense.py:30-84, 128-167
    q3k_planes            Q3_K blocks -> {hm, qs, sc, dd}                strata_mlx/blocks.py:403-414
    q3k_planes_weights    the weights the planes hold                     strata_mlx/blocks.py:417-424, 462-479
    hyper_connection      norm, low-rank gate and mix                    strata_mlx/fused.py:46-146, 280-323

Products are taken in float64 (the more exact side); values are rounded where the reference rounds them (the
residual, inject and mixed outputs to the activations' type; the weights of `scaled_floats` once).
"""

import numpy as np


def _half(b, at):
    return b[:, at : at + 2].copy().view("<f2").reshape(-1)


def q6k_parts(blocks, rows, cols):
    """A Q6_K tensor's blocks as (codes int8 (rows, cols): the six bits less 32 in the weights' order, scales int8
    (rows, cols / 16), d float16 (rows, cols / 256)). Weight 128 h + 32 q + l of a block takes the low nibble of
    ql[64 h + 32 (q % 2) + l] (shifted by 4 (q / 2)) and two high bits of qh[32 h + l] (shifted by 2 q)."""
    b = np.asarray(blocks, dtype=np.uint8).reshape(-1, 210)
    n = b.shape[0]
    codes = np.empty((n, 256), dtype=np.int16)
    for h in range(2):
        for q in range(4):
            lo = (b[:, 64 * h + 32 * (q % 2) : 64 * h + 32 * (q % 2) + 32] >> (4 * (q // 2))) & 15
            hi = (b[:, 128 + 32 * h : 128 + 32 * h + 32] >> (2 * q)) & 3
            codes[:, 128 * h + 32 * q : 128 * h + 32 * q + 32] = (lo | (hi << 4)).astype(np.int16) - 32
    scales = b[:, 192:208].copy().view(np.int8)
    d = _half(b, 208)
    return (codes.astype(np.int8).reshape(rows, cols), scales.reshape(rows, cols // 16), d.reshape(rows, cols // 256))


def scaled_floats(codes, scales, d, dtype=np.float32):
    """Every weight (float32(d) float32(scale)) float32(code), rounded once to `dtype`."""
    rows, cols = codes.shape
    d_step = cols // d.shape[1]
    s = (np.repeat(d.astype(np.float32), d_step // 16, axis=1) * scales.astype(np.float32)).astype(np.float32)
    return (np.repeat(s, 16, axis=1) * codes.astype(np.float32)).astype(np.float32).astype(dtype)


def scaled_window(codes, scales, d, x):
    """out[t] = W . x[t] with W = scaled_floats (float64 sums); x (tokens, cols) -> (tokens, rows) float64."""
    return np.asarray(x, dtype=np.float64) @ scaled_floats(codes, scales, d).astype(np.float64).T


def q3k_planes(blocks, rows, cols):
    """A Q3_K tensor's blocks (hmask 32 bytes, qs 64, scales 12, d float16 at 108) as planes: hm (8 little-endian
    words a block), qs (16 words), sc (16 int8: scale k's low four bits from byte k % 8 (>> 4 from the second
    group of eight), its two high bits from byte 8 + k % 4 at 2 (k / 4), less 32) and dd (float16)."""
    b = np.asarray(blocks, dtype=np.uint8).reshape(-1, 110)
    s = b[:, 96:108].astype(np.int16)
    sc = np.empty((b.shape[0], 16), dtype=np.int16)
    for k in range(16):
        low = (s[:, k] & 15) if k < 8 else (s[:, k - 8] >> 4)
        high = (s[:, 8 + k % 4] >> (2 * (k // 4))) & 3
        sc[:, k] = (low | (high << 4)) - 32
    return {"hm": np.ascontiguousarray(b[:, 0:32]).reshape(-1).view("<u4"),
            "qs": np.ascontiguousarray(b[:, 32:96]).reshape(-1).view("<u4"),
            "sc": sc.astype(np.int8).reshape(-1),
            "dd": _half(b, 108)}


def q3k_planes_weights(planes, rows, cols):
    """The float32 weights the planes hold: weight 128 n + 32 j + i of a block is (d sc[2 (4 n + j) + i / 16]) times
    the two bits of qs byte 32 n + i at 2 j, less 4 where bit 4 n + j of hm byte i is clear."""
    hm = np.asarray(planes["hm"]).view(np.uint8).reshape(-1, 32)
    qs = np.asarray(planes["qs"]).view(np.uint8).reshape(-1, 64)
    sc = np.asarray(planes["sc"]).reshape(-1, 16).astype(np.float32)
    dd = np.asarray(planes["dd"]).astype(np.float32).reshape(-1, 1)
    w = np.empty((hm.shape[0], 256), dtype=np.float32)
    i = np.arange(32)
    for n in range(2):
        for j in range(4):
            rr = 4 * n + j
            v = ((qs[:, 32 * n + i] >> (2 * j)) & 3).astype(np.int16) - np.where((hm[:, i] >> rr) & 1, 0, 4)
            scale = (dd * sc[:, 2 * rr + (i >= 16)]).astype(np.float32)
            w[:, 128 * n + 32 * j + i] = (scale * v.astype(np.float32)).astype(np.float32)
    return w.reshape(rows, cols)


def hyper_connection(before, out, inject_in, norm, down, up, inject_w, hc, eps=1e-6, dtype=np.float16):
    """FusedResidual.__call__ (strata_mlx/fused.py:307-323) for before (T, hc d), out (T, d), inject_in (T, hc):
    residual = before + out * inject_in (rounded to the type); per stream normed = h / sqrt(mean h^2 + eps) * norm
    (float64 here); total_j = row_j . normed / hc; low = total sigmoid(total) for rows of `down`, inject =
    2 sigmoid(total) (rounded) for rows of `inject_w`; mixed[c] = sum_s normed[s d + c] sigmoid(up[s d + c] . low)
    / hc (rounded). Returns (mixed, residual, inject or None)."""
    T, d = out.shape
    f = lambda a: np.asarray(a, dtype=np.float64)  # noqa: E731
    h = f(before).reshape(T, hc, d) + f(out)[:, None, :] * f(inject_in)[:, :, None]
    residual = h.reshape(T, hc * d).astype(dtype)
    scale = 1.0 / np.sqrt((h * h).mean(axis=2, keepdims=True) + eps)
    normed = (h * scale).reshape(T, hc * d) * f(norm)[None, :]
    sig = lambda z: 1.0 / (1.0 + np.exp(-z))  # noqa: E731
    total = normed @ f(down).T / hc
    low = total * sig(total)
    inject = None
    if inject_w is not None:
        inject = (2.0 * sig(normed @ f(inject_w).T / hc)).astype(dtype)
    gate = low @ f(up).T  # (T, hc d)
    mixed = (normed * sig(gate)).reshape(T, hc, d).sum(axis=1) / hc
    return mixed.astype(dtype), residual, inject
