"""Writes tests/golden/blocks.npz: block bytes of every type with the weights the reference's decoders give.

Run once, in a container that has the reference checkout (its path is the first argument, or the
STRATA_MLX_REFERENCE environment variable) and gguf-py 0.19.0, the decoder version the reference pins
(`uv.lock:135-136`):

    python tests/golden/make_golden.py [/path/to/strata-mlx]

For every type the expected float32 weights come from gguf-py's `quants.dequantize` (what the reference's
`tests/test_blocks.py:18-24` holds its kernels to). Where the reference has a CPU decoder of its own
(`strata_mlx/gguf.py`: `to_affine` for Q8_0, Q4_K, Q5_K, Q3_K, IQ4_NL, IQ4_XS, IQ3_S, Q2_0; `to_float` for
Q6_K) this script also runs it, expands its codes * scales + biases the way the reference's test does
(`tests/test_gguf.py:48-55`), and refuses to write the fixture unless the two agree bit for bit. Q2_0 has
no gguf-py decoder; its expected weights are the reference test's own restatement (`tests/test_gguf.py:34-38`).

The blocks are uniform random bytes with the float16 scale fields drawn from uniform(-0.05, 0.05) as in
`tests/test_gguf.py:17-30`, plus edge blocks: a zero scale, a negative one, and scales large enough that
weights overflow float16 (so the fixture's float16 bits pin the round-to-nearest-even overflow to inf).
"""

import os
import sys

import numpy as np

ROWS, COLS = 3, 2560
KINDS = ["Q8_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "IQ3_XXS", "IQ3_S", "IQ4_XS",
         "IQ4_NL", "IQ2_XXS", "IQ2_XS", "IQ2_S", "IQ1_M", "Q2_0"]


def main(ref_root):
    import gguf

    sys.path.insert(0, ref_root)
    from strata_mlx import gguf as ref  # the reference's own numpy decoders (imports numpy only)

    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.dirname(os.path.dirname(here)))
    from oracle.quants import SCALE_BYTES, TYPES

    out = {}
    rng = np.random.default_rng(20261201)
    for kind in KINDS:
        _, per_block, block_bytes = TYPES[kind]
        n = ROWS * COLS // per_block
        b = rng.integers(0, 256, (n, block_bytes), dtype=np.uint8)
        scales = rng.uniform(-0.05, 0.05, n)
        scales[0], scales[1], scales[2] = 0.0, -0.031, 900.0 if kind not in ("IQ1_M",) else 60000.0
        for at in SCALE_BYTES[kind]:
            b[:, at : at + 2] = scales.astype("<f2").reshape(-1, 1).view(np.uint8)
        if kind == "IQ1_M":
            d = scales.astype("<f2").view("<u2")
            words = b[:, 48:56].copy().view("<u2")
            for i in range(4):
                words[:, i] = (words[:, i] & 0x0FFF) | (((d >> (4 * i)) & 15) << 12)
            b[:, 48:56] = words.view(np.uint8)
        flat = b.reshape(-1)
        if kind == "Q2_0":
            code = np.stack([(b[:, 2:] >> s) & 3 for s in (0, 2, 4, 6)], axis=2).reshape(-1, 64)
            want = ((code.astype(np.float32) - 1) * b[:, :2].copy().view("<f2").astype(np.float32))
        else:
            qtype = getattr(gguf.GGMLQuantizationType, kind)
            want = gguf.quants.dequantize(flat.reshape(ROWS, -1), qtype)
        want = np.asarray(want, dtype=np.float32).reshape(ROWS, COLS)

        t = ref.Tensor(kind, (ROWS, COLS), kind, flat)
        checked = "gguf-py"
        if kind == "Q6_K":
            theirs = ref.to_float(t)
            checked += "+reference.to_float"
        elif kind in ("Q8_0", "Q4_K", "Q5_K", "Q3_K", "IQ4_NL", "IQ4_XS", "IQ3_S", "Q2_0"):
            a = ref.to_affine(t)
            theirs = (a.codes.astype(np.float32) * np.repeat(a.scales, a.group, -1)
                      + np.repeat(a.biases, a.group, -1))
            checked += "+reference.to_affine"
        else:
            theirs = want
        # to_affine's expansion code*scale+bias rounds twice; the reference's own test allows 1e-6 of the
        # largest weight (tests/test_gguf.py:43-45), and the float16 images must agree as values (a zero scale
        # gives -0 in gguf-py's product and +0 in the affine sum)
        tol = 1e-6 * np.abs(want[np.isfinite(want)]).max()
        finite = np.isfinite(want)
        assert np.abs(theirs[finite] - want[finite]).max() <= tol, kind
        with np.errstate(over="ignore"):
            assert np.array_equal(theirs.astype(np.float16)[finite], want.astype(np.float16)[finite]), kind
        out[f"{kind}/blocks"] = flat
        out[f"{kind}/f32"] = want
        with np.errstate(over="ignore"):
            out[f"{kind}/f16"] = want.astype(np.float16).view(np.uint16)
        print(f"{kind:8s} {n:3d} blocks  checked by {checked}")
    out["shape"] = np.array([ROWS, COLS])
    np.savez_compressed(os.path.join(here, "blocks.npz"), **out)


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("STRATA_MLX_REFERENCE")
    if not ref:
        sys.exit("usage: make_golden.py /path/to/strata-mlx (or set STRATA_MLX_REFERENCE)")
    main(ref)
