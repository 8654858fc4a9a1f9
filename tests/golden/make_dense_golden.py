"""Writes tests/golden/dense.npz: the reference's own Q6_K parts and Q3_K planes of seeded random blocks.

Run once, in a container that has the reference checkout (its path is the first argument, or the
STRATA_MLX_REFERENCE environment variable):

    python tests/golden/make_dense_golden.py [/path/to/strata-mlx]

  - `q6k_parts` (strata_mlx/gguf.py:150-165) is numpy code in a module that imports numpy only: it runs as is.
  - `q3k_planes` (strata_mlx/blocks.py:403-414) is numpy code in a module that imports MLX at its top, which is
    absent here: the function's own source is taken from the file (Python's ast) and run with `mx.array` standing
    for numpy's asarray, the one MLX name it uses (it wraps each plane as it returns it).

The blocks are uniform random bytes with their float16 d fields drawn from uniform(-0.05, 0.05), and a zero and
a negative d, as the block fixture's generator makes them.
"""

import ast
import os
import sys
import types

import numpy as np

ROWS, COLS = 4, 2560


def _q3k_planes_of(ref_root):
    path = os.path.join(ref_root, "strata_mlx", "blocks.py")
    tree = ast.parse(open(path).read())
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "q3k_planes")
    mod = ast.Module(body=[fn], type_ignores=[])
    shim = types.SimpleNamespace(array=np.asarray)
    scope = {"np": np, "mx": shim}
    exec(compile(mod, path, "exec"), scope)
    return scope["q3k_planes"]


def main(ref_root):
    sys.path.insert(0, ref_root)
    from strata_mlx import gguf as ref  # numpy only

    q3k_planes = _q3k_planes_of(ref_root)
    rng = np.random.default_rng(20261202)
    out = {}
    for kind, nbytes, d_at in (("Q6_K", 210, 208), ("Q3_K", 110, 108)):
        n = ROWS * COLS // 256
        b = rng.integers(0, 256, (n, nbytes), dtype=np.uint8)
        d = rng.uniform(-0.05, 0.05, n)
        d[0], d[1] = 0.0, -0.031
        b[:, d_at : d_at + 2] = d.astype("<f2").reshape(-1, 1).view(np.uint8)
        flat = b.reshape(-1)
        out[f"{kind}/blocks"] = flat
        if kind == "Q6_K":
            codes, scales, dd = ref.q6k_parts(ref.Tensor(kind, (ROWS, COLS), kind, flat))
            out["Q6_K/codes"], out["Q6_K/scales"] = np.asarray(codes), np.asarray(scales)
            out["Q6_K/d"] = np.asarray(dd).view(np.uint16)
        else:
            planes = q3k_planes(flat, ROWS, COLS)
            for name in ("hm", "qs", "sc", "dd"):
                a = np.asarray(planes[name])
                out[f"Q3_K/{name}"] = a.view(np.uint16) if name == "dd" else a
        print(f"{kind}: {n} blocks")
    out["shape"] = np.array([ROWS, COLS])
    np.savez_compressed(os.path.join(os.path.dirname(os.path.abspath(__file__)), "dense.npz"), **out)


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("STRATA_MLX_REFERENCE")
    if not ref:
        sys.exit("usage: make_dense_golden.py /path/to/strata-mlx (or set STRATA_MLX_REFERENCE)")
    main(ref)
