"""CPU oracle for the MoE hot path: TEST INFRASTRUCTURE ONLY.

A plain numpy restatement of strata-mlx's block decoders and MoE-block arithmetic, used as the checker for
the CUDA path. Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline leg may import it;
the product package (`strata_mlx_b200`) never does, and fails loudly when its CUDA library is missing.

Parity pin: `tests/golden/*.npz` hold block bytes with the weights that gguf-py 0.19.0 (the reference's
pinned decoder, `uv.lock:135-136`) and the reference's own `strata_mlx/gguf.py:to_affine`/`to_float` give
for them; `tests/test_oracle.py` checks this module against those fixtures bit for bit.
"""
