"""strata_mlx_b200: strata-mlx's mixture-of-experts hot path on GGUF quant blocks, built for B200 (sm_100a).

`blocks` and `fused` keep the call surface of the reference's `strata_mlx.blocks` / `strata_mlx.fused`;
the kernels live in libstrata_moe.so (C ABI: include/strata_moe.h), built by `strata_mlx_b200._build`.
"""

from . import blocks, fused  # noqa: F401
