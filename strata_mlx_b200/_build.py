"""Builds libstrata_moe.so in-tree from csrc/*.cu with nvcc for sm_100a (no GPU needed).

    python -m strata_mlx_b200._build [--force]

The codebook tables header is generated first from gguf-py (csrc/gen_tables.py). Objects go to
strata_mlx_b200/_build/, the library to strata_mlx_b200/libstrata_moe.so.
"""

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libstrata_moe.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-DSMOE_ARCH=1000", "--expt-relaxed-constexpr",
         "-Xcompiler", "-fvisibility=hidden"]


def _sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _newest_input():
    paths = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh", ".py"))]
    paths.append(os.path.join(HERE, "..", "include", "strata_moe.h"))
    paths.append(os.path.abspath(__file__))
    return max(os.path.getmtime(p) for p in paths if os.path.exists(p))


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every CUDA source and link the library; skipped when it is newer than all inputs."""
    sys.path.insert(0, CSRC)
    try:
        import gen_tables

        gen_tables.main(os.path.join(CSRC, "_tables.cuh"))
    finally:
        sys.path.pop(0)
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= _newest_input():
        return LIB
    os.makedirs(OBJ, exist_ok=True)

    def compile_one(src):
        obj = os.path.join(OBJ, src[:-3] + ".o")
        cmd = [NVCC, *ARCH, *FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stderr}")
        return obj, r.stderr

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        results = list(pool.map(compile_one, _sources()))
    if verbose:
        for _, err in results:
            sys.stderr.write(err)
    tmp = LIB + ".tmp"
    cmd = [NVCC, *ARCH, "-shared", "-o", tmp, *[o for o, _ in results], "-Xcompiler", "-fPIC"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
