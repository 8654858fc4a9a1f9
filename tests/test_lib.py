"""The C-ABI library: it loads, it exports every symbol include/strata_moe.h declares, and its host-side argument
checks answer without touching a GPU. No GPU needed."""

import ctypes
import os
import re

import pytest

from strata_mlx_b200 import _lib, blocks

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "strata_moe.h")


def declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"SMOE_API\s+[\w\s\*]+?\b(smoe_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(_lib.LIB_PATH):
        from strata_mlx_b200 import _build

        _build.build()
    return _lib.lib()


def test_header_declares_the_entry_points():
    names = declared()
    assert "smoe_tile_matmul" in names and "smoe_matvec" in names and len(names) >= 17


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing
    assert set(declared()) <= set(_lib.SIGNATURES)  # and the binding knows every one


def test_library_was_built_for_sm100a(lib):
    assert lib.smoe_built_arch() == 1000
    assert lib.smoe_version() >= 1


def test_block_table_matches_the_python_one(lib):
    for name, (per, nbytes) in blocks.BLOCK.items():
        p, b = ctypes.c_int(), ctypes.c_int()
        assert lib.smoe_block_info(blocks.KIND_ID[name], ctypes.byref(p), ctypes.byref(b)) == 0
        assert (p.value, b.value) == (per, nbytes), name
    assert lib.smoe_block_info(99, None, None) == 1  # SMOE_EKIND
    assert b"99" in lib.smoe_last_error()


def test_what_fits_in_tiles(lib):
    """tests/test_blocks.py:214-217 of the reference."""
    assert blocks.tileable("Q2_0", 640, 2560) and blocks.tileable("IQ3_S", 640, 2560)
    assert blocks.tileable("IQ4_NL", 2560, 640)
    assert not blocks.tileable("IQ3_S", 2560, 640)
    assert not blocks.tileable("Q2_0", 2, 2560)


def test_invalid_arguments_are_rejected_on_the_host(lib):
    # a shape that does not end on a block, an unknown type, a missing workspace: errors before any launch
    assert lib.smoe_dequant(21, None, 4, 100, None, 1, None) == 2  # SMOE_ESHAPE (100 % 256)
    assert lib.smoe_matvec(77, None, 1, 1, 256, None, 1, 1, None, None, 1, None) in (1, 4)
    assert lib.smoe_tiles_of(ctypes.c_void_p(16), 32, 2, 8, ctypes.c_void_p(16), ctypes.c_void_p(16),
                             ctypes.c_void_p(16), None, 0, None) == 5  # SMOE_EWORKSPACE
    assert lib.smoe_top_k(ctypes.c_void_p(16), 1, 4096, 8, ctypes.c_void_p(16), None, None) == 2
    v = ctypes.c_void_p(16)
    assert lib.smoe_route(v, None, v, 1, 1, 256, 512, 8, v, v, v, None, None, None) == 4  # no counters
    assert lib.smoe_route(v, v, v, 1, 1, 256, 512, 8, v, v, v, None, v, None) == 4  # gate weight, no output
    assert lib.smoe_route(v, None, v, 1, 1, 4096, 512, 8, v, v, v, None, v, None) == 2  # too many experts
    assert lib.smoe_route_counters(20) == 12
    # the fused route step: its counters hold two words before smoe_route's, and it checks its arguments first
    assert lib.smoe_route_step_counters(1) == 16 and lib.smoe_route_step_counters(20) == 32
    assert lib.smoe_route_matvec_batch(None, 0, None, None) == 4  # null route
    step = _lib.SmoeRouteStep(16, None, 16, 1, 1, 256, 512, 8, 16, 16, 16, None, 16, 200, 100, 16)
    assert lib.smoe_route_matvec_batch(ctypes.byref(step), 0, None, None) == 4  # [lo, lo + count) past the experts
    step.tokens = -1
    assert lib.smoe_route_matvec_batch(ctypes.byref(step), 0, None, None) == 4  # negative token count
    step.tokens = 0
    assert lib.smoe_route_matvec_batch(ctypes.byref(step), 0, None, None) == 0  # nothing to do
    with pytest.raises(ValueError):
        _lib.call("smoe_dequant", 21, None, 4, 100, None, 1, None)


def test_workspace_queries(lib):
    assert lib.smoe_tiles_of_workspace_size(9440, 256) >= 9440 * 4
    assert lib.smoe_tile_matmul_workspace_size(16 * 850) >= 850 * 16


def test_no_cpu_path(lib):
    torch = pytest.importorskip("torch")
    x = torch.zeros(4, 256, dtype=torch.uint8)
    with pytest.raises(ValueError, match="CUDA"):
        blocks.dequantize(x.reshape(-1), "IQ3_S", (4 * 256 // 110 * 0 + 1, 256))
