"""ctypes binding of libstrata_moe.so, the C ABI declared in include/strata_moe.h.

The library is built in-tree (`python -m strata_mlx_b200._build`) and loaded from this package's directory.
There is no fallback: if it is missing or fails to load, every entry point of the package raises.
"""

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libstrata_moe.so")

F32, F16 = 0, 1
ETIMEOUT = 6

_c = ctypes
_p, _i, _i64, _sz = _c.c_void_p, _c.c_int, _c.c_int64, _c.c_size_t



class SmoeMatvec(ctypes.Structure):
    """`SmoeMatvec` of include/strata_moe.h: one problem of smoe_matvec_batch."""

    _fields_ = [("kind", _i), ("blocks", _p), ("experts", _i64), ("rows", _i64), ("cols", _i64), ("idx", _p),
                ("pairs", _i64), ("share", _i64), ("x", _p), ("gate", _p), ("up", _p), ("out", _p), ("dtype", _i)]


class SmoeRouteStep(ctypes.Structure):
    """`SmoeRouteStep` of include/strata_moe.h: a decode step's route for smoe_route_matvec_batch."""

    _fields_ = [("weight", _p), ("gate_weight", _p), ("x", _p), ("x_dtype", _i), ("tokens", _i64), ("experts", _i64),
                ("hidden", _i64), ("k", _i64), ("logits", _p), ("idx", _p), ("weights", _p), ("gate_out", _p),
                ("counters", _p), ("lo", _i64), ("count", _i64), ("lidx", _p)]


class SmoeDecodeLayer(ctypes.Structure):
    """`SmoeDecodeLayer` of include/strata_moe.h: one MoE block for smoe_decode_layer."""

    _fields_ = [("router", _p), ("shared_gate", _p), ("experts", _i64), ("hidden", _i64), ("k", _i64), ("kind", _i),
                ("gate", _p), ("up", _p), ("down", _p), ("ffn", _i64), ("shared_kind", _i), ("sgate", _p),
                ("sup", _p), ("sdown", _p), ("sffn", _i64), ("logits", _p), ("idx", _p), ("weights", _p),
                ("gate_out", _p), ("out", _p), ("scratch", _p)]


class SmoeEpReduce(ctypes.Structure):
    """`SmoeEpReduce` of include/strata_moe.h: one rank's call of smoe_ep_reduce_combine."""

    _fields_ = [("rank", _i), ("ranks", _i), ("peers", _p * 16), ("y", _p), ("w", _p), ("lidx", _p),
                ("experts", _i64), ("s", _p), ("g", _p), ("tokens", _i64), ("k", _i64), ("d", _i64),
                ("capacity", _i64), ("out", _p), ("dtype", _i), ("wait_polls", _c.c_uint32)]


class SmoeHyper(ctypes.Structure):
    """`SmoeHyper` of include/strata_moe.h: a hyper-connection's weights and sizes."""

    _fields_ = [("norm", _p), ("down", _p), ("up", _p), ("inject_w", _p), ("hc", _i64), ("d", _i64), ("rank", _i64),
                ("eps", _c.c_float), ("dtype", _i)]


# name -> (restype, argtypes): the declarations of include/strata_moe.h
SIGNATURES = {
    "smoe_last_error": (_c.c_char_p, []),
    "smoe_version": (_i, []),
    "smoe_built_arch": (_i, []),
    "smoe_block_info": (_i, [_i, _c.POINTER(_i), _c.POINTER(_i)]),
    "smoe_dequant": (_i, [_i, _p, _i64, _i64, _p, _i, _p]),
    "smoe_matvec": (_i, [_i, _p, _i64, _i64, _i64, _p, _i64, _i64, _p, _p, _i, _p]),
    "smoe_matvec_gate_up": (_i, [_i, _p, _i, _p, _i64, _i64, _i64, _p, _i64, _i64, _p, _p, _p, _i, _p]),
    "smoe_matvec_glu": (_i, [_i, _p, _i64, _i64, _i64, _p, _i64, _p, _p, _p, _i, _p]),
    "smoe_matvec_batch": (_i, [_i, _c.POINTER(SmoeMatvec), _p]),
    "smoe_matvec_status": (_i, [_c.POINTER(_i), _i]),
    "smoe_matvec_wait_test": (_i, [_i64, _i]),
    "smoe_matvec_glu_combine": (_i, [_i, _p, _i64, _i64, _p, _i64, _p, _p, _p, _p, _p, _i64, _p, _i, _p]),
    "smoe_decode_layer_scratch": (_sz, [_i64, _i64, _i64, _i64]),
    "smoe_decode_layer": (_i, [_c.POINTER(SmoeDecodeLayer), _p, _p]),
    "smoe_decode_layer_status": (_i, [_p, _i64, _i64, _i64, _i64, _c.POINTER(_i)]),
    "smoe_decode_layer_wait_test": (_i, [_i]),
    "smoe_swiglu": (_i, [_p, _p, _i64, _p, _i, _p]),
    "smoe_swiglu_to": (_i, [_p, _p, _i64, _i, _p, _i, _p]),
    "smoe_router_logits": (_i, [_p, _p, _i, _i64, _i64, _i64, _p, _p]),
    "smoe_top_k": (_i, [_p, _i64, _i64, _i64, _p, _p, _p]),
    "smoe_combine": (_i, [_p, _p, _p, _p, _i64, _i64, _i64, _p, _i, _p]),
    "smoe_route_counters": (_sz, [_i64]),
    "smoe_route_step_counters": (_sz, [_i64]),
    "smoe_route_matvec_batch": (_i, [_c.POINTER(SmoeRouteStep), _i, _c.POINTER(SmoeMatvec), _p]),
    "smoe_route": (_i, [_p, _p, _p, _i, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _p]),
    "smoe_route_local": (_i, [_p, _p, _p, _i, _i64, _i64, _i64, _i64, _p, _p, _p, _p, _p, _i64, _i64, _p, _p]),
    "smoe_localize": (_i, [_p, _i64, _i64, _i64, _p, _p]),
    "smoe_partial_sums": (_i, [_p, _p, _p, _i64, _p, _i64, _i64, _i64, _p, _i, _p]),
    "smoe_combine_sums": (_i, [_p, _p, _i64, _i64, _p, _i, _p]),
    "smoe_ep_exchange_bytes": (_sz, [_i64, _i64, _i64]),
    "smoe_ep_exchange_alloc": (_i, [_sz, _c.POINTER(_p), _p]),
    "smoe_ep_exchange_open": (_i, [_p, _c.POINTER(_p)]),
    "smoe_ep_exchange_close": (_i, [_p]),
    "smoe_ep_exchange_free": (_i, [_p]),
    "smoe_ep_exchange_status": (_i, [_p, _c.POINTER(_i), _i]),
    "smoe_ep_reduce_combine": (_i, [_c.POINTER(SmoeEpReduce), _p]),
    "smoe_ep_reduce_combine_emulated": (_i, [_i, _c.POINTER(SmoeEpReduce), _p]),
    "smoe_ep_dispatch": (_i, [_p, _i64, _i64, _i64, _i64, _p, _i64, _i, _p, _p, _p, _p, _p]),
    "smoe_combine_rows": (_i, [_p, _p, _p, _p, _p, _i64, _i64, _i64, _p, _i, _p]),
    "smoe_hyper_workspace_size": (_sz, [_i64, _i64, _i64, _i64]),
    "smoe_hyper_connection": (_i, [_c.POINTER(SmoeHyper), _p, _p, _p, _i64, _p, _p, _p, _p, _sz, _p]),
    "smoe_q3k_planes": (_i, [_p, _i64, _i64, _p, _p, _p, _p, _p]),
    "smoe_q3k_planes_window": (_i, [_p, _p, _p, _p, _i64, _i64, _p, _i64, _p, _i, _p]),
    "smoe_q3k_planes_dequant": (_i, [_p, _p, _p, _p, _i64, _i64, _p, _i, _p]),
    "smoe_q6k_parts": (_i, [_p, _i64, _i64, _p, _p, _p, _p]),
    "smoe_scaled_window": (_i, [_p, _p, _p, _i64, _i64, _i64, _p, _i64, _p, _i, _p]),
    "smoe_scaled_floats": (_i, [_p, _p, _p, _i64, _i64, _i64, _p, _i, _p]),
    "smoe_tiles_of_workspace_size": (_sz, [_i64, _i64]),
    "smoe_tiles_of": (_i, [_p, _i64, _i64, _i64, _p, _p, _p, _p, _sz, _p]),
    "smoe_tiles_of_noalloc": (_i, [_p, _i64, _i64, _i64, _p, _p, _p, _p]),
    "smoe_tileable": (_i, [_i, _i64, _i64]),
    "smoe_tile_matmul_workspace_size": (_sz, [_i64]),
    "smoe_tile_matmul": (_i, [_i, _p, _i64, _i64, _i64, _p, _i, _i64, _p, _p, _p, _sz, _p]),
    "smoe_tile_matmul_rows": (_i, [_i, _p, _i64, _i64, _i64, _p, _i64, _i64, _p, _p, _i64, _p, _p, _sz, _p]),
    "smoe_slot_rows": (_i, [_p, _i64, _i64, _p, _p]),
    "smoe_tile_matmul_pair": (_i, [_i, _p, _p, _i64, _i64, _i64, _p, _i64, _p, _p, _p, _p, _sz, _p]),
    "smoe_tile_matmul_pair_rows": (_i, [_i, _p, _p, _i64, _i64, _i64, _p, _i64, _i64, _p, _p, _i64, _p, _p, _p, _sz,
                                        _p]),
}

_lib = None

# kernels each entry point launches (for the benchmark's launch count); 1 where not named
KERNELS_PER_CALL = {"smoe_tiles_of": 2, "smoe_tiles_of_noalloc": 2, "smoe_tile_matmul": 2, "smoe_tile_matmul_rows": 2,
                    "smoe_tile_matmul_pair": 2, "smoe_tile_matmul_pair_rows": 2, "smoe_ep_dispatch": 2,
                    "smoe_ep_exchange_alloc": 0, "smoe_ep_exchange_open": 0, "smoe_ep_exchange_close": 0,
                    "smoe_ep_exchange_free": 0, "smoe_ep_exchange_status": 0, "smoe_decode_layer_status": 0, "smoe_decode_layer_wait_test": 0,
                    "smoe_matvec_status": 0, "smoe_matvec_wait_test": 0, "smoe_hyper_connection": 3}
launches = 0


def lib():
    """The loaded library (loaded once). Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m strata_mlx_b200._build` "
                               "(there is no CPU fallback)")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype, fn.argtypes = res, args
        _lib = handle
    return _lib


def call(name, *args):
    """Call an entry point; a non-zero status raises ValueError (invalid argument) or RuntimeError (CUDA)."""
    global launches
    status = getattr(lib(), name)(*args)
    launches += KERNELS_PER_CALL.get(name, 1)
    if status != 0:
        msg = lib().smoe_last_error().decode(errors="replace")
        if status > 0:
            raise ValueError(f"{name}: {msg}")
        raise RuntimeError(f"{name}: {msg}")


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def dtype_code(dt) -> int:
    if dt == torch.float16:
        return F16
    if dt == torch.float32:
        return F32
    raise ValueError(f"activations of {dt} are not supported (float16 or float32)")


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("strata_mlx_b200 computes on CUDA tensors only (no CPU path)")
