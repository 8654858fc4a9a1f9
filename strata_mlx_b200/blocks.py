"""Mixture-of-experts products read straight from GGUF quant blocks on B200, behind the Python interface of
strata-mlx's `strata_mlx/blocks.py`.

Each stack of experts lives on the GPU as one uint8 tensor holding the file's bytes unchanged; hand-written
sm_100a kernels (libstrata_moe.so, C ABI in include/strata_moe.h) decode the blocks as they multiply:

    matvec      decode steps: each (token, expert) pair's rows dotted with its activation row
    matvec_glu  the down product of a few pairs, SwiGLU of (gate, up) formed while the activations are split
    tiles       a prompt chunk: pairs grouped by expert into 16-slot tiles (`tiles_of`), then one tensor-core
                grouped GEMM (tcgen05, accumulators in TMEM) per run of an expert's tiles (`tile_matmul`)
    dequant     a stack's weights expanded to float16 or float32

Names, signatures, tensor layouts, thresholds and the "None = path not taken" convention follow the
reference (strata_mlx/blocks.py), so an engine written against it can import this module instead. Tensors
are torch CUDA tensors; there is no CPU path and no fallback to another library's kernels.
"""

import ctypes
import math

import torch

from . import _lib

# GGML type name -> (weights a block holds, its size in bytes): the format constants of the reference's BLOCK
# (strata_mlx/blocks.py:36-38), extended by the K-types and Q8_0 this build also decodes on the GPU
# (strata_mlx/gguf.py:25-33)
BLOCK = {"IQ4_NL": (32, 18), "IQ4_XS": (256, 136), "IQ3_S": (256, 110), "IQ3_XXS": (256, 98),
         "IQ2_S": (256, 82), "IQ2_XS": (256, 74), "IQ2_XXS": (256, 66), "IQ1_M": (256, 56), "Q2_0": (64, 18),
         "Q3_K": (256, 110), "Q8_0": (32, 34), "Q2_K": (256, 84), "Q4_K": (256, 144), "Q5_K": (256, 176),
         "Q6_K": (256, 210)}
# GGML type ids, the `kind` of the C ABI
KIND_ID = {"Q8_0": 8, "Q2_K": 10, "Q3_K": 11, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "IQ2_XXS": 16, "IQ2_XS": 17,
           "IQ3_XXS": 18, "IQ4_NL": 20, "IQ3_S": 21, "IQ2_S": 22, "IQ4_XS": 23, "IQ1_M": 29, "Q2_0": 42}

# thresholds, module attributes as in the reference so that tests and engines can switch paths
TILES_FROM = 1600  # a call with at least this many (token, expert) pairs takes the tile path (strata_mlx/blocks.py:579)
TOKENS_TILE, ROWS_TILE, COLS_TILE = 16, 64, 64  # strata_mlx/blocks.py:580
BLOCK_GLU = True  # pairs unsorted, swiglu formed by the down kernel (strata_mlx/blocks.py:934)
MATVEC_GLU_UPTO = 30  # pairs up to which down forms swiglu itself (strata_mlx/blocks.py:936)
# pairs up to which a step of the block runs as the fused decode products (decode_products): the int8 down
# kernel forms swiglu itself at any pair count, so this is not the reference's MATVEC_GLU_UPTO
DECODE_UPTO = 256


def _kind(kind: str) -> int:
    if kind not in KIND_ID:
        raise ValueError(f"{kind} blocks are not supported")
    return KIND_ID[kind]


def row_bytes(kind: str, cols: int) -> int:
    per_block, block_bytes = BLOCK[kind]
    if cols % per_block:
        raise ValueError(f"{kind}: {cols} columns is not a whole number of {per_block}-weight blocks")
    return cols // per_block * block_bytes


def window_matvec(blocks: torch.Tensor, kind: str, rows: int, cols: int, x: torch.Tensor,
                  per_row: int | None = None) -> torch.Tensor:
    """The dense product of a verify window: every token of x (tokens, cols) times one layer's block matrix
    (rows, cols), giving (tokens, rows) in x's type (strata_mlx/blocks.py:349-396). On the CUDA-core
    kernels (the K-types, IQ3_XXS, IQ4_XS, the IQ2 / IQ1 types) a token gets the same bits as alone, whatever the
    window; on the int8 tensor-core kernel (IQ3_S, Q8_0) its integer sums are exact but the float32 partial sums
    of a row may be grouped over a different number of warps for another window, so a token's result can differ
    from its result alone in the last bits (the reference keeps the bits, strata_mlx/blocks.py:350, 485-486).
    `per_row` is the reference's threads-per-row hint and changes nothing here."""
    _lib.require_cuda(blocks, x)
    stack = BlockSwitchLinear(blocks, kind, (1, rows, cols))
    x2 = x.reshape(-1, cols).contiguous()
    return _matvec(stack, x2, _zeros_idx(x2.shape[0], x.device), 1, x.dtype)


# ---- Q3_K as planes: each field of the 110-byte blocks gathered into its own word-aligned array once, the
# weights unchanged, so the kernels load whole words; 114 bytes per block (strata_mlx/blocks.py:399-401)
Q3K_PLANE_BYTES = 114


def q3k_planes(blocks: torch.Tensor, rows: int, cols: int) -> dict:
    """Split a Q3_K matrix (rows, cols) into its planes on the GPU: {hm: high-bit masks, 8 words per block;
    qs: two-bit codes, 16 words; sc: the sixteen 6-bit scales minus 32, as int8; dd: the float16 d}
    (strata_mlx/blocks.py:403-414)."""
    _lib.require_cuda(blocks)
    if cols % 256 or blocks.numel() != rows * row_bytes("Q3_K", cols):
        raise ValueError(f"{blocks.numel()} bytes do not hold a Q3_K tensor of ({rows}, {cols})")
    n = rows * (cols // 256)
    dev = blocks.device
    planes = {"hm": torch.empty(n * 8, dtype=torch.int32, device=dev), "qs": torch.empty(n * 16, dtype=torch.int32, device=dev),
              "sc": torch.empty(n * 16, dtype=torch.int8, device=dev), "dd": torch.empty(n, dtype=torch.float16, device=dev)}
    _lib.call("smoe_q3k_planes", _lib.ptr(blocks.reshape(-1).contiguous()), rows, cols, _lib.ptr(planes["hm"]),
              _lib.ptr(planes["qs"]), _lib.ptr(planes["sc"]), _lib.ptr(planes["dd"]), _lib.stream())
    return planes


def q3k_planes_window(planes: dict, rows: int, cols: int, x: torch.Tensor) -> torch.Tensor:
    """Multiply a window of tokens x (tokens, cols) by a Q3_K matrix kept as planes; (tokens, rows) in x's type
    (strata_mlx/blocks.py:482-499). The split of a row's sum across lanes depends on the matrix's shape only, so
    each token's result has the same bits whether it comes alone or with others."""
    _lib.require_cuda(x, *planes.values())
    x2 = x.reshape(-1, cols).contiguous()
    out = torch.empty((x2.shape[0], rows), dtype=x.dtype, device=x.device)
    if x2.shape[0]:
        _lib.call("smoe_q3k_planes_window", _lib.ptr(planes["hm"]), _lib.ptr(planes["qs"]), _lib.ptr(planes["sc"]),
                  _lib.ptr(planes["dd"]), rows, cols, _lib.ptr(x2), x2.shape[0], _lib.ptr(out),
                  _lib.dtype_code(x.dtype), _lib.stream())
    return out


def q3k_planes_dequantize(planes: dict, rows: int, cols: int, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Expand a Q3_K matrix kept as planes to floats (rows, cols), with the same bits the block decoder gives
    (blocks.py:502-512)."""
    _lib.require_cuda(*planes.values())
    out = torch.empty((rows, cols), dtype=dtype, device=planes["dd"].device)
    _lib.call("smoe_q3k_planes_dequant", _lib.ptr(planes["hm"]), _lib.ptr(planes["qs"]), _lib.ptr(planes["sc"]),
              _lib.ptr(planes["dd"]), rows, cols, _lib.ptr(out), _lib.dtype_code(dtype), _lib.stream())
    return out


def dequantize(blocks: torch.Tensor, kind: str, shape: tuple, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Expand a block tensor to floats: `blocks` are the file's uint8 bytes of a tensor whose logical shape is
    `shape` (strata_mlx/blocks.py:515-522). A float16 result is gguf-py's float32 weight rounded once."""
    _lib.require_cuda(blocks)
    *lead, rows, cols = shape
    n = math.prod(lead) if lead else 1
    if blocks.numel() != n * rows * row_bytes(kind, cols):
        raise ValueError(f"{blocks.numel()} bytes do not hold a {kind} tensor of {tuple(shape)}")
    out = torch.empty(tuple(shape), dtype=dtype, device=blocks.device)
    _lib.call("smoe_dequant", _kind(kind), _lib.ptr(blocks), n * rows, cols, _lib.ptr(out),
              _lib.dtype_code(dtype), _lib.stream())
    return out


def _threads_per_row(runs: int) -> int:
    """As the reference (strata_mlx/blocks.py:303-308); kept for the `per_row` attribute only."""
    p = 1
    while p < 32 and runs % (2 * p) == 0 and runs // (2 * p) >= 4:
        p *= 2
    return p


def _matvec(lin, x2, idx_flat, share, out_dtype):
    pairs = idx_flat.numel()
    out = torch.empty((pairs, lin.output_dims), dtype=out_dtype, device=x2.device)
    if pairs:
        _lib.call("smoe_matvec", _kind(lin.kind), _lib.ptr(lin.blocks), lin.num_experts, lin.output_dims,
                  lin.input_dims, _lib.ptr(idx_flat), pairs, share, _lib.ptr(x2), _lib.ptr(out),
                  _lib.dtype_code(out_dtype), _lib.stream())
    return out


def _flat_idx(indices: torch.Tensor) -> torch.Tensor:
    flat = indices.reshape(-1)
    if flat.dtype in (torch.int32, torch.uint32):
        return flat.contiguous()
    return flat.to(torch.int32).contiguous()


class BlockSwitchLinear:
    """One projection of every expert (experts, out, in), stored as the stack's GGUF bytes on the device; its call
    takes what mlx-lm's `QuantizedSwitchLinear` takes (strata_mlx/blocks.py:525-558)."""

    # From this many pairs on one call, the products go by expert: grouped into tiles for the tensor-core GEMM
    # where the type and shape allow it (the reference unpacks the stack to floats for MLX's gather_mm there,
    # strata_mlx/blocks.py:528-531); otherwise the decode matvec, which takes any pair count. Neither expands a
    # whole stack.
    unpack_from = 5000

    def __init__(self, blocks: torch.Tensor, kind: str, shape: tuple, per_row: int | None = None):
        _kind(kind)
        self.blocks, self.kind = blocks.reshape(-1), kind
        self.num_experts, self.output_dims, self.input_dims = shape
        if self.blocks.numel() != self.num_experts * self.output_dims * row_bytes(kind, self.input_dims):
            raise ValueError(f"{self.blocks.numel()} bytes do not hold a {kind} stack of {tuple(shape)}")
        self.per_row = per_row or _threads_per_row(self.input_dims // 32)

    @property
    def shape(self):
        return (self.num_experts, self.output_dims, self.input_dims)

    def __call__(self, x: torch.Tensor, indices: torch.Tensor, sorted_indices: bool = False) -> torch.Tensor:
        """Each (token, expert) pair of `indices` times its activation row. x is (..., 1, in): either one row per
        entry of `indices`, or one row that all entries along the last axis of `indices` share (a token's k
        experts). Returns (*indices.shape, 1, out)."""
        _lib.require_cuda(x, indices, self.blocks)
        batch = tuple(x.shape[:-2])
        ishape = tuple(indices.shape)
        k = ishape[-1] if indices.dim() else 1
        if batch == ishape:
            share = 1
        elif batch == (*ishape[:-1], 1):
            share = k
        else:
            x, share = x.expand(*ishape, 1, self.input_dims), 1
        pairs = indices.numel()
        idx = _flat_idx(indices)
        if pairs >= self.unpack_from:
            out = self._many_pairs(x.reshape(-1, self.input_dims).contiguous(), idx, share)
        else:
            out = _matvec(self, x.reshape(-1, self.input_dims).contiguous(), idx, share, x.dtype)
        return out.reshape(*ishape, 1, self.output_dims)

    def _many_pairs(self, x2, idx, share):
        """(pairs, out) for a large call: rows x2[p // share] through expert idx[p], by tiles of one expert on the
        tensor cores where `tileable`, else the decode matvec."""
        if x2.dtype in (torch.float16, torch.float32) and tileable(self.kind, self.output_dims, self.input_dims):
            tiles, token, where = tiles_of(idx.reshape(-1, share), self.num_experts)
            a = x2.index_select(0, _as_int64(token))
            out = tile_matmul(self.blocks, self.kind, self.shape, a, tiles)
            return out.index_select(0, _as_int64(where)).to(x2.dtype)
        return _matvec(self, x2, idx, share, x2.dtype)


# ---- prompt chunks: pairs sorted into per-expert tiles, multiplied on the tensor cores

def tileable(kind: str, rows: int, cols: int) -> bool:
    """True when the tile GEMM handles matrices of this type and shape (strata_mlx/blocks.py:629-631)."""
    return bool(_lib.lib().smoe_tileable(_kind(kind), rows, cols))


def tile_matmul(blocks: torch.Tensor, kind: str, shape: tuple, a: torch.Tensor, tile_expert: torch.Tensor) -> torch.Tensor:
    """Grouped GEMM over tiles: row p of the (P, rows) float32 result is a[p] times the matrix of the expert its
    tile belongs to, for a stack `blocks` of `shape` (experts, rows, cols) (strata_mlx/blocks.py:634-654).

    `a` is (P, cols), float16 or float32, cut into tiles of TOKENS_TILE rows; tile_expert[i] is the expert of
    tile i. An entry of `experts` or more marks a padding tile: it is skipped and its result rows are left
    unwritten. Weights are rounded to a's type before the tensor cores multiply; accumulation is float32.
    """
    _lib.require_cuda(blocks, a, tile_expert)
    experts, rows, cols = shape
    p16 = a.shape[0]
    if p16 % TOKENS_TILE or tile_expert.numel() * TOKENS_TILE != p16:
        raise ValueError("a's rows must be TOKENS_TILE per entry of tile_expert")
    a = a.contiguous()
    te = tile_expert.reshape(-1).contiguous()
    if te.dtype not in (torch.int32, torch.uint32):
        te = te.to(torch.int32)
    out = torch.empty((p16, rows), dtype=torch.float32, device=a.device)
    ws = torch.empty(int(_lib.lib().smoe_tile_matmul_workspace_size(p16)), dtype=torch.uint8, device=a.device)
    _lib.call("smoe_tile_matmul", _kind(kind), _lib.ptr(blocks), experts, rows, cols, _lib.ptr(a),
              _lib.dtype_code(a.dtype), p16, _lib.ptr(te), _lib.ptr(out), _lib.ptr(ws), ws.numel(), _lib.stream())
    return out


def tile_matmul_rows(blocks: torch.Tensor, kind: str, shape: tuple, a: torch.Tensor, tile_expert: torch.Tensor,
                     slot_row, out_rows: int) -> torch.Tensor:
    """tile_matmul with the result read back in the caller's order, rounded once to float16: row slot_row[s] of
    the (out_rows, rows) float16 result is slot s's row (`tile_matmul(...)[where].astype(float16)` of the tiled
    path, strata_mlx/blocks.py:693, in one launch); without slot_row (None), row s for s < out_rows. `a` float16
    with at most TOKENS_TILE rows per tile (slots past its rows multiply zeros, so a dense layer's tokens need no
    padding); cols a multiple of 256."""
    _lib.require_cuda(blocks, a, tile_expert)
    experts, rows, cols = shape
    te = tile_expert.reshape(-1).contiguous()
    if te.dtype not in (torch.int32, torch.uint32):
        te = te.to(torch.int32)
    p16 = te.numel() * TOKENS_TILE
    if a.dtype != torch.float16 or not 0 < a.shape[0] <= p16:
        raise ValueError("tile_matmul_rows takes float16 activations of 1 to TOKENS_TILE rows per tile")
    a = a.contiguous()
    out = torch.empty((out_rows, rows), dtype=torch.float16, device=a.device)
    ws = torch.empty(int(_lib.lib().smoe_tile_matmul_workspace_size(p16)), dtype=torch.uint8, device=a.device)
    _lib.call("smoe_tile_matmul_rows", _kind(kind), _lib.ptr(blocks), experts, rows, cols, _lib.ptr(a), a.shape[0],
              p16, _lib.ptr(te), _lib.ptr(slot_row) if slot_row is not None else None, out_rows, _lib.ptr(out),
              _lib.ptr(ws), ws.numel(), _lib.stream())
    return out


def tile_matmul_pair(lin_a, lin_b, a: torch.Tensor, tile_expert: torch.Tensor, slot_row=None, out_rows=None):
    """Two stacks of one type and shape (a layer's gate and up) through the same tiles and activations in one
    launch: `tile_matmul` of each (float32, slot order), or with `out_rows` the rows form of each
    (`tile_matmul_rows`: float16, row slot_row[s] or s). `a` float16, cols a multiple of 256."""
    _lib.require_cuda(lin_a.blocks, lin_b.blocks, a, tile_expert)
    experts, rows, cols = lin_a.shape
    te = tile_expert.reshape(-1).contiguous()
    if te.dtype not in (torch.int32, torch.uint32):
        te = te.to(torch.int32)
    p16 = te.numel() * TOKENS_TILE
    a = a.contiguous()
    ws = torch.empty(int(_lib.lib().smoe_tile_matmul_workspace_size(p16)), dtype=torch.uint8, device=a.device)
    if out_rows is None:
        if a.shape[0] != p16:
            raise ValueError("a's rows must be TOKENS_TILE per entry of tile_expert")
        outs = [torch.empty((p16, rows), dtype=torch.float32, device=a.device) for _ in range(2)]
        _lib.call("smoe_tile_matmul_pair", _kind(lin_a.kind), _lib.ptr(lin_a.blocks), _lib.ptr(lin_b.blocks), experts,
                  rows, cols, _lib.ptr(a), p16, _lib.ptr(te), _lib.ptr(outs[0]), _lib.ptr(outs[1]), _lib.ptr(ws),
                  ws.numel(), _lib.stream())
    else:
        if not 0 < a.shape[0] <= p16:
            raise ValueError("a holds 1 to TOKENS_TILE rows per tile")
        outs = [torch.empty((out_rows, rows), dtype=torch.float16, device=a.device) for _ in range(2)]
        _lib.call("smoe_tile_matmul_pair_rows", _kind(lin_a.kind), _lib.ptr(lin_a.blocks), _lib.ptr(lin_b.blocks),
                  experts, rows, cols, _lib.ptr(a), a.shape[0], p16, _lib.ptr(te),
                  _lib.ptr(slot_row) if slot_row is not None else None, out_rows, _lib.ptr(outs[0]),
                  _lib.ptr(outs[1]), _lib.ptr(ws), ws.numel(), _lib.stream())
    return outs[0], outs[1]


def pair_takes(lin_a, lin_b, dtype) -> bool:
    """Whether tile_matmul_pair takes these two stacks with activations of `dtype`."""
    return (lin_a.kind == lin_b.kind and tuple(lin_a.shape) == tuple(lin_b.shape)
            and rows_take(lin_a.kind, lin_a.shape[2], dtype))


def slot_rows(where: torch.Tensor, slots: int) -> torch.Tensor:
    """The inverse of tiles_of's `where`: slot s -> the pair in it, 0xffffffff for slots no pair fills."""
    _lib.require_cuda(where)
    where = where.contiguous()
    out = torch.empty(slots, dtype=torch.uint32, device=where.device)
    _lib.call("smoe_slot_rows", _lib.ptr(where), where.numel(), slots, _lib.ptr(out), _lib.stream())
    return out


def rows_take(kind: str, cols: int, dtype) -> bool:
    """Whether tile_matmul_rows takes this stack with activations of `dtype`."""
    return dtype == torch.float16 and cols % 256 == 0


def tiles_of(indices: torch.Tensor, experts: int) -> tuple:
    """Group the (token, expert) pairs of `indices` (..., k) by expert into tiles of TOKENS_TILE slots
    (strata_mlx/blocks.py:657-681).

    Returns three uint32 tensors: tile_expert (each tile's expert; `experts` for tiles left empty), token (the
    token in each slot) and where (each pair's slot). Computed on the GPU; the tile count is a bound fixed by
    the pair count alone, so no host synchronisation is needed to size the outputs.
    """
    _lib.require_cuda(indices)
    k = indices.shape[-1]
    flat = indices.reshape(-1)
    flat = flat.view(torch.int32) if flat.dtype == torch.uint32 else flat.to(torch.int32)
    flat = flat.contiguous()
    pairs = flat.numel()
    most = pairs // TOKENS_TILE + min(experts, pairs)
    dev = indices.device
    tile_expert = torch.empty(most, dtype=torch.uint32, device=dev)
    token = torch.empty(most * TOKENS_TILE, dtype=torch.uint32, device=dev)
    where = torch.empty(pairs, dtype=torch.uint32, device=dev)
    if pairs:
        ws = torch.empty(int(_lib.lib().smoe_tiles_of_workspace_size(pairs, experts)), dtype=torch.uint8, device=dev)
        _lib.call("smoe_tiles_of", _lib.ptr(flat), pairs, k, experts, _lib.ptr(tile_expert), _lib.ptr(token),
                  _lib.ptr(where), _lib.ptr(ws), ws.numel(), _lib.stream())
    return tile_expert, token, where


def swiglu_to(gate: torch.Tensor, up: torch.Tensor, dtype) -> torch.Tensor:
    """swiglu(gate, up).to(dtype) in one pass: float32 gate and up to float16, the float32 SwiGLU rounded once."""
    if gate.dtype == dtype:
        return swiglu(gate, up)
    _lib.require_cuda(gate, up)
    gate, up = gate.contiguous(), up.contiguous()
    out = torch.empty(gate.shape, dtype=dtype, device=gate.device)
    _lib.call("smoe_swiglu_to", _lib.ptr(gate), _lib.ptr(up), gate.numel(), _lib.dtype_code(gate.dtype), _lib.ptr(out),
              _lib.dtype_code(dtype), _lib.stream())
    return out


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """mlx-lm's swiglu = silu(gate) * up in the inputs' type (sigmoid in float32 rounded to the type, then two
    products in the type), as the reference relies on it (strata_mlx/blocks.py:222-237)."""
    _lib.require_cuda(gate, up)
    gate, up = gate.contiguous(), up.contiguous()
    out = torch.empty_like(gate)
    _lib.call("smoe_swiglu", _lib.ptr(gate), _lib.ptr(up), gate.numel(), _lib.ptr(out), _lib.dtype_code(gate.dtype),
              _lib.stream())
    return out


def _as_int64(t):
    return (t.view(torch.int32) if t.dtype == torch.uint32 else t).to(torch.int64)


def _tiled_glu(x: torch.Tensor, indices: torch.Tensor, up, gate, down) -> torch.Tensor:
    """A prompt chunk's SwiGLU experts on the tile path: tiles_of, gather of the token rows, gate and up tile
    GEMMs, SwiGLU, the down tile GEMM, and the results read back in pair order (strata_mlx/blocks.py:684-694)."""
    tiles, token, where = tiles_of(indices, gate.num_experts)
    a = x.reshape(-1, x.shape[-1]).index_select(0, token.view(torch.int32))

    def product(lin, a):
        return tile_matmul(lin.blocks, lin.kind, lin.shape, a, tiles)

    if x.dtype == torch.float16 and rows_take(down.kind, down.input_dims, x.dtype):
        # the same values in fewer passes: the SwiGLU of the float32 sums rounded once to float16, and the down
        # product written in pair order as float16 by its own launch
        if pair_takes(gate, up, x.dtype):
            g32, u32 = tile_matmul_pair(gate, up, a, tiles)
        else:
            g32, u32 = product(gate, a), product(up, a)
        h = swiglu_to(g32, u32, x.dtype)
        out = tile_matmul_rows(down.blocks, down.kind, down.shape, h, tiles, slot_rows(where, h.shape[0]),
                               where.numel())
        return out.reshape(*indices.shape, down.output_dims)
    h = swiglu(product(gate, a), product(up, a)).to(x.dtype)
    out = product(down, h).index_select(0, _as_int64(where)).to(x.dtype)
    return out.reshape(*indices.shape, down.output_dims)


# types whose float16 products run on the tensor-core decode kernel, with the columns of its stage
MMA_MATVEC = {"IQ3_S": 256, "Q8_0": 128}
# the int8 tensor-core decode kernel forms the SwiGLU of down's input itself: types, the columns it splits the
# activations by, and the bytes of activations the shared down product with the combine may hold (one launch)
FUSED_GLU = ("IQ3_S", "Q8_0")
FUSED_GLU_COLS, FUSED_GLU_BYTES = 256, 64 << 10
BATCHED_DOWN = False  # decode_products: the routed and the shared down product in one launch
PREFETCH_DOWN = False  # decode_products: the down stacks' experts fetched into L2 by the gate/up launch (measured slower)


def matvec_glu(lin, idx: torch.Tensor, gate: torch.Tensor, up: torch.Tensor):
    """The down projection of SwiGLU(gate, up): row p of gate and up (pairs, in) goes through expert idx[p] of
    `lin`, giving (pairs, out) (strata_mlx/blocks.py:939-955). Returns None for activation types the kernels
    do not take.

    The SwiGLU is the same function (so the same bits) everywhere: the int8 tensor-core decode kernel forms
    it while it splits the activations (as the reference's _MATVEC_GLU forms it in the matvec,
    strata_mlx/blocks.py:222-224); for a product it does not take whose type has the float16 tensor-core
    kernel, a small kernel forms it first; the CUDA-core kernel forms it inside the product."""
    if gate.dtype not in (torch.float16, torch.float32) or up.dtype != gate.dtype:
        return None
    _lib.require_cuda(idx, gate, up, lin.blocks)
    idx = _flat_idx(idx)
    pairs = idx.numel()
    # (the kernel takes the pairs in as many launches as their activations need)
    fused = gate.dtype == torch.float16 and lin.kind in FUSED_GLU and lin.input_dims % FUSED_GLU_COLS == 0
    if not fused and gate.dtype == torch.float16 and lin.input_dims % MMA_MATVEC.get(lin.kind, 1 << 30) == 0:
        h = swiglu(gate.reshape(pairs, -1), up.reshape(pairs, -1))
        return _matvec(lin, h, idx, 1, gate.dtype)
    gate = gate.reshape(pairs, -1).contiguous()
    up = up.reshape(pairs, -1).contiguous()
    out = torch.empty((pairs, lin.output_dims), dtype=gate.dtype, device=gate.device)
    if pairs:
        _lib.call("smoe_matvec_glu", _kind(lin.kind), _lib.ptr(lin.blocks), lin.num_experts, lin.output_dims,
                  lin.input_dims, _lib.ptr(idx), pairs, _lib.ptr(gate), _lib.ptr(up), _lib.ptr(out),
                  _lib.dtype_code(gate.dtype), _lib.stream())
    return out


def gate_up(gate, up, x2: torch.Tensor, idx_flat: torch.Tensor, share: int):
    """The gate and up products of the same pairs in one launch (two BlockSwitchLinear calls of the
    reference, strata_mlx/blocks.py:971). x2 (pairs / share, in) -> two (pairs, out)."""
    pairs = idx_flat.numel()
    g = torch.empty((pairs, gate.output_dims), dtype=x2.dtype, device=x2.device)
    u = torch.empty_like(g)
    if gate.kind != up.kind or gate.shape != up.shape:
        return _matvec(gate, x2, idx_flat, share, x2.dtype), _matvec(up, x2, idx_flat, share, x2.dtype)
    if pairs:
        _lib.call("smoe_matvec_gate_up", _kind(gate.kind), _lib.ptr(gate.blocks), _kind(up.kind), _lib.ptr(up.blocks),
                  gate.num_experts, gate.output_dims, gate.input_dims, _lib.ptr(idx_flat), pairs, share,
                  _lib.ptr(x2), _lib.ptr(g), _lib.ptr(u), _lib.dtype_code(x2.dtype), _lib.stream())
    return g, u


def switch_glu(x: torch.Tensor, indices: torch.Tensor, up, gate, down) -> torch.Tensor:
    """Each token's chosen experts as SwiGLU feed-forwards, down(silu(gate x) * up x): x (..., in) and
    indices (..., k) give (..., k, out). Picks the tile path, the fused decode matvecs or the plain products by
    pair count, type and shape (strata_mlx/blocks.py:958-986)."""
    _lib.require_cuda(x, indices)
    lins = (up, gate, down)
    if (indices.numel() >= TILES_FROM and x.dtype in (torch.float16, torch.float32)
            and all(tileable(lin.kind, lin.output_dims, lin.input_dims) for lin in lins)):
        return _tiled_glu(x, indices, up, gate, down)
    k = indices.shape[-1]
    idx = _flat_idx(indices)
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    if idx.numel() != x2.shape[0] * k:
        raise ValueError("indices must hold k experts for every token of x")
    if idx.numel() >= min(lin.unpack_from for lin in lins):
        g = gate._many_pairs(x2, idx, k)
        u = up._many_pairs(x2, idx, k)
        out = down._many_pairs(swiglu(g, u), idx, 1)
        return out.reshape(*indices.shape, down.output_dims)
    g, u = gate_up(gate, up, x2, idx, k)
    if BLOCK_GLU and idx.numel() <= MATVEC_GLU_UPTO:
        out = matvec_glu(down, idx, g, u)
    else:
        out = _matvec(down, swiglu(g, u), idx, 1, x.dtype)
    return out.reshape(*indices.shape, down.output_dims)


def _problem(lin, idx, pairs, share, out, x=None, gate=None, up=None):
    """One smoe_matvec_batch problem; out None names lin's experts idx[:pairs] for an L2 prefetch."""
    return _lib.SmoeMatvec(_kind(lin.kind), lin.blocks.data_ptr(), lin.num_experts, lin.output_dims, lin.input_dims,
                           idx.data_ptr(), pairs, share, x.data_ptr() if x is not None else None,
                           gate.data_ptr() if gate is not None else None, up.data_ptr() if up is not None else None,
                           out.data_ptr() if out is not None else None,
                           _lib.dtype_code(out.dtype if out is not None else torch.float16))


def matvec_batch(problems, route=None) -> None:
    """Run several products in one smoe_matvec_batch call (each an smoe_matvec or smoe_matvec_glu problem); with
    `route` (a deferred route's SmoeRouteStep) the route too, in the same launch where the kernel takes both
    (smoe_route_matvec_batch)."""
    arr = (_lib.SmoeMatvec * len(problems))(*problems)
    if route is None:
        _lib.call("smoe_matvec_batch", len(problems), arr, _lib.stream())
    else:
        _lib.call("smoe_route_matvec_batch", ctypes.byref(route), len(problems), arr, _lib.stream())


def decode_products(switch_mlp, shared, x: torch.Tensor, indices: torch.Tensor, w=None, g=None, batched_down=None,
                    route_step=None):
    """(switch_mlp(x, indices), shared(x)) for a step that runs both on the decode matvec, with the routed and
    the shared expert's gate and up products in one launch (the same products, within the kernel's rounding,
    as the separate calls), then the two down products. With the combine's w (..., k) float32 and g (..., 1),
    the shared down product also forms the block's output, `moe_combine(y, w, g, shared(x))` (same bits), and
    the result is (None, out). `batched_down` (default: the module's BATCHED_DOWN) puts both down products in
    one launch and returns (y, s). None where either would take another path (a prompt's tiles, unpacked
    floats, a SwiGLU the down product does not take, activations of another type). Indices at or past a stack's
    expert count name pairs the products leave out (their rows are not written).

    `route_step`: the deferred route (`fused.route(..., defer=True)`) that writes `indices` (and w, g); it is
    launched with the gate / up products. When the result is None nothing was launched, the route included."""
    lins = (switch_mlp.gate_proj, switch_mlp.up_proj, switch_mlp.down_proj)
    slins = (shared.gate_proj, shared.up_proj, shared.down_proj)
    if x.dtype != torch.float16 or indices.numel() >= TILES_FROM or not BLOCK_GLU:
        return None
    k = indices.shape[-1]
    idx = _flat_idx(indices)
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    tokens, pairs = x2.shape[0], idx.numel()
    if (pairs != tokens * k or pairs > DECODE_UPTO or pairs >= min(lin.unpack_from for lin in lins)
            or any(lin.gemm(x2) for lin in slins)):
        return None
    _lib.require_cuda(x, indices, *(lin.blocks for lin in lins), *(lin.blocks for lin in slins))
    dev, dt = x.device, x.dtype
    gate, up, down = lins
    sg, su, sd = (lin.stack for lin in slins)
    zeros = _zeros_idx(tokens, dev)
    g_r = torch.empty((pairs, gate.output_dims), dtype=dt, device=dev)
    u_r = torch.empty((pairs, up.output_dims), dtype=dt, device=dev)
    gs = torch.empty((tokens, sg.output_dims), dtype=dt, device=dev)
    us = torch.empty((tokens, su.output_dims), dtype=dt, device=dev)
    if pairs:
        # with the two down stacks' weights fetched into L2 meanwhile (the gate/up launch is compute-bound)
        ahead = [_problem(down, idx, pairs, 1, None), _problem(sd, zeros, tokens, 1, None)] if PREFETCH_DOWN else []
        matvec_batch([_problem(gate, idx, pairs, k, g_r, x=x2), _problem(up, idx, pairs, k, u_r, x=x2),
                      _problem(sg, zeros, tokens, 1, gs, x=x2), _problem(su, zeros, tokens, 1, us, x=x2)] + ahead,
                     route=route_step)
    if batched_down is None:
        batched_down = BATCHED_DOWN
    if batched_down and sd.kind in FUSED_GLU and down.kind in FUSED_GLU:
        # both down products in one launch (the shared expert's Q8_0 rows and the routed experts' in the same
        # CTAs, so the SMs stream one while they decode the other); the combine is its own launch
        y = torch.empty((pairs, down.output_dims), dtype=dt, device=dev)
        s = torch.empty((tokens, sd.output_dims), dtype=dt, device=dev)
        if pairs:
            matvec_batch([_problem(down, idx, pairs, 1, y, gate=g_r, up=u_r), _problem(sd, zeros, tokens, 1, s, gate=gs, up=us)])
        return y.reshape(*indices.shape, down.output_dims), s.reshape(*x.shape[:-1], sd.output_dims)
    y = matvec_glu(down, idx, g_r, u_r)
    fused = (w is not None and g is not None and sd.kind in FUSED_GLU and sd.input_dims % FUSED_GLU_COLS == 0
             and tokens * sd.input_dims * 2 <= FUSED_GLU_BYTES and w.dtype == torch.float32 and g.dtype == dt
             and sd.output_dims == down.output_dims)
    if fused:
        out = torch.empty((tokens, sd.output_dims), dtype=dt, device=dev)
        if tokens:
            _lib.call("smoe_matvec_glu_combine", _kind(sd.kind), _lib.ptr(sd.blocks), sd.output_dims, sd.input_dims,
                      _lib.ptr(zeros), tokens, _lib.ptr(gs), _lib.ptr(us), _lib.ptr(y), _lib.ptr(w.contiguous()),
                      _lib.ptr(g.contiguous()), k, _lib.ptr(out), _lib.dtype_code(dt), _lib.stream())
        return None, out.reshape(*x.shape[:-1], sd.output_dims)
    s = matvec_glu(sd, zeros, gs, us)
    return y.reshape(*indices.shape, down.output_dims), s.reshape(*x.shape[:-1], sd.output_dims)


class BlockSwitchGLU:
    """The routed experts of one layer (gate, up and down stacks); calls like mlx-lm's `SwitchGLU`
    (strata_mlx/blocks.py:989-996)."""

    def __init__(self, gate: BlockSwitchLinear, up: BlockSwitchLinear, down: BlockSwitchLinear):
        self.gate_proj, self.up_proj, self.down_proj = gate, up, down

    def __call__(self, x: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
        return switch_glu(x, indices, self.up_proj, self.gate_proj, self.down_proj)


_ZEROS = {}


def _zeros_idx(n: int, device) -> torch.Tensor:
    """A cached all-zero index vector: every row of a one-expert stack is expert 0."""
    key = (n, str(device))
    t = _ZEROS.get(key)
    if t is None:
        t = _ZEROS[key] = torch.zeros(n, dtype=torch.int32, device=device)
    return t


GEMM_FROM = 32  # tokens from which a one-expert layer goes through the tensor-core tile product


def _dense_tiles(lin, x2: torch.Tensor, dtype=None) -> torch.Tensor:
    """x2 (tokens, in) through a one-expert stack on the tile product, tokens in tiles of 16 of expert 0.
    Returns (tokens, out) float32 (weights rounded to x's type, float32 sums, as `tile_matmul`), or with
    `dtype` those sums rounded to it: float16 activations take the rows variant (no padding rows, float16
    written by the product's own launch)."""
    tokens = x2.shape[0]
    p16 = (tokens + TOKENS_TILE - 1) // TOKENS_TILE * TOKENS_TILE
    te = _zeros_idx(p16 // TOKENS_TILE, x2.device)
    if dtype == torch.float16 and rows_take(lin.kind, lin.input_dims, x2.dtype):
        return tile_matmul_rows(lin.blocks, lin.kind, lin.shape, x2, te, None, tokens)
    a = x2 if p16 == tokens else torch.cat([x2, x2.new_zeros(p16 - tokens, x2.shape[1])])
    out = tile_matmul(lin.blocks, lin.kind, lin.shape, a, te)[:tokens]
    return out if dtype is None else out.to(dtype)


class BlockLinear:
    """One linear layer kept as the file's blocks (the shared expert's gate/up/down; the reference holds
    these as MLX QuantizedLinear from `to_affine`, strata_mlx/load.py:253-256). x (..., in) -> (..., out).

    A few tokens go through the decode matvec; from GEMM_FROM tokens on (a prompt's chunk) the tensor-core tile
    product reads the blocks once for all of them."""

    def __init__(self, blocks: torch.Tensor, kind: str, shape: tuple):
        self.stack = BlockSwitchLinear(blocks, kind, (1, *shape))
        self.kind, self.output_dims, self.input_dims = kind, shape[0], shape[1]

    @property
    def blocks(self):
        return self.stack.blocks

    def gemm(self, x2: torch.Tensor) -> bool:
        return (x2.shape[0] >= GEMM_FROM and x2.dtype in (torch.float16, torch.float32)
                and tileable(self.kind, self.output_dims, self.input_dims))

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        x2 = x.reshape(-1, self.input_dims).contiguous()
        if self.gemm(x2):
            out = _dense_tiles(self.stack, x2, x.dtype)
        else:
            idx = _zeros_idx(x2.shape[0], x.device)
            out = _matvec(self.stack, x2, idx, 1, x.dtype)
        return out.reshape(*x.shape[:-1], self.output_dims)


class BlockMLP:
    """The shared expert: down(silu(gate(x)) * up(x)) on blocks (mlx-lm's MLP, strata_mlx/load.py:419-421),
    gate and up in one launch and swiglu formed by the down kernel."""

    def __init__(self, gate: BlockLinear, up: BlockLinear, down: BlockLinear):
        self.gate_proj, self.up_proj, self.down_proj = gate, up, down

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        if all(p.gemm(x2) for p in (self.gate_proj, self.up_proj, self.down_proj)):
            # a prompt's chunk: the three products on the tensor cores, rounded to x's type as QuantizedLinear does
            gs, us = self.gate_proj.stack, self.up_proj.stack
            if x.dtype == torch.float16 and pair_takes(gs, us, x2.dtype):
                # gate and up in one launch (one-expert stacks: tiles of expert 0, no padding rows)
                tokens = x2.shape[0]
                te = _zeros_idx((tokens + TOKENS_TILE - 1) // TOKENS_TILE, x2.device)
                g, u = tile_matmul_pair(gs, us, x2, te, None, tokens)
            else:
                g = _dense_tiles(gs, x2, x.dtype)
                u = _dense_tiles(us, x2, x.dtype)
            out = _dense_tiles(self.down_proj.stack, swiglu(g, u), x.dtype)
            return out.reshape(*x.shape[:-1], self.down_proj.output_dims)
        idx = _zeros_idx(x2.shape[0], x.device)
        g, u = gate_up(self.gate_proj.stack, self.up_proj.stack, x2, idx, 1)
        out = matvec_glu(self.down_proj.stack, idx, g, u)
        return out.reshape(*x.shape[:-1], self.down_proj.output_dims)
