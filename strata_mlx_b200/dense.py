"""Dense layers on either side of the MoE block, on B200: the call surface of strata-mlx's `strata_mlx/dense.py`.

    ScaledLinear    a Q6_K layer as a signed byte a weight, a scale per 16 and d per 256 (dense.py:109-167)
    BlockLinear     a dense layer kept as the file's blocks; Q3_K as planes (dense.py:226-260)
    BlockEmbedding  an embedding kept as the file's blocks, a token's row decoded when it comes (dense.py:263-276)
    q6k_parts       a Q6_K tensor's three parts, made on the GPU from its blocks (strata_mlx/gguf.py:150-165)

A window of up to MAX_TOKENS tokens multiplies on the kernels of libstrata_moe.so with float32 sums in an order
fixed by the layer's shape (a token gets the same bits alone as in a window); a longer chunk of a prompt
multiplies the layer's weights made floats by the same library, as the reference does with MLX's product.
Tensors are torch CUDA tensors.
"""

import torch

from . import _lib
from .blocks import BLOCK, dequantize, q3k_planes, q3k_planes_dequantize, q3k_planes_window, window_matvec

MAX_TOKENS = 8  # beyond this many tokens a call is a prompt chunk and multiplies the expanded floats (dense.py:33)
AS_BLOCKS = ("Q3_K", "IQ4_XS")  # dense types kept as the file's blocks (strata_mlx/dense.py:190)
PLANES = True  # Q3_K's blocks held as planes (strata_mlx/dense.py:191)


def fits(rows: int, cols: int) -> bool:
    """True for the shapes ScaledLinear accepts: the reference's rule (strata_mlx/dense.py:96-98), rows in fours
    and columns in 256s; the kernel here needs only columns in groups of 16."""
    return rows % 4 == 0 and cols % 256 == 0


def q6k_parts(blocks: torch.Tensor, rows: int, cols: int):
    """A Q6_K tensor (rows, cols) as (codes int8 (rows, cols), scales int8 (rows, cols / 16), d float16
    (rows, cols / 256)): a weight is code * scale * d (strata_mlx/gguf.py:150-165), made on the GPU."""
    _lib.require_cuda(blocks)
    if cols % 256 or blocks.numel() != rows * cols // 256 * 210:
        raise ValueError(f"{blocks.numel()} bytes do not hold a Q6_K tensor of ({rows}, {cols})")
    dev = blocks.device
    codes = torch.empty((rows, cols), dtype=torch.int8, device=dev)
    scales = torch.empty((rows, cols // 16), dtype=torch.int8, device=dev)
    d = torch.empty((rows, cols // 256), dtype=torch.float16, device=dev)
    _lib.call("smoe_q6k_parts", _lib.ptr(blocks.reshape(-1).contiguous()), rows, cols, _lib.ptr(codes),
              _lib.ptr(scales), _lib.ptr(d), _lib.stream())
    return codes, scales, d


class ScaledLinear:
    """A Q6_K matrix kept as three arrays, weight = code x scale x d (int8 code per weight, int8 scale per 16,
    float16 d per d_step); used like `nn.Linear` (strata_mlx/dense.py:109-167)."""

    def __init__(self, codes: torch.Tensor, scales: torch.Tensor, d: torch.Tensor):
        _lib.require_cuda(codes, scales, d)
        self.codes, self.scales, self.d = codes.contiguous(), scales.contiguous(), d.contiguous()
        self.output_dims, self.input_dims = codes.shape
        self.d_step = self.input_dims // d.shape[1]  # weights sharing one d (256 unless the columns were permuted)
        self._floats = None
        self.keep = True  # keep the expanded floats after a prompt chunk, for the chunks that follow
        if not fits(*codes.shape) or scales.shape != (self.output_dims, self.input_dims // 16):
            raise ValueError(f"a layer of {tuple(codes.shape)} does not fit the kernel")

    @classmethod
    def from_blocks(cls, blocks: torch.Tensor, rows: int, cols: int) -> "ScaledLinear":
        return cls(*q6k_parts(blocks, rows, cols))

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.codes, self.scales, self.d))

    def floats(self, dtype: torch.dtype) -> torch.Tensor:
        """The weights (out, in), each (d scale) code in float32 rounded once to `dtype` (dense.py:128-145)."""
        out = torch.empty((self.output_dims, self.input_dims), dtype=dtype, device=self.codes.device)
        _lib.call("smoe_scaled_floats", _lib.ptr(self.codes), _lib.ptr(self.scales), _lib.ptr(self.d),
                  self.output_dims, self.input_dims, self.d_step, _lib.ptr(out), _lib.dtype_code(dtype), _lib.stream())
        return out

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        _lib.require_cuda(x)
        rows, cols = self.output_dims, self.input_dims
        lead = x.shape[:-1]
        x2 = x.reshape(-1, cols).contiguous()
        tokens = x2.shape[0]
        if tokens > MAX_TOKENS:
            # a chunk of a prompt: the floats, made at the first chunk and kept (dense.py:151-160)
            if not self.keep:
                return (x2 @ self.floats(x.dtype).T).reshape(*lead, rows)
            if self._floats is None or self._floats.dtype != x.dtype:
                self._floats = self.floats(x.dtype)
            return (x2 @ self._floats.T).reshape(*lead, rows)
        out = torch.empty((tokens, rows), dtype=x.dtype, device=x.device)
        if tokens:
            _lib.call("smoe_scaled_window", _lib.ptr(self.codes), _lib.ptr(self.scales), _lib.ptr(self.d), rows, cols,
                      self.d_step, _lib.ptr(x2), tokens, _lib.ptr(out), _lib.dtype_code(x.dtype), _lib.stream())
        return out.reshape(*lead, rows)


class BlockLinear:
    """A dense matrix kept as its GGUF blocks; used like `nn.Linear` (strata_mlx/dense.py:226-260).

    Row r of `blocks` is output r. When the model's inputs come in another order than the file's columns,
    `inputs[i]` names the file column of input i; a block cannot be permuted internally, so each call permutes
    the activations into the file's order instead. With PLANES a Q3_K matrix is kept as planes."""

    def __init__(self, blocks: torch.Tensor, kind: str, shape: tuple, inputs=None):
        _lib.require_cuda(blocks)
        self.blocks, self.kind = blocks.reshape(-1), kind
        self.output_dims, self.input_dims = shape
        self.to_file = None
        if inputs is not None:
            order = torch.as_tensor(inputs).argsort()
            self.to_file = order.to(device=blocks.device, dtype=torch.int64)
        self.planes = None
        if kind == "Q3_K" and PLANES:
            self.planes, self.blocks = q3k_planes(self.blocks, *shape), None

    @property
    def nbytes(self) -> int:
        if self.planes is None:
            return self.blocks.numel()
        return sum(a.numel() * a.element_size() for a in self.planes.values())

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        _lib.require_cuda(x)
        rows, cols = self.output_dims, self.input_dims
        lead = x.shape[:-1]
        x2 = x.reshape(-1, cols)
        tokens = x2.shape[0]
        if self.to_file is not None:
            x2 = x2.index_select(1, self.to_file)
        x2 = x2.contiguous()
        window = tokens <= MAX_TOKENS
        if window:  # decode or verify: the kernels read the blocks (or planes) directly
            out = (q3k_planes_window(self.planes, rows, cols, x2) if self.planes is not None
                   else window_matvec(self.blocks, self.kind, rows, cols, x2))
        else:  # a prompt chunk: floats expanded for this call only, then a dense product
            w = (q3k_planes_dequantize(self.planes, rows, cols, x.dtype) if self.planes is not None
                 else dequantize(self.blocks, self.kind, (rows, cols), x.dtype))
            out = x2 @ w.T
        return out.reshape(*lead, rows)


class BlockEmbedding:
    """A token embedding kept as its GGUF blocks; only the rows of the tokens asked for are decoded, at lookup
    (strata_mlx/dense.py:263-276)."""

    def __init__(self, blocks: torch.Tensor, kind: str, shape: tuple, dtype: torch.dtype):
        _lib.require_cuda(blocks)
        self.num_embeddings, self.dims = shape
        self.kind, self.dtype = kind, dtype
        per, nbytes = BLOCK[kind]
        self.rows = blocks.reshape(self.num_embeddings, self.dims // per * nbytes)

    @property
    def nbytes(self) -> int:
        return self.rows.numel()

    def __call__(self, ids: torch.Tensor) -> torch.Tensor:
        taken = self.rows.index_select(0, ids.reshape(-1).to(device=self.rows.device, dtype=torch.int64))
        out = dequantize(taken.reshape(-1), self.kind, (ids.numel(), 1, self.dims), self.dtype)
        return out.reshape(*ids.shape, self.dims)


__all__ = ["AS_BLOCKS", "BlockEmbedding", "BlockLinear", "MAX_TOKENS", "PLANES", "ScaledLinear", "fits", "q6k_parts"]
