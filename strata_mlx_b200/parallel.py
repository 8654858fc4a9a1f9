"""Expert parallelism across the GPUs of one node: one process per GPU, NCCL over NVLink / NVSwitch.

The reference runs on one device; SURVEY's multi-GPU plan splits its MoE block (`_Routed.__call__`,
strata_mlx/fused.py:487-497) at the combine:

    rank r of N holds experts [r E/N, (r+1) E/N) of every stack and rows / columns [r F/N, (r+1) F/N) of the
    shared expert's ffn; every rank computes the router and top-k itself (2 MB of weights, cheaper than
    exchanging the choice), runs its own pairs and its slice of the shared expert, writes float32 partial
    sums (routed | shared), and one all-reduce of [tokens, 2 hidden] float32 ends the block; every rank then
    applies the combine's rounding to the summed partials.

The sums are taken in a fixed order on each rank and NCCL's reduction across ranks, so the result depends on
N at the level of float32 rounding (within the 1e-3 rel-L2 budget), not on timing. No TMA multicast anywhere.
"""

import torch
import torch.distributed as dist

from . import _lib
from .blocks import BlockLinear, BlockMLP, BlockSwitchGLU, BlockSwitchLinear, gate_up, matvec_glu, row_bytes
from .fused import SparseMoeBlock, WindowLinear, top_k_softmax


def expert_range(rank: int, world: int, experts: int):
    """(first expert, count) of `rank`'s contiguous share of `experts`."""
    if experts % world:
        raise ValueError(f"{experts} experts do not split evenly over {world} ranks")
    n = experts // world
    return rank * n, n


def shard_stack(blocks: torch.Tensor, kind: str, shape: tuple, rank: int, world: int):
    """The bytes of `rank`'s experts of a stack (experts, rows, cols): a contiguous slice of the file's bytes."""
    experts, rows, cols = shape
    lo, n = expert_range(rank, world, experts)
    per = rows * row_bytes(kind, cols)
    return blocks.reshape(-1)[lo * per : (lo + n) * per], (n, rows, cols)


def slice_rows(blocks: torch.Tensor, kind: str, shape: tuple, r0: int, r1: int) -> torch.Tensor:
    """Rows [r0, r1) of a (rows, cols) tensor of blocks (contiguous)."""
    rb = row_bytes(kind, shape[1])
    return blocks.reshape(-1)[r0 * rb : r1 * rb]


def slice_cols(blocks: torch.Tensor, kind: str, shape: tuple, c0: int, c1: int) -> torch.Tensor:
    """Columns [c0, c1) of a (rows, cols) tensor of blocks, repacked into rows of their own (c0, c1 on blocks)."""
    from .blocks import BLOCK

    rows, cols = shape
    per, nbytes = BLOCK[kind]
    if c0 % per or c1 % per:
        raise ValueError(f"{kind}: columns {c0}..{c1} do not fall on blocks of {per}")
    rb = row_bytes(kind, cols)
    return blocks.reshape(rows, rb)[:, c0 // per * nbytes : c1 // per * nbytes].contiguous().reshape(-1)


def shard_layer(router, gate, up, down, shared, shared_gate, top_k: int, rank: int, world: int) -> SparseMoeBlock:
    """`rank`'s part of a MoE layer: its experts of the routed stacks (each a (blocks, kind, shape)) and its
    slice of the shared expert's ffn (gate/up rows, down columns); router and shared gate replicated."""
    def local_stack(b, kd, s):
        lb, ls = shard_stack(b, kd, s, rank, world)
        return BlockSwitchLinear(lb, kd, ls)

    sw = BlockSwitchGLU(local_stack(*gate), local_stack(*up), local_stack(*down))
    (gb, gk, (fs, hid)), (ub, uk, _), (db, dk, _) = shared
    lo, n = expert_range(rank, world, fs)
    sh = BlockMLP(BlockLinear(slice_rows(gb, gk, (fs, hid), lo, lo + n), gk, (n, hid)),
                  BlockLinear(slice_rows(ub, uk, (fs, hid), lo, lo + n), uk, (n, hid)),
                  BlockLinear(slice_cols(db, dk, (hid, fs), lo, lo + n), dk, (hid, n)))
    return SparseMoeBlock(router, sw, sh, shared_gate, top_k)


class ExpertParallelMoE:
    """A MoE block whose experts are spread over the ranks of `group`: call it on every rank with the same x.

    `layer` is this rank's part (`shard_layer`): the full router and shared-expert gate, the rank's experts,
    its slice of the shared expert. Returns the whole block's output on every rank."""

    def __init__(self, layer: SparseMoeBlock, rank: int, world: int, experts: int, group=None):
        self.layer, self.rank, self.world, self.group = layer, rank, world, group
        self.lo, self.count = expert_range(rank, world, experts)
        self.experts = experts

    def local_indices(self, idx: torch.Tensor) -> torch.Tensor:
        """This rank's view of the chosen experts: idx - lo for its own, `count` (left out) for the others."""
        flat = idx.reshape(-1).contiguous()
        out = torch.empty_like(flat)
        _lib.call("smoe_localize", _lib.ptr(flat), flat.numel(), self.lo, self.count, _lib.ptr(out), _lib.stream())
        return out.reshape(idx.shape)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        layer = self.layer
        lead, hidden = x.shape[:-1], x.shape[-1]
        x2 = x.reshape(-1, hidden).contiguous()
        tokens, k = x2.shape[0], layer.top_k
        logits = layer.gate(x2)
        idx, w = top_k_softmax(logits, k)
        lidx = self.local_indices(idx).reshape(-1)
        sw = layer.switch_mlp
        g, u = gate_up(sw.gate_proj, sw.up_proj, x2, lidx, k)
        y = matvec_glu(sw.down_proj, lidx, g, u)
        s = layer.shared_expert(x2)
        sums = torch.empty((tokens, 2 * hidden), dtype=torch.float32, device=x.device)
        _lib.call("smoe_partial_sums", _lib.ptr(y), _lib.ptr(w.contiguous()), _lib.ptr(lidx), self.count, _lib.ptr(s),
                  tokens, k, hidden, _lib.ptr(sums), _lib.dtype_code(x.dtype), _lib.stream())
        if self.world > 1:
            dist.all_reduce(sums, group=self.group)
        gs = layer.shared_expert_gate(x2).to(x.dtype).contiguous()
        out = torch.empty((tokens, hidden), dtype=x.dtype, device=x.device)
        _lib.call("smoe_combine_sums", _lib.ptr(sums), _lib.ptr(gs), tokens, hidden, _lib.ptr(out),
                  _lib.dtype_code(x.dtype), _lib.stream())
        return out.reshape(*lead, hidden)


__all__ = ["ExpertParallelMoE", "expert_range", "shard_stack", "shard_layer", "slice_cols", "slice_rows",
           "WindowLinear"]
