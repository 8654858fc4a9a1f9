"""Expert parallelism across the GPUs of one node: one process per GPU, NCCL over NVLink / NVSwitch.

The reference runs on one device; the multi-GPU plan here splits its MoE block (`_Routed.__call__`,
strata_mlx/fused.py:487-497) at the combine:

    rank r of N holds experts [r E/N, (r+1) E/N) of every stack and rows / columns [r F/N, (r+1) F/N) of the
    shared expert's ffn; every rank computes the router and top-k itself (2 MB of weights, cheaper than
    exchanging the choice), runs its own pairs and its slice of the shared expert, writes float32 partial
    sums (routed | shared), and one all-reduce of [tokens, 2 hidden] float32 ends the block; every rank then
    applies the combine's rounding to the summed partials.

The sums are taken in a fixed order on each rank and NCCL's reduction across ranks, so the result depends on
N at the level of float32 rounding (within the 1e-3 rel-L2 budget), not on timing.

A prompt chunk splits by tokens as well (`ExpertParallelPrompt`): each rank routes its own tokens, sends every
pair's token row to the rank of its expert (an all-to-all of the counts, then of the rows and the experts'
local numbers), runs the grouped products over what it received, sends the outputs back by the reverse
all-to-all, and combines at the tokens' home with the whole shared expert. A pair's output is computed by the
same kernels from the same row as on one device, and the combine reads the outputs in the same order, so the
result differs from one device's only where the receiving rank's pair count chooses another product path.
No TMA multicast anywhere.
"""

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .blocks import (BlockLinear, BlockMLP, BlockSwitchGLU, BlockSwitchLinear, decode_products, gate_up, matvec_glu,
                     row_bytes)
from . import fused as _fused
from .fused import SparseMoeBlock, WindowLinear, launch_route, route, top_k_softmax


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


def shard_layer(router, gate, up, down, shared, shared_gate, top_k: int, rank: int, world: int,
                whole_shared: bool = False) -> SparseMoeBlock:
    """`rank`'s part of a MoE layer: its experts of the routed stacks (each a (blocks, kind, shape)) and its
    slice of the shared expert's ffn (gate/up rows, down columns), or with `whole_shared` the whole shared
    expert (a prompt chunk's ranks each run it on their own tokens); router and shared gate replicated."""
    def local_stack(b, kd, s):
        lb, ls = shard_stack(b, kd, s, rank, world)
        return BlockSwitchLinear(lb, kd, ls)

    sw = BlockSwitchGLU(local_stack(*gate), local_stack(*up), local_stack(*down))
    if whole_shared:
        return SparseMoeBlock(router, sw, BlockMLP(*(BlockLinear(b, kd, s) for b, kd, s in shared)), shared_gate,
                              top_k)
    (gb, gk, (fs, hid)), (ub, uk, _), (db, dk, _) = shared
    lo, n = expert_range(rank, world, fs)
    sh = BlockMLP(BlockLinear(slice_rows(gb, gk, (fs, hid), lo, lo + n), gk, (n, hid)),
                  BlockLinear(slice_rows(ub, uk, (fs, hid), lo, lo + n), uk, (n, hid)),
                  BlockLinear(slice_cols(db, dk, (hid, fs), lo, lo + n), dk, (hid, n)))
    return SparseMoeBlock(router, sw, sh, shared_gate, top_k)


class PeerExchange:
    """The buffers of a decode step's one exchange over NVLink peer memory (`smoe_ep_reduce_combine`): one per
    rank, `hidden` values of up to `max_tokens` tokens, mapped by every rank of the node through CUDA IPC
    handles. Make it on every rank of `group` at the same point (the handles are all-gathered); the calls that
    use it must be ordered on one stream per rank, and every rank must make the same calls in the same order.

    `reduce_combine` is the end of an expert-parallel MoE block: each rank's partial sums go to every rank, are
    added in rank order and rounded as the combine rounds them, so every rank gets the same bits. A wait that
    gives up (a rank that never arrives) leaves the outputs unwritten and `failed()` true."""

    HANDLE = 64

    def __init__(self, rank: int, world: int, hidden: int, max_tokens: int = 64, group=None, device=None):
        self.rank, self.world, self.hidden, self.max_tokens = rank, world, hidden, max_tokens
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        nbytes = int(_lib.lib().smoe_ep_exchange_bytes(world, max_tokens, hidden))
        if nbytes == 0:
            raise ValueError(f"no exchange for {world} ranks of {max_tokens} x {hidden} values")
        buf, handle = ctypes.c_void_p(), (ctypes.c_uint8 * self.HANDLE)()
        with torch.cuda.device(self.device):
            _lib.call("smoe_ep_exchange_alloc", nbytes, ctypes.byref(buf), handle)
        self.buffer = buf.value
        self.peers, self._opened = [], []
        if world == 1:
            self.peers = [self.buffer]
            return
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=self.device)
        everyone = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(everyone, mine, group=group)
        for r, h in enumerate(everyone):
            if r == rank:
                self.peers.append(self.buffer)
                continue
            hb = (ctypes.c_uint8 * self.HANDLE)(*h.cpu().tolist())
            p = ctypes.c_void_p()
            with torch.cuda.device(self.device):
                _lib.call("smoe_ep_exchange_open", hb, ctypes.byref(p))
            self.peers.append(p.value)
            self._opened.append(p.value)

    def spec(self, y, w, lidx, experts: int, s, g, out, wait_polls: int = 0) -> "_lib.SmoeEpReduce":
        tokens, k = w.shape[0], w.shape[-1]
        d = out.shape[-1]
        return _lib.SmoeEpReduce(self.rank, self.world, (ctypes.c_void_p * 16)(*self.peers), y.data_ptr(),
                                 w.data_ptr(), lidx.data_ptr(), experts, s.data_ptr() if s is not None else None,
                                 g.data_ptr(), tokens, k, d, self.max_tokens * self.hidden, out.data_ptr(),
                                 _lib.dtype_code(out.dtype), wait_polls)

    def reduce_combine(self, y, w, lidx, experts: int, s, g, out, wait_polls: int = 0) -> torch.Tensor:
        """out (tokens, hidden) = the block's end from every rank's y (tokens, k, hidden) of its experts, w
        (tokens, k) float32, lidx (tokens, k) local experts (>= `experts` for another rank's), s (tokens, hidden)
        its slice of the shared expert (or None) and g (tokens) the shared expert's gate value."""
        _lib.require_cuda(y, w, lidx, g, out, s)
        if out.shape[0] > self.max_tokens or out.shape[-1] != self.hidden:
            raise ValueError(f"the exchange holds up to {self.max_tokens} tokens of {self.hidden}")
        spec = self.spec(y, w, lidx, experts, s, g, out, wait_polls)
        _lib.call("smoe_ep_reduce_combine", ctypes.byref(spec), _lib.stream())
        return out

    def failed(self, clear: bool = False) -> bool:
        """Whether a wait of this rank's exchange gave up (synchronizes the device)."""
        flag = ctypes.c_int(0)
        with torch.cuda.device(self.device):
            _lib.call("smoe_ep_exchange_status", ctypes.c_void_p(self.buffer), ctypes.byref(flag), int(clear))
        return flag.value != 0

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (after every rank is done with it: barrier first)."""
        with torch.cuda.device(self.device):
            for p in self._opened:
                _lib.call("smoe_ep_exchange_close", ctypes.c_void_p(p))
            self._opened = []
            if self.buffer:
                _lib.call("smoe_ep_exchange_free", ctypes.c_void_p(self.buffer))
                self.buffer = None


class ExpertParallelMoE:
    """A MoE block whose experts are spread over the ranks of `group`: call it on every rank with the same x.

    `layer` is this rank's part (`shard_layer`): the full router and shared-expert gate, the rank's experts,
    its slice of the shared expert. Returns the whole block's output on every rank.

    With a `PeerExchange`, a decode step of float16 tokens is four launches overlapped by programmatic
    dependent launch: the route (router, top-k, softmax, shared gate and this rank's view of the choice), the
    routed and shared gate / up products in one launch (with `fused.FUSED_ROUTE`, the route goes into that
    launch: `smoe_route_matvec_batch`), both down products in one launch, and `smoe_ep_reduce_combine` (the
    exchange of the partial sums over peer memory with the combine). Without one (or for other activations),
    the partial sums go through one all-reduce of the process group."""

    def __init__(self, layer: SparseMoeBlock, rank: int, world: int, experts: int, group=None,
                 exchange: "PeerExchange | None" = None):
        self.layer, self.rank, self.world, self.group = layer, rank, world, group
        self.lo, self.count = expert_range(rank, world, experts)
        self.experts = experts
        self.exchange = exchange

    def local_indices(self, idx: torch.Tensor) -> torch.Tensor:
        """This rank's view of the chosen experts: idx - lo for its own, `count` (left out) for the others."""
        flat = idx.reshape(-1).contiguous()
        out = torch.empty_like(flat)
        _lib.call("smoe_localize", _lib.ptr(flat), flat.numel(), self.lo, self.count, _lib.ptr(out), _lib.stream())
        return out.reshape(idx.shape)

    def _exchange_step(self, x2: torch.Tensor):
        """The block through the peer exchange, or None where it does not apply."""
        ex, layer = self.exchange, self.layer
        tokens, hidden = x2.shape
        if (ex is None or tokens == 0 or tokens > ex.max_tokens or hidden != ex.hidden
                or x2.dtype not in (torch.float16, torch.float32)):
            return None
        k = layer.top_k
        r = route(layer.gate, layer.shared_expert_gate, x2, k, local=(self.lo, self.count), defer=True)
        if r is None:
            return None
        idx, w, g, lidx, step = r
        if not _fused.FUSED_ROUTE:
            launch_route(step)
            step = None
        sw, sh = layer.switch_mlp, layer.shared_expert
        ys = None
        if isinstance(sw, BlockSwitchGLU) and isinstance(sh, BlockMLP):
            # the route in the gate / up launch
            ys = decode_products(sw, sh, x2, lidx, batched_down=True, route_step=step)
        if ys is None and step is not None:
            launch_route(step)
        if ys is None or ys[0] is None:
            ys = (sw(x2, lidx), sh(x2))
        y, s = ys
        out = torch.empty((tokens, hidden), dtype=x2.dtype, device=x2.device)
        return ex.reduce_combine(y.reshape(tokens, k, hidden), w, lidx, self.count, s.reshape(tokens, hidden),
                                 g.reshape(tokens), out)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        layer = self.layer
        lead, hidden = x.shape[:-1], x.shape[-1]
        x2 = x.reshape(-1, hidden).contiguous()
        out = self._exchange_step(x2)
        if out is not None:
            return out.reshape(*lead, hidden)
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


def exchange_counts(counts: torch.Tensor, group=None) -> torch.Tensor:
    """All-to-all of one int32 per rank: element r of the result is what rank r has for this one."""
    out = torch.empty_like(counts)
    dist.all_to_all_single(out, counts, group=group)
    return out


def exchange_rows(rows: torch.Tensor, send: list, recv: list, group=None) -> torch.Tensor:
    """All-to-all of rows: the first send[r] rows of `rows` (after those for ranks before r) go to rank r,
    and the result holds recv[r] rows from each rank r, in rank order. Integer rows travel as int32."""
    out = torch.empty((sum(recv),) + tuple(rows.shape[1:]), dtype=rows.dtype, device=rows.device)
    src = rows[: sum(send)]
    if rows.dtype == torch.uint32:
        src, out = src.view(torch.int32), out.view(torch.int32)
    dist.all_to_all_single(out, src.contiguous(), recv, send, group=group)
    return out.view(rows.dtype) if rows.dtype == torch.uint32 else out


def dispatch(idx: torch.Tensor, x: torch.Tensor, experts: int, world: int):
    """The send side of a prompt chunk's exchange (`smoe_ep_dispatch`): per-rank pair counts (int32, world),
    each pair's place in the send order (int32, -1 if not sent), the expert of each place in its owner's
    numbering (uint32) and the token row of each place. idx (tokens, k) uint32, x (tokens, hidden)."""
    tokens, k = idx.shape
    hidden = x.shape[-1]
    pairs = tokens * k
    counts = torch.empty(world, dtype=torch.int32, device=x.device)
    where = torch.empty(pairs, dtype=torch.int32, device=x.device)
    send_expert = torch.empty(pairs, dtype=torch.uint32, device=x.device)
    send_x = torch.empty((pairs, hidden), dtype=x.dtype, device=x.device)
    _lib.call("smoe_ep_dispatch", _lib.ptr(idx.contiguous()), pairs, k, experts, world, _lib.ptr(x), hidden,
              _lib.dtype_code(x.dtype), _lib.ptr(counts), _lib.ptr(where), _lib.ptr(send_expert), _lib.ptr(send_x),
              _lib.stream())
    return counts, where, send_expert, send_x


def combine_rows(y: torch.Tensor, where: torch.Tensor, w: torch.Tensor, g: torch.Tensor, s: torch.Tensor):
    """The block's combine with each pair's expert output at row where[t k + j] of y (`smoe_combine_rows`)."""
    tokens, k = w.shape
    hidden = s.shape[-1]
    out = torch.empty((tokens, hidden), dtype=s.dtype, device=s.device)
    _lib.call("smoe_combine_rows", _lib.ptr(y), _lib.ptr(where), _lib.ptr(w.contiguous()),
              _lib.ptr(g.contiguous()), _lib.ptr(s.contiguous()), tokens, k, hidden, _lib.ptr(out),
              _lib.dtype_code(s.dtype), _lib.stream())
    return out


class ExpertParallelPrompt:
    """A prompt chunk through a MoE block whose experts are spread over the ranks of `group`, each rank holding
    its own tokens: call it on every rank with that rank's tokens (any count, 0 included).

    `layer` is this rank's part with the whole shared expert (`shard_layer(..., whole_shared=True)`). Per call:
    the router and top-k of the rank's tokens, `smoe_ep_dispatch`, the all-to-all of the counts (the one host
    synchronisation: NCCL needs the split sizes), of the token rows and of the experts' numbers, the grouped
    products of the received pairs (`switch_glu`, one pair per row), the reverse all-to-all of the outputs and
    the combine at home (`smoe_combine_rows`). `received` is the pair count the last call computed here."""

    def __init__(self, layer: SparseMoeBlock, rank: int, world: int, experts: int, group=None):
        self.layer, self.rank, self.world, self.group = layer, rank, world, group
        self.experts = experts
        expert_range(rank, world, experts)
        self.received = 0

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        layer = self.layer
        lead, hidden = x.shape[:-1], x.shape[-1]
        x2 = x.reshape(-1, hidden).contiguous()
        if x2.shape[0] == 0:
            # a rank with no tokens of this chunk still takes part in every exchange: it routes one zero token
            # (its pairs are computed where they land and dropped here), so no exchange or product of this rank
            # is empty
            self(x2.new_zeros(1, hidden))
            return x2.new_zeros(*lead, hidden)
        k = layer.top_k
        idx, w = top_k_softmax(layer.gate(x2), k)
        counts, where, send_expert, send_x = dispatch(idx, x2, self.experts, self.world)
        if self.world > 1:
            recv_counts = exchange_counts(counts, self.group)
            send, recv = counts.tolist(), recv_counts.tolist()
            rows = exchange_rows(send_x, send, recv, self.group)
            local = exchange_rows(send_expert, send, recv, self.group)
        else:
            send = recv = counts.tolist()
            rows, local = send_x[: send[0]], send_expert[: send[0]]
        self.received = rows.shape[0]
        if self.received:
            y = layer.switch_mlp(rows, local.reshape(-1, 1)).reshape(-1, hidden)
        else:
            y = rows
        back = exchange_rows(y, recv, send, self.group) if self.world > 1 else y
        s = layer.shared_expert(x2)
        g = layer.shared_expert_gate(x2).to(x.dtype)
        return combine_rows(back, where, w, g, s).reshape(*lead, hidden)


__all__ = ["ExpertParallelMoE", "ExpertParallelPrompt", "PeerExchange", "combine_rows", "dispatch", "exchange_counts",
           "exchange_rows", "expert_range", "shard_stack", "shard_layer", "slice_cols", "slice_rows", "WindowLinear"]
