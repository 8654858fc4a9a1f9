"""The MoE block's router, top-k choice and combine on B200: the MoE part of strata-mlx's `strata_mlx/fused.py`.

    WindowLinear   float16 router weights times the activations, float32 sums and result
    top_k          the k largest logits of each row, largest first, ties to the lower index
    moe_combine    sum_k y_k w_k rounded to the type, plus sigmoid(g) * the shared expert, in MLX's order
    SparseMoeBlock the model's MoE block as `_Routed.__call__` computes it (strata_mlx/fused.py:484-497)
    FusedResidual  the hyper-connection before and after every block: norm, low-rank gate, mix (fused.py:280-323)

Names and conventions follow the reference; tensors are torch CUDA tensors and every product runs in the
sm_100a kernels of libstrata_moe.so.
"""

import ctypes

import torch

from . import _lib
from .blocks import BlockMLP, BlockSwitchGLU, decode_products

ROUTER_TOPK = True  # strata_mlx/fused.py:420 (the kernel is the only top-k here; kept for engines that set it)
ROUTER_AS_IS = True  # the router reads float16 activations as they are (strata_mlx/fused.py:421)
COMBINE_UPTO = 16  # strata_mlx/fused.py:464: tokens the reference's kernel takes; this one takes any count


class WindowLinear:
    """The router's product: float16 weights (rows, cols) times float16 or float32 activations, accumulated and
    returned in float32, no bias (strata_mlx/fused.py:357-390).

    Takes a weight tensor or any object with a `.weight`. Every token count runs on the same kernel, and the
    order of each token's sum is fixed by the weight's shape, so a token's logits do not depend on its window."""

    upto, groups = 8, 16

    def __init__(self, linear):
        self.linear = linear
        w = self.weight
        self.rows, self.cols = w.shape

    @property
    def weight(self) -> torch.Tensor:
        return self.linear if isinstance(self.linear, torch.Tensor) else self.linear.weight

    def takes(self, x: torch.Tensor) -> bool:
        return self.weight.dtype == torch.float16 and x.dtype in (torch.float16, torch.float32)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        w = self.weight
        _lib.require_cuda(w, x)
        if not self.takes(x):
            raise ValueError("WindowLinear takes float16 weights and float16/float32 activations")
        tokens = x.numel() // self.cols
        x2 = x.reshape(tokens, self.cols).contiguous()
        out = torch.empty((tokens, self.rows), dtype=torch.float32, device=x.device)
        if tokens:
            _lib.call("smoe_router_logits", _lib.ptr(w.contiguous()), _lib.ptr(x2), _lib.dtype_code(x.dtype), tokens,
                      self.rows, self.cols, _lib.ptr(out), _lib.stream())
        return out.reshape(*x.shape[:-1], self.rows)


def _top_k(logits: torch.Tensor, k: int, with_weights: bool):
    _lib.require_cuda(logits)
    if logits.dtype != torch.float32:
        raise ValueError("top_k takes float32 logits")
    n = logits.shape[-1]
    rows = logits.numel() // n
    lg = logits.reshape(rows, n).contiguous()
    idx = torch.empty((rows, k), dtype=torch.uint32, device=logits.device)
    w = torch.empty((rows, k), dtype=torch.float32, device=logits.device) if with_weights else None
    if rows:
        _lib.call("smoe_top_k", _lib.ptr(lg), rows, n, k, _lib.ptr(idx), _lib.ptr(w), _lib.stream())
    shape = (*logits.shape[:-1], k)
    return idx.reshape(shape), (w.reshape(shape) if w is not None else None)


def top_k(logits: torch.Tensor, k: int) -> torch.Tensor:
    """uint32 positions of the k biggest float32 logits in each row of (..., N), biggest first and equal values
    in index order: what `mx.argpartition(-logits, k - 1)[..., :k]` picks (strata_mlx/fused.py:424-436)."""
    return _top_k(logits, k, False)[0]


def top_k_softmax(logits: torch.Tensor, k: int):
    """`top_k` and `softmax(take_along_axis(logits, idx), precise=True)` in one launch
    (strata_mlx/fused.py:490-491) -> (idx uint32, w float32)."""
    return _top_k(logits, k, True)


_COUNTERS = {}

FUSED_ROUTE = False  # decode: the route in the gate / up launch (smoe_route_matvec_batch; measured slower)
LAYER_KERNEL = False  # one launch per one-token step (smoe_decode_layer) where the types and shapes allow it
_LAYER_SCRATCH = {}


def decode_layer(block: "SparseMoeBlock", x: torch.Tensor):
    """block(x) for one float16 token in a single persistent launch (smoe_decode_layer: router, top-k, the
    shared gate, the gate / up and down products of the routed and the shared expert, the combine), or None
    where the kernel does not apply: another type than IQ3_S routed / Q8_0 shared stacks, other shapes, more
    than one token."""
    if not LAYER_KERNEL or x.dtype != torch.float16 or x.numel() != block.gate.cols or not x.is_cuda:
        return None
    sw, sh = block.switch_mlp, block.shared_expert
    if not isinstance(sw, BlockSwitchGLU) or not isinstance(sh, BlockMLP):
        return None
    g, u, d = sw.gate_proj, sw.up_proj, sw.down_proj
    sg, su, sd = sh.gate_proj.stack, sh.up_proj.stack, sh.down_proj.stack
    if any(lin.kind != "IQ3_S" for lin in (g, u, d)) or any(lin.kind != "Q8_0" for lin in (sg, su, sd)):
        return None
    router, sgw = block.gate.weight, block.shared_expert_gate.weight
    experts, hidden, k = block.gate.rows, block.gate.cols, block.top_k
    ffn, sffn = g.output_dims, sg.output_dims
    if (g.shape != (experts, ffn, hidden) or u.shape != g.shape or d.shape != (experts, hidden, ffn)
            or sg.shape != (1, sffn, hidden) or su.shape != sg.shape or sd.shape != (1, hidden, sffn)):
        return None
    if (router.dtype != torch.float16 or sgw.dtype != torch.float16 or sgw.numel() != hidden
            or hidden % 512 or ffn % 512 or sffn % 256 or experts > 256 or not 1 <= k <= min(experts, 32)):
        return None
    if k >= min(lin.unpack_from for lin in (g, u, d)):
        return None
    dev = x.device
    key = (str(dev), hidden, k, ffn, sffn)
    scratch = _LAYER_SCRATCH.get(key)
    if scratch is None:
        nbytes = int(_lib.lib().smoe_decode_layer_scratch(hidden, k, ffn, sffn))
        scratch = _LAYER_SCRATCH[key] = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    logits = torch.empty(experts, dtype=torch.float32, device=dev)
    idx = torch.empty(k, dtype=torch.uint32, device=dev)
    w = torch.empty(k, dtype=torch.float32, device=dev)
    gate_out = torch.empty(1, dtype=x.dtype, device=dev)
    out = torch.empty(hidden, dtype=x.dtype, device=dev)
    spec = _lib.SmoeDecodeLayer(
        _lib.ptr(router.contiguous()), _lib.ptr(sgw.contiguous()), experts, hidden, k, 21, _lib.ptr(g.blocks),
        _lib.ptr(u.blocks), _lib.ptr(d.blocks), ffn, 8, _lib.ptr(sg.blocks), _lib.ptr(su.blocks), _lib.ptr(sd.blocks),
        sffn, _lib.ptr(logits), _lib.ptr(idx), _lib.ptr(w), _lib.ptr(gate_out), _lib.ptr(out), _lib.ptr(scratch))
    _lib.call("smoe_decode_layer", ctypes.byref(spec), _lib.ptr(x.contiguous()), _lib.stream())
    return out.reshape(x.shape)


def decode_layer_failed(x: torch.Tensor, block: "SparseMoeBlock") -> bool:
    """Whether a wait of the one-launch decode step gave up since the scratch was made (its outputs are then
    not valid). Reads the flag back from the device."""
    g, sg = block.switch_mlp.gate_proj, block.shared_expert.gate_proj.stack
    key = (str(x.device), block.gate.cols, block.top_k, g.output_dims, sg.output_dims)
    scratch = _LAYER_SCRATCH.get(key)
    if scratch is None:
        return False
    flag = ctypes.c_int(0)
    _lib.call("smoe_decode_layer_status", _lib.ptr(scratch), block.gate.cols, block.top_k, g.output_dims,
              sg.output_dims, ctypes.byref(flag))
    return flag.value != 0


def route(gate: "WindowLinear", shared_gate, x: torch.Tensor, k: int, local=None, defer: bool = False):
    """The start of the MoE block in one launch: (idx, w, g) = (top_k_softmax(gate(x), k),
    shared_gate(x).to(x.dtype)) with the same sums and choice as those calls (strata_mlx/fused.py:487-491).
    shared_gate: a WindowLinear of one row, or None (g is then None). With `local` = (lo, count), an expert-
    parallel rank's experts, a fourth result lidx: idx - lo for those experts, `count` for the others, from the
    same launch. None where the kernel does not take x.

    With `defer`, nothing is launched yet: the result gains a last item, the route's `SmoeRouteStep`, which
    either the products that read its choice take into their own launch (`decode_products(route_step=...)`)
    or `launch_route` launches alone; the outputs are written by that launch."""
    if not gate.takes(x) or gate.rows > 2048 or not 1 <= k <= min(gate.rows, 32):
        return None
    if shared_gate is not None and (not shared_gate.takes(x) or shared_gate.rows != 1 or shared_gate.cols != gate.cols):
        return None
    _lib.require_cuda(gate.weight, x)
    tokens = x.numel() // gate.cols
    x2 = x.reshape(tokens, gate.cols).contiguous()
    dev = x.device
    logits = torch.empty((tokens, gate.rows), dtype=torch.float32, device=dev)
    idx = torch.empty((tokens, k), dtype=torch.uint32, device=dev)
    w = torch.empty((tokens, k), dtype=torch.float32, device=dev)
    g = torch.empty((tokens,), dtype=x.dtype, device=dev) if shared_gate is not None else None
    nbytes = int(_lib.lib().smoe_route_step_counters(tokens) if defer else _lib.lib().smoe_route_counters(tokens))
    key = (str(dev), nbytes, defer)
    counters = _COUNTERS.get(key)
    if counters is None:
        counters = _COUNTERS[key] = torch.zeros(nbytes // 4, dtype=torch.int32, device=dev)
    lidx = torch.empty((tokens, k), dtype=torch.uint32, device=dev) if local is not None else None
    lead = x.shape[:-1]
    if defer:
        wt = gate.weight.contiguous()
        gw = shared_gate.weight.contiguous() if shared_gate is not None else None
        step = _lib.SmoeRouteStep(_lib.ptr(wt), _lib.ptr(gw) if gw is not None else None, _lib.ptr(x2),
                                  _lib.dtype_code(x.dtype), tokens, gate.rows, gate.cols, k, _lib.ptr(logits),
                                  _lib.ptr(idx), _lib.ptr(w), _lib.ptr(g) if g is not None else None,
                                  _lib.ptr(counters), local[0] if local is not None else 0,
                                  local[1] if local is not None else 0, _lib.ptr(lidx) if lidx is not None else None)
        step._keep = (wt, gw, x2, logits, idx, w, g, counters, lidx)  # (the tensors the pointers name)
        out = (idx.reshape(*lead, k), w.reshape(*lead, k), g.reshape(*lead, 1) if g is not None else None)
        return (out if local is None else out + (lidx.reshape(*lead, k),)) + (step,)
    if tokens:
        common = (_lib.ptr(gate.weight.contiguous()),
                  _lib.ptr(shared_gate.weight.contiguous()) if shared_gate is not None else None, _lib.ptr(x2),
                  _lib.dtype_code(x.dtype), tokens, gate.rows, gate.cols, k, _lib.ptr(logits), _lib.ptr(idx),
                  _lib.ptr(w), _lib.ptr(g) if g is not None else None, _lib.ptr(counters))
        if local is None:
            _lib.call("smoe_route", *common, _lib.stream())
        else:
            _lib.call("smoe_route_local", *common, local[0], local[1], _lib.ptr(lidx), _lib.stream())
    out = (idx.reshape(*lead, k), w.reshape(*lead, k), g.reshape(*lead, 1) if g is not None else None)
    return out if local is None else out + (lidx.reshape(*lead, k),)


def launch_route(step) -> None:
    """Launch a deferred route (`route(..., defer=True)`) by itself."""
    if step.tokens:
        _lib.call("smoe_route_matvec_batch", ctypes.byref(step), 0, None, _lib.stream())


def moe_combine(y: torch.Tensor, w: torch.Tensor, g: torch.Tensor, s: torch.Tensor):
    """y (..., K, D), w (..., K) float32, g (..., 1), s (..., D) -> (..., D) in y's type
    (strata_mlx/fused.py:467-481). None where the types are not the kernel's."""
    *lead, k, d = y.shape
    if y.dtype not in (torch.float16, torch.float32) or w.dtype != torch.float32:
        return None
    if g.dtype != y.dtype or s.dtype != y.dtype:
        return None
    _lib.require_cuda(y, w, g, s)
    rows = y.numel() // (k * d)
    out = torch.empty((rows, d), dtype=y.dtype, device=y.device)
    if rows:
        _lib.call("smoe_combine", _lib.ptr(y.contiguous()), _lib.ptr(w.contiguous()), _lib.ptr(g.contiguous()),
                  _lib.ptr(s.contiguous()), rows, k, d, _lib.ptr(out), _lib.dtype_code(y.dtype), _lib.stream())
    return out.reshape(*lead, d)


class SparseMoeBlock:
    """One MoE layer of the model: router logits, `top_k` choice, softmax over the chosen, the routed experts, the
    gated shared expert and `moe_combine`, in the order `_Routed.__call__` runs them (strata_mlx/fused.py:484-497):

        logits = gate(x) (float32); idx = top_k(logits, k); w = softmax(logits[idx]);
        y = switch_mlp(x, idx); g = shared_expert_gate(x); s = shared_expert(x); out = moe_combine(y, w, g, s)

    gate: WindowLinear or float16 weight (experts, hidden); switch_mlp: BlockSwitchGLU; shared_expert:
    BlockMLP; shared_expert_gate: float16 weight (1, hidden)."""

    def __init__(self, gate, switch_mlp: BlockSwitchGLU, shared_expert: BlockMLP, shared_expert_gate, top_k: int):
        self.gate = gate if isinstance(gate, WindowLinear) else WindowLinear(gate)
        self.switch_mlp, self.shared_expert = switch_mlp, shared_expert
        self.shared_expert_gate = shared_expert_gate if isinstance(shared_expert_gate, WindowLinear) else WindowLinear(
            shared_expert_gate)
        self.top_k = top_k

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        out = decode_layer(self, x)
        if out is not None:
            return out
        # the route goes into the gate / up launch of the decode products where they take it (FUSED_ROUTE)
        r = route(self.gate, self.shared_expert_gate, x, self.top_k, defer=FUSED_ROUTE)
        step = None
        if r is not None and FUSED_ROUTE:
            idx, w, g, step = r
        elif r is not None:
            idx, w, g = r
        else:
            logits = self.gate(x)
            idx, w = top_k_softmax(logits, self.top_k)
            g = self.shared_expert_gate(x).to(x.dtype)
        ys = None
        if isinstance(self.switch_mlp, BlockSwitchGLU) and isinstance(self.shared_expert, BlockMLP):
            ys = decode_products(self.switch_mlp, self.shared_expert, x, idx, w, g, route_step=step)
        if ys is None and step is not None:
            launch_route(step)
        if ys is not None and ys[0] is None:
            return ys[1]  # the shared expert's down product formed the combine
        y, s = ys if ys is not None else (self.switch_mlp(x, idx), self.shared_expert(x))
        out = moe_combine(y, w, g, s)
        if out is None:
            raise ValueError("the combine takes float16 or float32 activations")
        return out


_Routed = SparseMoeBlock


class FusedResidual:
    """The model's hyper-connection (`GatedResidual`) between two blocks: the previous block's output is added
    into the residual streams and the next block's input is read from them, in three sm_100a launches
    (`smoe_hyper_connection`; strata_mlx/fused.py:280-323).

    `gr` has the model's weights: `hc_norm.weight` (hc d), `input_mix_weight_down.weight` (rank, hc d),
    `input_mix_weight_up.weight` (hc d, rank), `block_inject_weight` (None, or with `.weight` (hc, hc d)) and `hc`,
    as torch CUDA tensors of the activations' type. Any window of tokens takes the same kernels, and a token gets
    the same bits alone as in a window."""

    def __init__(self, gr, eps: float = 1e-6):
        self.norm = gr.hc_norm.weight
        self.down, self.up = gr.input_mix_weight_down.weight, gr.input_mix_weight_up.weight
        inj = getattr(gr, "block_inject_weight", None)
        self.inject_w = inj.weight if inj is not None else None
        self.rank, self.wide = self.down.shape
        self.hc, self.eps = int(gr.hc), eps
        _lib.require_cuda(self.norm, self.down, self.up, self.inject_w)

    def __call__(self, before: torch.Tensor, out: torch.Tensor, inject_in: torch.Tensor):
        """Inputs: the streams before the write, before (1, T, hc d); the previous block's output, out (1, T, d);
        its per-stream weights, inject_in (1, T, hc). The new residual is before + out * inject_in.

        Outputs: the next block's input (1, T, d), the new residual (1, T, hc d), and the weights that block's
        own output will be written back with (1, T, hc); inject_in itself where there is no inject weight."""
        _lib.require_cuda(before, out, inject_in)
        T, d, dtype = before.shape[1], out.shape[2], before.dtype
        if out.dtype != dtype or inject_in.dtype != dtype or self.down.dtype != dtype:
            raise ValueError("FusedResidual takes weights and activations of one type (float16 or float32)")
        dev = before.device
        mixed = torch.empty((T, d), dtype=dtype, device=dev)
        residual = torch.empty((T, self.wide), dtype=dtype, device=dev)
        inject = torch.empty((T, self.hc), dtype=dtype, device=dev) if self.inject_w is not None else None
        nbytes = int(_lib.lib().smoe_hyper_workspace_size(T, self.hc, d, self.rank))
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
        spec = _lib.SmoeHyper(self.norm.data_ptr(), self.down.data_ptr(), self.up.data_ptr(),
                              self.inject_w.data_ptr() if self.inject_w is not None else None, self.hc, d, self.rank,
                              self.eps, _lib.dtype_code(dtype))
        _lib.call("smoe_hyper_connection", ctypes.byref(spec), _lib.ptr(before.reshape(T, -1).contiguous()),
                  _lib.ptr(out.reshape(T, d).contiguous()), _lib.ptr(inject_in.reshape(T, self.hc).contiguous()), T,
                  _lib.ptr(mixed), _lib.ptr(residual), _lib.ptr(inject), _lib.ptr(ws), ws.numel(), _lib.stream())
        return mixed[None], residual[None], (inject[None] if inject is not None else inject_in)


def install_routers(layers) -> None:
    """Swap each `layer.mlp.gate` of `layers` for a WindowLinear over its weight, so that router products run on
    the float32-summing kernel (strata_mlx/fused.py:500-507)."""
    for layer in layers:
        mlp = getattr(layer, "mlp", None)
        if mlp is None:
            continue
        gate = getattr(mlp, "gate", None)
        if gate is not None and not isinstance(gate, WindowLinear):
            mlp.gate = WindowLinear(gate)


class GraphedBlock:
    """A MoE block captured once as a CUDA graph for a fixed number of tokens: a decode engine's step.

    Calling it copies x into the graph's static input, replays every launch of `block(x)` without host
    work in between, and returns the graph's static output (overwritten by the next call). Kernels, shapes
    and numerics are those of `block(x)`.

    With `host_io` the step's copies are in the graph too: the host-to-device copy of the token from a pinned
    host buffer and the device-to-host copy of the result into another, so a step is one graph launch. Call it
    with a host tensor; it returns the pinned host result, valid once the stream has reached the step
    (`torch.cuda.current_stream().synchronize()`, or `ready.synchronize()`). A call first waits for this graph's
    previous replay to have read its input buffer."""

    def __init__(self, block, tokens: int, hidden: int, dtype=torch.float16, device=None, host_io: bool = False):
        device = device or torch.device("cuda", torch.cuda.current_device())
        self.block, self.host_io = block, host_io
        self.x = torch.zeros(tokens, hidden, dtype=dtype, device=device)
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            for _ in range(2):  # load the library, size the allocator's pool
                out = block(self.x)
        torch.cuda.current_stream(device).wait_stream(side)
        if host_io:
            self.host_x = torch.zeros(tokens, hidden, dtype=dtype).pin_memory()
            self.host_out = torch.empty(tuple(out.shape), dtype=out.dtype).pin_memory()
            self.ready = torch.cuda.Event()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            if host_io:
                self.x.copy_(self.host_x, non_blocking=True)
            self.out = block(self.x)
            if host_io:
                self.host_out.copy_(self.out, non_blocking=True)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if self.host_io:
            self.ready.synchronize()  # (the previous replay has read host_x and filled host_out)
            if x.data_ptr() != self.host_x.data_ptr():
                self.host_x.copy_(x.reshape(self.host_x.shape))
            self.graph.replay()
            self.ready.record()
            return self.host_out
        self.x.copy_(x.reshape(self.x.shape), non_blocking=True)
        self.graph.replay()
        return self.out
