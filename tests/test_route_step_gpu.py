"""The route taken into the gate / up launch (smoe_route_matvec_batch) against the route and the batch as two
calls, through the C ABI: the same choice, weights, shared gate and rank's view bit for bit, the same products
within the batch's bar, and the launch number moving on once per fused launch (the fused kernel ran, not the two
calls). Its bounded wait for the route runs out when a test withholds the route: a status the host reads, no fault.

The route restates `_Routed.__call__`'s start (strata_mlx/fused.py:487-491); the products `switch_mlp`'s and
`shared_expert`'s gate and up (strata_mlx/blocks.py:939-986, strata_mlx/load.py:419-421).
"""

import ctypes

import numpy as np
import pytest

from oracle import quants as Q

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
from strata_mlx_b200 import _lib  # noqa: E402
from strata_mlx_b200 import blocks as B  # noqa: E402
from strata_mlx_b200 import fused as F  # noqa: E402


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def make(rng, H, F_, E, Fs, routed_kind="IQ3_S"):
    def stack(kind, experts, rows, cols):
        per = Q.TYPES[kind][1]
        return dev(Q.random_blocks(kind, experts * rows * cols // per, rng, normal=0.001).reshape(-1))

    gate = B.BlockSwitchLinear(stack(routed_kind, E, F_, H), routed_kind, (E, F_, H))
    up = B.BlockSwitchLinear(stack(routed_kind, E, F_, H), routed_kind, (E, F_, H))
    sg = B.BlockLinear(stack("Q8_0", 1, Fs, H), "Q8_0", (Fs, H)).stack
    su = B.BlockLinear(stack("Q8_0", 1, Fs, H), "Q8_0", (Fs, H)).stack
    router = F.WindowLinear(dev((0.02 * rng.standard_normal((E, H))).astype(np.float16)))
    sgate = F.WindowLinear(dev((0.02 * rng.standard_normal((1, H))).astype(np.float16)))
    return gate, up, sg, su, router, sgate


def products(gate, up, sg, su, x, idx, k, route=None):
    tokens = x.shape[0]
    pairs = tokens * k
    flat = idx.reshape(-1)
    zeros = B._zeros_idx(tokens, x.device)
    out = [torch.empty((pairs, gate.output_dims), dtype=x.dtype, device=x.device),
           torch.empty((pairs, up.output_dims), dtype=x.dtype, device=x.device),
           torch.empty((tokens, sg.output_dims), dtype=x.dtype, device=x.device),
           torch.empty((tokens, su.output_dims), dtype=x.dtype, device=x.device)]
    B.matvec_batch([B._problem(gate, flat, pairs, k, out[0], x=x), B._problem(up, flat, pairs, k, out[1], x=x),
                    B._problem(sg, zeros, tokens, 1, out[2], x=x), B._problem(su, zeros, tokens, 1, out[3], x=x)],
                   route=route)
    return out


def status(clear):
    v = ctypes.c_int(-1)
    assert _lib.lib().smoe_matvec_status(ctypes.byref(v), int(clear)) == 0
    return v.value


@pytest.mark.parametrize("tokens", [1, 3, 8, 16])
@pytest.mark.parametrize("local", [None, (64, 96)])
def test_the_route_in_the_gate_up_launch_is_the_route_then_the_batch(cuda, tokens, local):
    """Up to 8 tokens in one launch; 16 as the two calls, through counters the fused launches use too."""
    rng = np.random.default_rng(tokens * 31 + (0 if local is None else 1))
    H, F_, E, Fs, k = 1024, 512, 256, 1024, 8
    gate, up, sg, su, router, sgate = make(rng, H, F_, E, Fs)
    assert status(True) in (0, _lib.ETIMEOUT)
    for trial in range(3):  # (the launch number and the arrival count carry over from call to call)
        x = dev(rng.standard_normal((tokens, H)).astype(np.float16))
        ref = F.route(router, sgate, x, k, local=local)
        want = products(gate, up, sg, su, x, ref[3] if local else ref[0], k)
        got_r = F.route(router, sgate, x, k, local=local, defer=True)
        step = got_r[-1]
        counters = step._keep[7]
        before = int(counters[1].item())
        got = products(gate, up, sg, su, x, got_r[3] if local else got_r[0], k, route=step)
        torch.cuda.synchronize()
        assert int(counters[1].item()) == before + (1 if tokens <= 8 else 0), "the fused launch did (not) run"
        assert int(counters[0].item()) == 0
        for a, b in zip(got_r[:-1], ref):
            assert torch.equal(a, b)
        for a, b in zip(got, want):
            assert a.shape == b.shape
            bar = 1e-3 * b.float().abs().max().item()
            assert (a.float() - b.float()).abs().max().item() <= bar
    assert status(False) == 0


def test_a_block_calls_the_fused_route_step_by_step_and_in_a_graph(cuda, monkeypatch):
    """The block's own call (SparseMoeBlock at decode, FUSED_ROUTE on) goes through the fused launch, eagerly and
    replayed from a CUDA graph, call after call with the same bits."""
    monkeypatch.setattr(F, "FUSED_ROUTE", True)
    rng = np.random.default_rng(5)
    H, F_, E, Fs, k = 1024, 512, 256, 1024, 8
    gate, up, sg, su, router, sgate = make(rng, H, F_, E, Fs)

    def stack(kind, experts, rows, cols):
        return dev(Q.random_blocks(kind, experts * rows * cols // Q.TYPES[kind][1], rng, normal=0.001).reshape(-1))

    down = B.BlockSwitchLinear(stack("IQ3_S", E, H, F_), "IQ3_S", (E, H, F_))
    sdown = B.BlockLinear(stack("Q8_0", 1, H, Fs), "Q8_0", (H, Fs))
    block = F.SparseMoeBlock(router, B.BlockSwitchGLU(gate, up, down),
                             B.BlockMLP(B.BlockLinear(sg.blocks, "Q8_0", (Fs, H)),
                                        B.BlockLinear(su.blocks, "Q8_0", (Fs, H)), sdown), sgate, k)
    x = dev(rng.standard_normal((1, H)).astype(np.float16))
    first = block(x)
    key = [key for key in F._COUNTERS if key[2]]
    assert key, "the block did not take the deferred route"
    counters = F._COUNTERS[key[0]]
    n0 = int(counters[1].item())
    for _ in range(4):
        assert torch.equal(block(x).view(torch.int16), first.view(torch.int16))
    torch.cuda.synchronize()
    assert int(counters[1].item()) == n0 + 4
    step = F.GraphedBlock(block, 1, H, torch.float16, x.device)
    for _ in range(4):
        assert torch.equal(step(x).view(torch.int16), first.view(torch.int16))
    assert status(False) == 0


def test_a_route_that_never_comes_is_a_status_the_host_reads(cuda):
    """With the route withheld (a test hook: the launch never announces it) and a short bound, the routed
    products' waits for it run out: SMOE_ETIMEOUT in the status word, the copies in flight land, the device
    stays usable; back to the default, the same call is exact again."""
    lib = _lib.lib()
    rng = np.random.default_rng(77)
    H, F_, E, Fs, k = 1024, 512, 256, 1024, 8
    gate, up, sg, su, router, sgate = make(rng, H, F_, E, Fs)
    x = dev(rng.standard_normal((1, H)).astype(np.float16))
    ref = F.route(router, sgate, x, k)
    want = products(gate, up, sg, su, x, ref[0], k)
    torch.cuda.synchronize()
    assert status(True) in (0, _lib.ETIMEOUT)
    try:
        assert lib.smoe_matvec_wait_test(2, 2) == 0
        for _ in range(2):
            r = F.route(router, sgate, x, k, defer=True)
            products(gate, up, sg, su, x, r[0], k, route=r[-1])
        assert status(True) == _lib.ETIMEOUT
    finally:
        assert lib.smoe_matvec_wait_test(-1, 0) == 0
    r = F.route(router, sgate, x, k, defer=True)
    got = products(gate, up, sg, su, x, r[0], k, route=r[-1])
    torch.cuda.synchronize()
    assert status(False) == 0
    assert torch.equal(r[0], ref[0])
    for a, b in zip(got, want):
        assert (a.float() - b.float()).abs().max().item() <= 1e-3 * b.float().abs().max().item()
