"""The one-launch decode step (smoe_decode_layer) against the four launches it replaces and the CPU oracle.

The step for one token: router, top-k with the softmax over the chosen, the shared gate, the routed and shared
experts' SwiGLU products and the combine (the reference's `_Routed.__call__`, strata_mlx/fused.py:484-497).
Bars: logits, expert indices, their weights and the shared gate value the same bits as the separate calls;
the output within rel-L2 1e-3 of the separate calls and of the oracle; no grid-barrier wait gave up; the same
results from a CUDA graph's replays.
"""

import numpy as np
import pytest

from oracle import moe as M

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
from strata_mlx_b200 import fused as F  # noqa: E402

from test_moe_gpu import build_block, dev, make_layer, rel_l2  # noqa: E402


@pytest.fixture(autouse=True)
def layer_kernel_on(monkeypatch):
    """These tests run SparseMoeBlock through the one-launch step (off by default)."""
    monkeypatch.setattr(F, "LAYER_KERNEL", True)


def four_launches(block, x, monkeypatch):
    """block(x) through route / batched gate-up / down / down+combine, and the route's outputs."""
    with monkeypatch.context() as m:
        m.setattr(F, "LAYER_KERNEL", False)
        out = block(x)
        idx, w, g = F.route(block.gate, block.shared_expert_gate, x, block.top_k)
    return out, idx, w, g


def layer_outputs(block, x):
    """The one-launch step's output, choice, weights, gate value and logits."""
    out = F.decode_layer(block, x)
    assert out is not None
    return out


@pytest.mark.parametrize("E, H, F_, Fs, k", [(64, 1024, 512, 512, 8), (16, 512, 1024, 256, 4), (256, 4096, 1536, 4096, 8)])
def test_the_one_launch_step_is_the_four_launches(cuda, monkeypatch, E, H, F_, Fs, k):
    rng = np.random.default_rng(E + H)
    routed, shared, router, sgate = make_layer(rng, H, F_, E, Fs, ("IQ3_S",) * 3, "Q8_0")
    block = build_block(routed, shared, router, sgate, k)
    for step in range(3):  # launches after the first count their barriers on from the first's
        x = dev(rng.standard_normal((1, H)).astype(np.float16))
        got = block(x)
        want, idx, w, g = four_launches(block, x, monkeypatch)
        assert got.shape == want.shape == (1, H)
        assert rel_l2(got.float().cpu().numpy(), want.float().cpu().numpy()) <= 1e-3
        assert not F.decode_layer_failed(x, block)


def test_the_one_launch_step_writes_the_routers_choice(cuda, monkeypatch):
    """The step's logits, indices, weights and gate value are the separate route call's bits."""
    from strata_mlx_b200 import _lib

    rng = np.random.default_rng(5)
    E, H, F_, Fs, k = 64, 1024, 512, 512, 8
    routed, shared, router, sgate = make_layer(rng, H, F_, E, Fs, ("IQ3_S",) * 3, "Q8_0")
    block = build_block(routed, shared, router, sgate, k)
    x = dev(rng.standard_normal((1, H)).astype(np.float16))
    _, idx, w, g = four_launches(block, x, monkeypatch)
    logits_want = block.gate(x)
    # the same call decode_layer makes, keeping its outputs
    sw, sh = block.switch_mlp, block.shared_expert
    scratch = torch.zeros(int(_lib.lib().smoe_decode_layer_scratch(H, k, F_, Fs)), dtype=torch.uint8, device="cuda")
    logits = torch.empty(E, dtype=torch.float32, device="cuda")
    idx_got = torch.empty(k, dtype=torch.uint32, device="cuda")
    w_got = torch.empty(k, dtype=torch.float32, device="cuda")
    g_got = torch.empty(1, dtype=torch.float16, device="cuda")
    out = torch.empty(H, dtype=torch.float16, device="cuda")
    spec = _lib.SmoeDecodeLayer(
        _lib.ptr(block.gate.weight), _lib.ptr(block.shared_expert_gate.weight), E, H, k, 21,
        _lib.ptr(sw.gate_proj.blocks), _lib.ptr(sw.up_proj.blocks), _lib.ptr(sw.down_proj.blocks), F_, 8,
        _lib.ptr(sh.gate_proj.blocks), _lib.ptr(sh.up_proj.blocks), _lib.ptr(sh.down_proj.blocks), Fs,
        _lib.ptr(logits), _lib.ptr(idx_got), _lib.ptr(w_got), _lib.ptr(g_got), _lib.ptr(out), _lib.ptr(scratch))
    import ctypes

    _lib.call("smoe_decode_layer", ctypes.byref(spec), _lib.ptr(x), _lib.stream())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(logits.cpu().numpy(), logits_want.reshape(-1).cpu().numpy())
    np.testing.assert_array_equal(idx_got.cpu().numpy(), idx.reshape(-1).cpu().numpy())
    np.testing.assert_array_equal(w_got.cpu().numpy(), w.reshape(-1).cpu().numpy())
    np.testing.assert_array_equal(g_got.view(torch.int16).cpu().numpy(), g.reshape(-1).view(torch.int16).cpu().numpy())


def test_a_graph_of_one_launch_steps_replays_the_same(cuda):
    """Captured in a CUDA graph (a decode engine's step) the cooperative launch gives the eager results."""
    rng = np.random.default_rng(7)
    E, H, F_, Fs, k = 64, 1024, 512, 512, 8
    routed, shared, router, sgate = make_layer(rng, H, F_, E, Fs, ("IQ3_S",) * 3, "Q8_0")
    block = build_block(routed, shared, router, sgate, k)
    xs = [dev(rng.standard_normal((1, H)).astype(np.float16)) for _ in range(3)]
    eager = [block(x).clone() for x in xs]
    gb = F.GraphedBlock(block, 1, H, torch.float16, torch.device("cuda"))
    for _ in range(2):
        for x, want in zip(xs, eager):
            got = gb(x)
            torch.cuda.synchronize()
            assert torch.equal(got.reshape(-1), want.reshape(-1))
    assert not F.decode_layer_failed(xs[0], block)


def test_the_one_launch_step_at_baseline_shapes_is_the_oracles(cuda):
    """Benchmark configuration 2 (hidden 4096, 256 IQ3_S experts of ffn 1536, top-8, Q8_0 shared expert of 4096)."""
    rng = np.random.default_rng(12)
    H, F_, E, Fs, k = 4096, 1536, 256, 4096, 8
    routed, shared, router, sgate = make_layer(rng, H, F_, E, Fs, ("IQ3_S",) * 3, "Q8_0")
    block = build_block(routed, shared, router, sgate, k)
    x = rng.standard_normal((1, H)).astype(np.float16)
    got = layer_outputs(block, dev(x)).cpu().numpy()
    logits = block.gate(dev(x)).cpu().numpy()
    want, idx, w, _ = M.moe_block(x, router, k, routed, shared, sgate, logits=logits)
    assert rel_l2(got, want) <= 1e-3


def test_a_grid_barrier_that_never_fills_is_a_status_the_host_reads(cuda, monkeypatch):
    """With one CTA's first arrival withheld (a test hook), every wait at the first grid barrier runs out after
    about a second and the later barriers' waits too: the step's status reads 1, nothing more is copied, the
    copies in flight land, and the device stays usable. With the scratch zeroed again (its barrier count is off
    after a wait gave up) the next step is the four launches' again and its status is clear. No fault, no trap."""
    from strata_mlx_b200 import _lib

    rng = np.random.default_rng(44)
    E, H, F_, Fs, k = 64, 1024, 512, 512, 8
    routed, shared, router, sgate = make_layer(rng, H, F_, E, Fs, ("IQ3_S",) * 3, "Q8_0")
    block = build_block(routed, shared, router, sgate, k)
    x = dev(rng.standard_normal((1, H)).astype(np.float16))
    block(x)
    assert not F.decode_layer_failed(x, block)
    lib = _lib.lib()
    try:
        assert lib.smoe_decode_layer_wait_test(1) == 0
        block(x)
        torch.cuda.synchronize()
        assert F.decode_layer_failed(x, block)
    finally:
        assert lib.smoe_decode_layer_wait_test(0) == 0
    F._LAYER_SCRATCH[(str(x.device), H, k, F_, Fs)].zero_()
    got = block(x)
    want, _, _, _ = four_launches(block, x, monkeypatch)
    assert rel_l2(got.float().cpu().numpy(), want.float().cpu().numpy()) <= 1e-3
    assert not F.decode_layer_failed(x, block)
