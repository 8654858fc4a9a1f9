"""The router, top-k, combine and the whole MoE block on the GPU against the CPU oracle, through the C ABI.

Mirrors the reference's tests/test_fused.py (cited per test). Bars: router logits within 1e-5 of the largest
(float64 oracle) and the same bits for a token alone as inside a window; top-k indices exactly those of a
stable arg-sort of the kernel's own logits; the combine bit-equal to the oracle's restatement of MLX's order;
the MoE block's output within rel-L2 1e-3 of the oracle (the path's stated tolerance), its expert
indices exact.
"""

import numpy as np
import pytest

from oracle import moe as M
from oracle import quants as Q

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
from strata_mlx_b200 import blocks as B  # noqa: E402
from strata_mlx_b200 import fused as F  # noqa: E402


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def rel_l2(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return np.linalg.norm(got - want) / np.linalg.norm(want)


@pytest.mark.parametrize("tokens", [1, 3, 8, 20, 1180])
def test_a_router_product_in_float32_from_float16_weights(cuda, tokens):
    """tests/test_fused.py:90-106."""
    rng = np.random.default_rng(tokens)
    w = (0.02 * rng.standard_normal((256, 4096))).astype(np.float16)
    x = rng.standard_normal((1, tokens, 4096)).astype(np.float16)
    router = F.WindowLinear(dev(w))
    got = router(dev(x))
    assert got.shape == (1, tokens, 256) and got.dtype == torch.float32
    want = M.router_logits(w, x[0])
    assert np.abs(got[0].cpu().numpy() - want).max() <= 1e-5 * np.abs(want).max()
    if tokens <= 20:  # a token's sum does not depend on the window it is in
        alone = torch.cat([router(dev(x[:, t : t + 1])) for t in range(tokens)], dim=1)
        assert torch.equal(alone, got)


@pytest.mark.parametrize("tokens", [1, 5, 8, 9, 20])
@pytest.mark.parametrize("experts, k", [(256, 8), (60, 4), (1024, 16)])
@pytest.mark.parametrize("dtype", [np.float16, np.float32])
@pytest.mark.parametrize("with_gate", [True, False])
def test_route_in_one_launch_is_the_three_calls(cuda, tokens, experts, k, dtype, with_gate):
    """The fused start of the block (router, top-k with softmax, shared gate) gives the bits of the separate
    calls (strata_mlx/fused.py:487-491), call after call (its counters come back to zero)."""
    rng = np.random.default_rng(tokens * 7 + experts + k)
    w = dev((0.02 * rng.standard_normal((experts, 512))).astype(np.float16))
    gw = dev((0.02 * rng.standard_normal((1, 512))).astype(np.float16))
    router, sgate = F.WindowLinear(w), F.WindowLinear(gw)
    for trial in range(3):
        x = dev(rng.standard_normal((tokens, 512)).astype(dtype))
        idx, wt, g = F.route(router, sgate if with_gate else None, x, k)
        want_idx, want_w = F.top_k_softmax(router(x), k)
        assert torch.equal(idx, want_idx) and torch.equal(wt, want_w)
        if with_gate:
            assert torch.equal(g, sgate(x).to(x.dtype))
        else:
            assert g is None


@pytest.mark.parametrize("tokens", [1, 3, 8, 40])
@pytest.mark.parametrize("ties", [False, True])
@pytest.mark.parametrize("n, k", [(512, 10), (256, 8), (100, 3)])
def test_the_routers_choice_is_argpartitions(cuda, tokens, ties, n, k):
    """tests/test_fused.py:109-120: the stable order, ties to the lower index, 20 trials."""
    rng = np.random.default_rng(tokens + 10 * ties + n)
    for _ in range(20):
        logits = rng.standard_normal((1, tokens, n)).astype(np.float32)
        if ties:
            logits = np.round(logits * 4) / 4
        idx, w = F.top_k_softmax(dev(logits), k)
        np.testing.assert_array_equal(idx.cpu().numpy().astype(np.int64), M.top_k(logits, k).astype(np.int64))
        want_w = M.softmax_chosen(logits, M.top_k(logits, k))
        assert np.abs(w.cpu().numpy() - want_w).max() <= 1e-6
        assert torch.equal(F.top_k(dev(logits), k), idx)


@pytest.mark.parametrize("tokens", [1, 3, 8, 16, 40])
@pytest.mark.parametrize("k, d", [(10, 2560), (8, 4096), (8, 1028)])
def test_the_end_of_the_moe_block_is_the_restated_bits(cuda, tokens, k, d):
    """tests/test_fused.py:124-138: bit-equal to (y * w).sum(-2).astype(half) + sigmoid(g) * s in MLX's order."""
    rng = np.random.default_rng(tokens)
    for _ in range(5):
        y = (rng.standard_normal((tokens, k, d)) * 0.5).astype(np.float16)
        lw = rng.standard_normal((tokens, k)).astype(np.float32)
        w = np.exp(lw) / np.exp(lw).sum(-1, keepdims=True)
        w = w.astype(np.float32)
        g = (2 * rng.standard_normal((tokens,))).astype(np.float16)
        s = (0.5 * rng.standard_normal((tokens, d))).astype(np.float16)
        got = F.moe_combine(dev(y), dev(w), dev(g[:, None]), dev(s)).cpu().numpy()
        want = M.combine(y, w, g, s)
        np.testing.assert_array_equal(got.view(np.uint16), want.view(np.uint16))


def make_layer(rng, H, F_, E, Fs, kinds, shared_kind, scale=0.001):
    """A layer of random blocks: routed (gate, up, down) stacks of the given kinds, the shared expert, the
    router and the shared expert's gate. Block scales are |N(0, scale)|; the benchmark's 0.02 makes the down
    product overflow float16 at hidden 4096 (gate ~ 200, swiglu ~ 4e4), so parity is taken at 0.001 where
    every output is finite."""
    def blocks_of(kind, rows, cols, experts=1):
        per, _ = B.BLOCK[kind]
        return Q.random_blocks(kind, experts * rows * cols // per, rng, normal=scale).reshape(-1)

    gk, uk, dk = kinds
    routed = [(blocks_of(gk, F_, H, E), gk, (E, F_, H)), (blocks_of(uk, F_, H, E), uk, (E, F_, H)),
              (blocks_of(dk, H, F_, E), dk, (E, H, F_))]
    shared = [(blocks_of(shared_kind, Fs, H), shared_kind, (Fs, H)), (blocks_of(shared_kind, Fs, H), shared_kind, (Fs, H)),
              (blocks_of(shared_kind, H, Fs), shared_kind, (H, Fs))]
    router = (0.02 * rng.standard_normal((E, H))).astype(np.float16)
    sgate = (0.02 * rng.standard_normal((1, H))).astype(np.float16)
    return routed, shared, router, sgate


def build_block(routed, shared, router, sgate, k):
    sw = B.BlockSwitchGLU(*(B.BlockSwitchLinear(dev(b), kind, shape) for b, kind, shape in routed))
    sh = B.BlockMLP(*(B.BlockLinear(dev(b), kind, shape) for b, kind, shape in shared))
    return F.SparseMoeBlock(dev(router), sw, sh, dev(sgate), k)


@pytest.mark.parametrize("tokens", [1, 5, 16])
@pytest.mark.parametrize("kinds", [("IQ3_S", "IQ3_S", "IQ3_S"), ("Q4_K", "IQ4_XS", "Q6_K"), ("Q2_K", "Q3_K", "IQ3_XXS")])
def test_the_moe_block_is_the_oracles(cuda, tokens, kinds):
    rng = np.random.default_rng(tokens)
    H, F_, E, Fs, k = 512, 256, 16, 512, 4
    routed, shared, router, sgate = make_layer(rng, H, F_, E, Fs, kinds, "Q8_0")
    block = build_block(routed, shared, router, sgate, k)
    x = rng.standard_normal((tokens, H)).astype(np.float16)
    got = block(dev(x)).cpu().numpy()
    logits = block.gate(dev(x)).cpu().numpy()
    want, idx, w, _ = M.moe_block(x, router, k, routed, shared, sgate, logits=logits)
    np.testing.assert_array_equal(F.top_k(dev(logits), k).cpu().numpy().astype(np.int64), idx.astype(np.int64))
    assert rel_l2(got, want) <= 1e-3


def test_a_prompt_chunk_through_tiles_and_the_shared_gemm_is_the_oracles(cuda):
    """Enough pairs for the routed tiles (TILES_FROM) and tokens for the shared expert's tile product."""
    from strata_mlx_b200 import blocks as Bm

    rng = np.random.default_rng(9)
    H, F_, E, Fs, k, tokens = 512, 256, 16, 512, 4, 450
    routed, shared, router, sgate = make_layer(rng, H, F_, E, Fs, ("Q2_K", "Q2_K", "Q2_K"), "Q8_0")
    block = build_block(routed, shared, router, sgate, k)
    assert tokens * k >= Bm.TILES_FROM and tokens >= Bm.GEMM_FROM
    x = rng.standard_normal((tokens, H)).astype(np.float16)
    got = block(dev(x)).cpu().numpy()
    logits = block.gate(dev(x)).cpu().numpy()
    want, idx, w, _ = M.moe_block(x, router, k, routed, shared, sgate, logits=logits)
    assert rel_l2(got, want) <= 1e-3


def test_the_decode_layer_at_baseline_shapes_is_the_oracles(cuda):
    """Benchmark configuration 2: hidden 4096, 256 experts of IQ3_S (gate/up 1536 x 4096, down 4096 x 1536), top-8,
    shared expert ffn 4096 in Q8_0, batch 1."""
    rng = np.random.default_rng(2)
    H, F_, E, Fs, k = 4096, 1536, 256, 4096, 8
    routed, shared, router, sgate = make_layer(rng, H, F_, E, Fs, ("IQ3_S",) * 3, "Q8_0")
    block = build_block(routed, shared, router, sgate, k)
    x = rng.standard_normal((1, H)).astype(np.float16)
    got = block(dev(x)).cpu().numpy()
    logits = block.gate(dev(x)).cpu().numpy()
    assert np.abs(logits - M.router_logits(router, x)).max() <= 1e-5 * np.abs(logits).max()
    want, idx, w, _ = M.moe_block(x, router, k, routed, shared, sgate, logits=logits)
    assert rel_l2(got, want) <= 1e-3


def test_a_prompt_chunk_at_baseline_shapes_is_the_oracles(cuda):
    """Benchmark configuration 3 at its shapes: 1,180 tokens, hidden 4096, ffn 1536, Q2_K routed experts, top-8 of
    router logits biased so expert load is Zipf-skewed (s = 1.1), the Q8_0 shared expert of ffn 4096 on the tile
    product. 24 experts where the benchmark has 256 (the oracle decodes every expert hit on the CPU: 72 Q2_K
    matrices of 6.3 M weights); every expert is hit, the busiest by most tokens. Indices exact, the block within
    rel-L2 1e-3."""
    rng = np.random.default_rng(33)
    H, F_, E, Fs, k, T = 4096, 1536, 24, 4096, 8, 1180
    routed, shared, router, sgate = make_layer(rng, H, F_, E, Fs, ("Q2_K",) * 3, "Q8_0")
    rank = np.empty(E)
    rank[rng.permutation(E)] = np.arange(1, E + 1)
    logp = -1.1 * np.log(rank)
    logp -= np.log(np.exp(logp).sum())
    u = rng.standard_normal(H)
    u /= np.linalg.norm(u)
    router = (router.astype(np.float64) + logp[:, None] * u[None, :]).astype(np.float16)
    x = rng.standard_normal((T, H))
    x = (x - (x @ u)[:, None] * u[None, :] + u[None, :]).astype(np.float16)
    block = build_block(routed, shared, router, sgate, k)
    got = block(dev(x)).cpu().numpy()
    logits = block.gate(dev(x)).cpu().numpy()
    assert np.abs(logits - M.router_logits(router, x)).max() <= 1e-5 * np.abs(logits).max()
    want, idx, w, _ = M.moe_block(x, router, k, routed, shared, sgate, logits=logits)
    np.testing.assert_array_equal(F.top_k(dev(logits), k).cpu().numpy().astype(np.int64), idx.astype(np.int64))
    counts = np.bincount(idx.reshape(-1), minlength=E)
    assert counts.min() > 0 and counts.max() > 2 * counts.mean()  # skewed, every expert hit
    assert np.isfinite(got).all()
    assert rel_l2(got, want) <= 1e-3


def test_a_graph_with_its_host_copies_gives_the_eager_bits(cuda):
    """GraphedBlock(host_io=True): the token's copy in from pinned host memory and the result's copy out are in
    the graph; a step returns the eager block's bits on the host, calls in a row included."""
    rng = np.random.default_rng(12)
    H, F_, E, Fs, k = 512, 256, 16, 512, 4
    routed, shared, router, sgate = make_layer(rng, H, F_, E, Fs, ("IQ3_S",) * 3, "Q8_0")
    block = build_block(routed, shared, router, sgate, k)
    xs = [rng.standard_normal((1, H)).astype(np.float16) for _ in range(3)]
    eager = [block(dev(x)).cpu().numpy() for x in xs]
    gb = F.GraphedBlock(block, 1, H, torch.float16, cuda, host_io=True)
    for _ in range(2):
        for x, want in zip(xs, eager):
            got = gb(torch.from_numpy(x))
            gb.ready.synchronize()
            assert not got.is_cuda and got.is_pinned()
            np.testing.assert_array_equal(got.numpy().view(np.uint16), want.view(np.uint16))


@pytest.mark.parametrize("lo, count", [(0, 64), (64, 64), (192, 64), (0, 256), (96, 32)])
def test_route_with_the_ranks_view_is_route_then_localize(cuda, lo, count):
    """smoe_route_local: the same logits, choice, weights and gate bits as smoe_route, and the local indices
    smoe_localize gives for the experts [lo, lo + count)."""
    from strata_mlx_b200 import _lib

    rng = np.random.default_rng(lo + count)
    E, H, k, T = 256, 4096, 8, 3
    router = dev((0.02 * rng.standard_normal((E, H))).astype(np.float16))
    sgate = dev((0.02 * rng.standard_normal((1, H))).astype(np.float16))
    x = dev(rng.standard_normal((T, H)).astype(np.float16))
    gate, sg = F.WindowLinear(router), F.WindowLinear(sgate)
    idx, w, g = F.route(gate, sg, x, k)
    idx2, w2, g2, lidx = F.route(gate, sg, x, k, local=(lo, count))
    assert torch.equal(idx, idx2) and torch.equal(w, w2) and torch.equal(g, g2)
    want = torch.empty_like(idx)
    flat = idx.reshape(-1).contiguous()
    _lib.call("smoe_localize", _lib.ptr(flat), flat.numel(), lo, count, _lib.ptr(want), _lib.stream())
    assert torch.equal(lidx.reshape(-1), want.reshape(-1))
