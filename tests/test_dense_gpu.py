"""The dense steps around the MoE block on the GPU against the oracle: the hyper-connection (strata_mlx/fused.py
FusedResidual, with the tolerances of the reference's tests/test_fused.py:19-37), Q3_K planes and Q6_K parts
(bit for bit against the fixture made by the reference's own code), their window products (a token gets the same
bits alone as in a window) and their weights as floats (the block decoders' bits)."""

import os
import types

import numpy as np
import pytest

from oracle import dense as D
from oracle import quants as Q

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

DENSE = os.path.join(os.path.dirname(__file__), "golden", "dense.npz")


def _gr(rng, hc, d, rank, combine, dtype, dev):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a.astype(dtype))).to(dev)  # noqa: E731
    ns = types.SimpleNamespace
    w = {"norm": 1 + 0.2 * rng.standard_normal(hc * d), "down": 0.05 * rng.standard_normal((rank, hc * d)),
         "up": 0.05 * rng.standard_normal((hc * d, rank)),
         "inject": 0.05 * rng.standard_normal((hc, hc * d)) if combine else None}
    gr = ns(hc=hc, hc_norm=ns(weight=t(w["norm"])), input_mix_weight_down=ns(weight=t(w["down"])),
            input_mix_weight_up=ns(weight=t(w["up"])),
            block_inject_weight=ns(weight=t(w["inject"])) if combine else None)
    host = {k: (v.astype(dtype) if v is not None else None) for k, v in w.items()}
    return gr, host


@pytest.mark.parametrize("dtype, tol", [(np.float32, 2e-5), (np.float16, 4e-3)])
@pytest.mark.parametrize("tokens", [1, 2, 5, 8, 11])
@pytest.mark.parametrize("combine", [True, False])
def test_hyper_connection_is_the_oracles(cuda, dtype, tol, tokens, combine):
    from strata_mlx_b200.fused import FusedResidual

    rng = np.random.default_rng(tokens * 2 + combine)
    hc, d, rank = 4, 96, 24
    gr, w = _gr(rng, hc, d, rank, combine, dtype, cuda)
    before = rng.standard_normal((1, tokens, hc * d)).astype(dtype)
    out = rng.standard_normal((1, tokens, d)).astype(dtype)
    inject_in = (2 * rng.random((1, tokens, hc))).astype(dtype)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    got = FusedResidual(gr)(t(before), t(out), t(inject_in))
    want = D.hyper_connection(before[0], out[0], inject_in[0], w["norm"], w["down"], w["up"], w["inject"], hc, dtype=dtype)
    for g, wv in zip(got, want):
        if wv is None:
            continue
        g = g[0].cpu().numpy()
        assert g.shape == wv.shape and g.dtype == dtype
        assert np.abs(g.astype(np.float64) - wv.astype(np.float64)).max() <= tol * np.abs(wv.astype(np.float64)).max()
    if not combine:
        assert got[2] is not None and torch.equal(got[2], t(inject_in))


@pytest.mark.parametrize("dtype", [np.float32, np.float16])
def test_hyper_connection_gives_a_token_its_bits_alone_and_in_a_window(cuda, dtype):
    """As the reference's tests/test_fused.py:51-71: every token's sums in the same order whatever the window."""
    from strata_mlx_b200.fused import FusedResidual

    rng = np.random.default_rng(7)
    hc, d, rank = 4, 2560, 64
    gr, _ = _gr(rng, hc, d, rank, True, dtype, cuda)
    fused = FusedResidual(gr)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    before = t(rng.standard_normal((1, 12, hc * d)).astype(dtype))
    out = t(rng.standard_normal((1, 12, d)).astype(dtype))
    inject_in = t((2 * rng.random((1, 12, hc))).astype(dtype))
    window = fused(before, out, inject_in)
    for s in (slice(t0, t0 + 1) for t0 in range(12)):
        alone = fused(before[:, s], out[:, s], inject_in[:, s])
        assert all(torch.equal(a, w[:, s]) for a, w in zip(alone, window))
    three = fused(before[:, 2:5], out[:, 2:5], inject_in[:, 2:5])
    assert all(torch.equal(a, w[:, 2:5]) for a, w in zip(three, window))


def test_hyper_connection_with_nothing_before_is_a_plain_read(cuda):
    from strata_mlx_b200.fused import FusedResidual

    rng = np.random.default_rng(6)
    gr, w = _gr(rng, 4, 96, 24, True, np.float32, cuda)
    h = torch.from_numpy(rng.standard_normal((1, 2, 4 * 96)).astype(np.float32)).to(cuda)
    mixed, residual, inject = FusedResidual(gr)(h, torch.zeros((1, 2, 96), device=cuda), torch.zeros((1, 2, 4), device=cuda))
    assert torch.equal(residual, h)
    want = D.hyper_connection(h[0].cpu().numpy(), np.zeros((2, 96)), np.zeros((2, 4)), w["norm"], w["down"], w["up"],
                              w["inject"], 4, dtype=np.float32)
    np.testing.assert_allclose(mixed[0].cpu().numpy(), want[0], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(inject[0].cpu().numpy(), want[2], rtol=1e-4, atol=1e-5)


# ---------------------------------------------------------------- Q3_K planes


def test_q3k_planes_are_the_references_bit_for_bit(cuda):
    from strata_mlx_b200 import blocks as B

    g = np.load(DENSE)
    rows, cols = (int(v) for v in g["shape"])
    p = B.q3k_planes(torch.from_numpy(g["Q3_K/blocks"]).to(cuda), rows, cols)
    np.testing.assert_array_equal(p["hm"].cpu().numpy().view(np.uint32), g["Q3_K/hm"])
    np.testing.assert_array_equal(p["qs"].cpu().numpy().view(np.uint32), g["Q3_K/qs"])
    np.testing.assert_array_equal(p["sc"].cpu().numpy(), g["Q3_K/sc"])
    np.testing.assert_array_equal(p["dd"].cpu().numpy().view(np.uint16), g["Q3_K/dd"])
    want = Q.dequantize(g["Q3_K/blocks"], "Q3_K", (rows, cols))
    for dt, npdt in ((torch.float32, np.float32), (torch.float16, np.float16)):
        got = B.q3k_planes_dequantize(p, rows, cols, dt).cpu().numpy()
        np.testing.assert_array_equal(got.view(np.uint32 if npdt == np.float32 else np.uint16),
                                      want.astype(npdt).view(np.uint32 if npdt == np.float32 else np.uint16))


@pytest.mark.parametrize("rows, cols", [(640, 2560), (1536, 4096), (10240, 2560)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_q3k_planes_window_is_the_oracles_and_keeps_a_tokens_bits(cuda, rows, cols, dtype):
    from strata_mlx_b200 import blocks as B

    rng = np.random.default_rng(rows + cols)
    blocks = Q.random_blocks("Q3_K", rows * cols // 256, rng).reshape(-1)
    p = B.q3k_planes(torch.from_numpy(blocks).to(cuda), rows, cols)
    x = rng.standard_normal((9, cols)).astype(np.float16)
    xd = torch.from_numpy(x).to(cuda).to(dtype)
    got = B.q3k_planes_window(p, rows, cols, xd)
    w = Q.dequantize(blocks, "Q3_K", (rows, cols)).astype(np.float64)
    want = x.astype(np.float64) @ w.T
    bound = 1e-5 * np.abs(w).max() * np.sqrt(cols) * np.abs(x).max() + (1e-3 if dtype == torch.float16 else 0) * np.abs(want).max()
    assert np.abs(got.double().cpu().numpy() - want).max() <= bound
    for t0 in (0, 4, 8):
        assert torch.equal(B.q3k_planes_window(p, rows, cols, xd[t0 : t0 + 1]), got[t0 : t0 + 1])


def test_a_dense_q3k_layer_on_planes_matches_window_matvec_on_its_blocks(cuda):
    """dense.BlockLinear holds Q3_K as planes: a window through them, and a chunk through the planes' floats."""
    from strata_mlx_b200 import blocks as B
    from strata_mlx_b200 import dense as DN

    rng = np.random.default_rng(12)
    rows, cols = 512, 2560
    blocks = torch.from_numpy(Q.random_blocks("Q3_K", rows * cols // 256, rng).reshape(-1)).to(cuda)
    lin = DN.BlockLinear(blocks, "Q3_K", (rows, cols))
    assert lin.planes is not None and lin.nbytes == rows * cols // 256 * B.Q3K_PLANE_BYTES
    x = torch.from_numpy(rng.standard_normal((1, 5, cols)).astype(np.float16)).to(cuda)
    w = Q.dequantize(blocks.cpu().numpy(), "Q3_K", (rows, cols)).astype(np.float64)
    want = x[0].double().cpu().numpy() @ w.T
    for xx in (x, torch.cat([x] * 4, dim=1)):  # a window, and a chunk of 20 tokens
        got = lin(xx).double().cpu().numpy().reshape(-1, rows)[:5]
        assert np.abs(got - want).max() <= 2e-3 * np.abs(want).max()


# ---------------------------------------------------------------- Q6_K parts (ScaledLinear)


def test_q6k_parts_are_the_references_bit_for_bit(cuda):
    from strata_mlx_b200 import dense as DN

    g = np.load(DENSE)
    rows, cols = (int(v) for v in g["shape"])
    codes, scales, d = DN.q6k_parts(torch.from_numpy(g["Q6_K/blocks"]).to(cuda), rows, cols)
    np.testing.assert_array_equal(codes.cpu().numpy(), g["Q6_K/codes"])
    np.testing.assert_array_equal(scales.cpu().numpy(), g["Q6_K/scales"])
    np.testing.assert_array_equal(d.cpu().numpy().view(np.uint16), g["Q6_K/d"])
    lin = DN.ScaledLinear(codes, scales, d)
    want = Q.dequantize(g["Q6_K/blocks"], "Q6_K", (rows, cols))
    np.testing.assert_array_equal(lin.floats(torch.float32).cpu().numpy().view(np.uint32), want.view(np.uint32))
    np.testing.assert_array_equal(lin.floats(torch.float16).cpu().numpy().view(np.uint16),
                                  want.astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("rows, cols", [(640, 2560), (4096, 4096)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_scaled_linear_window_is_the_oracles_and_keeps_a_tokens_bits(cuda, rows, cols, dtype):
    from strata_mlx_b200 import dense as DN

    rng = np.random.default_rng(rows)
    blocks = Q.random_blocks("Q6_K", rows * cols // 256, rng).reshape(-1)
    lin = DN.ScaledLinear.from_blocks(torch.from_numpy(blocks).to(cuda), rows, cols)
    x = rng.standard_normal((8, cols)).astype(np.float16)
    xd = torch.from_numpy(x).to(cuda).to(dtype)
    got = lin(xd)
    codes, scales, d = D.q6k_parts(blocks, rows, cols)
    want = D.scaled_window(codes, scales, d, x)
    w = D.scaled_floats(codes, scales, d)
    bound = 1e-5 * np.abs(w).max() * np.sqrt(cols) * np.abs(x).max() + (1e-3 if dtype == torch.float16 else 0) * np.abs(want).max()
    assert np.abs(got.double().cpu().numpy() - want).max() <= bound
    for t0 in (0, 3, 7):
        assert torch.equal(lin(xd[t0 : t0 + 1]), got[t0 : t0 + 1])
    # a chunk of a prompt (more than MAX_TOKENS) multiplies the floats
    chunk = torch.cat([xd, xd], dim=0)
    assert torch.allclose(lin(chunk)[:8].double(), torch.from_numpy(want).to(cuda), rtol=0, atol=2e-3 * float(np.abs(want).max()))


def test_block_embedding_rows_are_the_decoders(cuda):
    from strata_mlx_b200 import dense as DN

    rng = np.random.default_rng(3)
    vocab, dims = 50, 2560
    blocks = Q.random_blocks("Q4_K", vocab * dims // 256, rng).reshape(-1)
    emb = DN.BlockEmbedding(torch.from_numpy(blocks).to(cuda), "Q4_K", (vocab, dims), torch.float16)
    ids = torch.tensor([[3, 0, 49, 3]], device=cuda)
    got = emb(ids).cpu().numpy()
    w = Q.dequantize(blocks, "Q4_K", (vocab, dims)).astype(np.float16)
    np.testing.assert_array_equal(got[0].view(np.uint16), w[[3, 0, 49, 3]].view(np.uint16))
