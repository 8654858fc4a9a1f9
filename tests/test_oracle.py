"""The CPU oracle against the golden fixtures (gguf-py 0.19.0 and the reference's own decoders) and against the
reference tests' semantics. No GPU."""

import os

import numpy as np
import pytest

from oracle import moe as M
from oracle import quants as Q

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "blocks.npz")
KINDS = sorted(Q.TYPES)


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("kind", KINDS)
def test_oracle_decoders_are_the_reference_weights_bit_for_bit(golden, kind):
    rows, cols = golden["shape"]
    got = Q.dequantize(golden[f"{kind}/blocks"], kind, (rows, cols))
    want = golden[f"{kind}/f32"]
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    with np.errstate(over="ignore"):
        np.testing.assert_array_equal(got.astype(np.float16).view(np.uint16), golden[f"{kind}/f16"])


@pytest.mark.parametrize("kind", KINDS)
def test_oracle_decoders_match_gguf_py_on_fresh_blocks(kind):
    gguf = pytest.importorskip("gguf")
    rng = np.random.default_rng(hash(kind) % 1000)
    _, per, nbytes = Q.TYPES[kind]
    b = Q.random_blocks(kind, 64, rng)
    got = Q.DECODERS[kind](b)
    if kind == "Q2_0":
        pytest.skip("gguf-py has no Q2_0; pinned by the reference's restatement in the golden fixture")
    want = gguf.quants.dequantize(b.reshape(-1), getattr(gguf.GGMLQuantizationType, kind)).reshape(got.shape)
    np.testing.assert_array_equal(got.view(np.uint32), want.astype(np.float32).view(np.uint32))


def test_fixture_covers_the_edge_scales(golden):
    # zero scale, negative scale and a scale whose weights overflow float16 are in every fixture
    w = golden["Q8_0/f16"].view(np.float16)
    assert np.isinf(w).any() and (w == 0).any()


@pytest.mark.parametrize("tokens, k, experts", [(211, 3, 7), (5, 2, 40), (64, 10, 512), (1, 1, 3)])
def test_oracle_tiles_hold_every_pair_with_its_expert(tokens, k, experts):
    """The invariants of the reference's tests/test_blocks.py:182-200, on the oracle's tiles_of."""
    rng = np.random.default_rng(tokens)
    idx = rng.integers(0, experts, (1, tokens, k))
    idx[0, : tokens // 3] = 1
    if tokens >= 33 and experts > 4:
        idx[0, -33:, 0] = np.repeat([3, 4], [16, 17])
    tile_expert, token, where = M.tiles_of(idx, experts)
    flat = idx.reshape(-1)
    assert len(tile_expert) * 16 == len(token) and len(where) == len(flat)
    assert len(set(where.tolist())) == len(flat)
    np.testing.assert_array_equal(tile_expert[where // 16], flat)
    np.testing.assert_array_equal(token[where], np.arange(len(flat)) // k)
    used = np.zeros(len(tile_expert), dtype=bool)
    used[where // 16] = True
    assert (tile_expert[~used] == experts).all() and (tile_expert[used] < experts).all()
    assert used.sum() == sum(-(-c // 16) for c in np.bincount(flat))


@pytest.mark.parametrize("ties", [False, True])
def test_oracle_top_k_is_stable_argpartition(ties):
    """tests/test_fused.py:109-120: top_k == argpartition(-logits, k-1)[..., :k] with ties to the lower index."""
    rng = np.random.default_rng(7)
    logits = rng.standard_normal((40, 512)).astype(np.float32)
    if ties:
        logits = np.round(logits * 4) / 4
    idx = M.top_k(logits, 10)
    for r in range(40):
        order = sorted(range(512), key=lambda j: (-logits[r, j], j))[:10]
        assert idx[r].tolist() == order


def test_oracle_combine_order_is_mlx_col_reduce_small():
    # k = 10: partial sums j = 0..7 over k = j, j + 8, then the partials in order
    rng = np.random.default_rng(3)
    y = (rng.standard_normal((2, 10, 256)) * 0.5).astype(np.float16)
    w = rng.random((2, 10)).astype(np.float32)
    g = rng.standard_normal(2).astype(np.float16)
    s = rng.standard_normal((2, 256)).astype(np.float16)
    out = M.combine(y, w, g, s)
    y32 = y.astype(np.float32)
    acc = None
    for j in range(8):
        part = np.float32(0)
        for kk in range(j, 10, 8):
            part = np.float32(y32[0, kk, 5] * w[0, kk]) + part
        acc = part if acc is None else np.float32(part + acc)
    gate = np.float16(1 / (1 + np.exp(-np.float32(g[0]))))
    want = np.float16(np.float32(np.float16(acc)) + np.float32(np.float16(np.float32(gate) * np.float32(s[0, 5]))))
    assert out[0, 5] == want


def test_oracle_swiglu_rounds_in_the_activation_type():
    g = np.array([-3.0, -0.5, 0.0, 0.7, 12.0], dtype=np.float16)
    u = np.array([1.0, 2.0, 3.0, -1.5, 0.25], dtype=np.float16)
    got = M.swiglu(g, u)
    assert got.dtype == np.float16
    want = g.astype(np.float64) / (1 + np.exp(-g.astype(np.float64))) * u
    assert np.abs(got - want).max() <= 2e-3 * np.abs(want).max()


# ---------------------------------------------------------------- the dense steps (oracle/dense.py)

DENSE = os.path.join(os.path.dirname(__file__), "golden", "dense.npz")


def test_oracle_q6k_parts_are_the_references():
    """Against the reference's own q6k_parts (strata_mlx/gguf.py:150-165), run to make tests/golden/dense.npz."""
    from oracle import dense as D

    g = np.load(DENSE)
    rows, cols = g["shape"]
    codes, scales, d = D.q6k_parts(g["Q6_K/blocks"], rows, cols)
    np.testing.assert_array_equal(codes, g["Q6_K/codes"])
    np.testing.assert_array_equal(scales, g["Q6_K/scales"])
    np.testing.assert_array_equal(d.view(np.uint16), g["Q6_K/d"])
    # and their weights are the block decoder's, bit for bit
    w = D.scaled_floats(codes, scales, d)
    np.testing.assert_array_equal(w.view(np.uint32), Q.dequantize(g["Q6_K/blocks"], "Q6_K", (rows, cols)).view(np.uint32))


def test_oracle_q3k_planes_are_the_references():
    """Against the reference's own q3k_planes (strata_mlx/blocks.py:403-414), run to make tests/golden/dense.npz."""
    from oracle import dense as D

    g = np.load(DENSE)
    rows, cols = g["shape"]
    p = D.q3k_planes(g["Q3_K/blocks"], rows, cols)
    for name in ("hm", "qs", "sc"):
        np.testing.assert_array_equal(p[name], g[f"Q3_K/{name}"])
    np.testing.assert_array_equal(p["dd"].view(np.uint16), g["Q3_K/dd"])
    w = D.q3k_planes_weights(p, rows, cols)
    np.testing.assert_array_equal(w.view(np.uint32), Q.dequantize(g["Q3_K/blocks"], "Q3_K", (rows, cols)).view(np.uint32))


def test_oracle_hyper_connection_reads_before_plainly_when_nothing_was_written():
    """strata_mlx's tests/test_fused.py:40-48 in the oracle: out = 0 and inject_in = 0 leave the residual `before`,
    and the read is the hyper-connection of `before` alone."""
    from oracle import dense as D

    rng = np.random.default_rng(6)
    hc, d, rank, T = 4, 96, 24, 2
    before = rng.standard_normal((T, hc * d)).astype(np.float32)
    norm = (1 + 0.2 * rng.standard_normal(hc * d)).astype(np.float32)
    down = (0.1 * rng.standard_normal((rank, hc * d))).astype(np.float32)
    up = (0.1 * rng.standard_normal((hc * d, rank))).astype(np.float32)
    inj = (0.1 * rng.standard_normal((hc, hc * d))).astype(np.float32)
    mixed, residual, inject = D.hyper_connection(before, np.zeros((T, d)), np.zeros((T, hc)), norm, down, up, inj, hc,
                                                 dtype=np.float32)
    np.testing.assert_array_equal(residual, before)
    assert mixed.shape == (T, d) and inject.shape == (T, hc) and np.all((inject > 0) & (inject < 2))
