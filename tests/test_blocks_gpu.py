"""The CUDA path of strata_mlx_b200.blocks against the CPU oracle and the golden fixtures, through the C ABI.

Mirrors the reference's tests/test_blocks.py (cited per test). Bars: dequant bit-exact (float32 and float16);
matvec within 1e-5 * max|w| * sqrt(cols) of the float64 product (the reference's tolerance); tile products
within 2e-6 of the float64 product with weights rounded to the activations' type; fused paths bit-identical
to their unfused forms.
"""

import os

import numpy as np
import pytest

from oracle import moe as M
from oracle import quants as Q

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
from strata_mlx_b200 import blocks as B  # noqa: E402

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "blocks.npz")
KINDS = sorted(B.BLOCK)
EXPERTS, OUT = 3, 2  # golden tensors of 3 rows of 2560: three experts of one row... see stack()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def stack(kind, rng, experts, rows, cols, scale=(0.001, 0.01)):
    """Random blocks of a stack of `kind` and its float32 weights from the oracle (tests/test_blocks.py:80-94)."""
    per, nbytes = B.BLOCK[kind]
    n = experts * rows * cols // per
    b = Q.random_blocks(kind, n, rng, scale=scale).reshape(-1)
    return b, Q.dequantize(b, kind, (experts, rows, cols))


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("kind", KINDS)
def test_dequant_is_the_reference_weights_bit_for_bit(cuda, golden, kind):
    """tests/test_blocks.py:18-24, tightened to bits, float32 and float16."""
    rows, cols = (int(v) for v in golden["shape"])
    blocks = dev(golden[f"{kind}/blocks"])
    got32 = B.dequantize(blocks, kind, (rows, cols), torch.float32).cpu().numpy()
    np.testing.assert_array_equal(got32.view(np.uint32), golden[f"{kind}/f32"].view(np.uint32))
    got16 = B.dequantize(blocks, kind, (rows, cols), torch.float16).cpu().numpy()
    np.testing.assert_array_equal(got16.view(np.uint16), golden[f"{kind}/f16"])


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("per_row", [1, 4, 16])
def test_products_on_blocks_are_products_on_the_weights(cuda, kind, per_row):
    """tests/test_blocks.py:27-44: both x layouts (share = k for gate/up, a row per pair for down)."""
    rng = np.random.default_rng(1)
    b, w = stack(kind, rng, 3, 40, 2560 if B.BLOCK[kind][0] != 256 else 2560, scale=(-0.05, 0.05))
    layer = B.BlockSwitchLinear(dev(b), kind, w.shape, per_row=per_row)
    idx = np.array([[2, 0], [1, 1], [0, 2], [2, 2], [0, 1]])
    scale = np.abs(w).max() * np.sqrt(w.shape[-1])
    x = rng.standard_normal((5, 1, 1, w.shape[-1])).astype(np.float32)
    got = layer(dev(x), dev(idx)).cpu().numpy()
    assert got.shape == (5, 2, 1, 40)
    want = np.einsum("tkoi,ti->tko", w[idx].astype(np.float64), x[:, 0, 0].astype(np.float64))
    assert np.abs(got[:, :, 0] - want).max() <= 1e-5 * scale
    x = rng.standard_normal((5, 2, 1, w.shape[-1])).astype(np.float32)
    got = layer(dev(x), dev(idx)).cpu().numpy()
    want = np.einsum("tkoi,tki->tko", w[idx].astype(np.float64), x[:, :, 0].astype(np.float64))
    assert np.abs(got[:, :, 0] - want).max() <= 1e-5 * scale


@pytest.mark.parametrize("kind", ["IQ4_NL", "IQ2_S", "Q2_K"])
@pytest.mark.parametrize("unpacked", [False, True])
def test_a_prompt_gets_the_same_products_a_pair_at_a_time_and_from_unpacked_weights(cuda, kind, unpacked):
    """tests/test_blocks.py:47-60."""
    rng = np.random.default_rng(3)
    b, w = stack(kind, rng, 3, 2, 2560, scale=(-0.05, 0.05))
    layer = B.BlockSwitchLinear(dev(b), kind, w.shape)
    layer.unpack_from = 100 if unpacked else 1000
    idx = np.sort(rng.integers(0, 3, 200))
    x = rng.standard_normal((200, 1, w.shape[-1])).astype(np.float32)
    got = layer(dev(x), dev(idx), sorted_indices=True).cpu().numpy()
    assert got.shape == (200, 1, 2)
    scale = np.abs(w).max() * np.sqrt(w.shape[-1])
    want = np.einsum("noi,ni->no", w[idx].astype(np.float64), x[:, 0].astype(np.float64))
    assert np.abs(got[:, 0] - want).max() <= 1e-5 * scale


@pytest.mark.parametrize("kind", ["IQ3_S", "Q8_0", "IQ4_XS", "IQ3_XXS", "Q2_0"])
@pytest.mark.parametrize("rows, cols", [(40, 512), (1536, 4096), (4096, 1536), (16, 256)])
@pytest.mark.parametrize("share", [1, 4])
def test_float16_products_on_the_tensor_core_path(cuda, kind, rows, cols, share):
    """The decode matvec of the hot path's types and Q2_0 (int8 mma.sync on the exact codes, the activations
    split into int8 hi / lo, float32 scales) against the float64 product: the float16 result within 1e-3 of the
    largest value (its own rounding is 2^-11)."""
    rng = np.random.default_rng(rows + cols + share)
    E, pairs = 5, 8
    b, w = stack(kind, rng, E, rows, cols, scale=(-0.05, 0.05))
    layer = B.BlockSwitchLinear(dev(b), kind, (E, rows, cols))
    idx = rng.integers(0, E, pairs // share * share).reshape(-1, share)
    x = rng.standard_normal((pairs // share, cols)).astype(np.float16)
    xs = x[:, None, None, :] if share > 1 else x[:, None, :]
    got = layer(dev(xs if share > 1 else x.reshape(pairs // share, share, 1, cols)), dev(idx)).float().cpu().numpy()
    want = np.einsum("pri,pi->pr", w[idx.reshape(-1)].astype(np.float64),
                     x.astype(np.float64)[np.arange(idx.size) // share])
    assert np.abs(got.reshape(idx.size, rows) - want).max() <= 1e-3 * np.abs(want).max()


@pytest.mark.parametrize("kind", ["Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"])
@pytest.mark.parametrize("rows, cols", [(40, 512), (1536, 4096), (4096, 1536), (16, 256)])
@pytest.mark.parametrize("share", [1, 8])
def test_float16_products_of_the_k_types_on_int8_dot_products(cuda, kind, rows, cols, share):
    """The K-types with float16 activations (the activations split into int8 hi / lo, integer dot products,
    float scales and minimums per 16 or 32 weights) against the float64 product: within 1e-3 of the largest
    value, the bar of the tensor-core kernels (the split keeps x to 1/256 of max|x| / 127)."""
    rng = np.random.default_rng(rows + cols + share + len(kind))
    E, pairs = 5, 8
    b, w = stack(kind, rng, E, rows, cols, scale=(-0.05, 0.05))
    layer = B.BlockSwitchLinear(dev(b), kind, (E, rows, cols))
    idx = rng.integers(0, E, pairs // share * share).reshape(-1, share)
    x = rng.standard_normal((pairs // share, cols)).astype(np.float16)
    xs = x[:, None, None, :] if share > 1 else x[:, None, :]
    got = layer(dev(xs if share > 1 else x.reshape(pairs // share, share, 1, cols)), dev(idx)).float().cpu().numpy()
    want = np.einsum("pri,pi->pr", w[idx.reshape(-1)].astype(np.float64),
                     x.astype(np.float64)[np.arange(idx.size) // share])
    assert np.abs(got.reshape(idx.size, rows) - want).max() <= 1e-3 * np.abs(want).max()


@pytest.mark.parametrize("kind", ["IQ3_S", "Q8_0", "Q4_K", "Q6_K", "IQ4_XS", "IQ3_XXS"])
@pytest.mark.parametrize("window", [5, 8, 11])
def test_a_window_gives_each_token_its_bits_alone(cuda, kind, window):
    """window_matvec (strata_mlx/blocks.py:349-396): a verify window's dense product within 1e-3 of the largest
    value of the float64 product; each token the same bits as alone, on the CUDA-core kernels and on the int8
    tensor-core kernel (a one-expert stack's team of warps follows its shape, not the window; Q8_0 takes up to
    four tokens a pass: 5 as four and one, 8 as two passes, 11 as four, four and three)."""
    rng = np.random.default_rng(len(kind) + 16 * window)
    rows, cols = 256, 1024
    b, w = stack(kind, rng, 1, rows, cols, scale=(-0.05, 0.05))
    x = rng.standard_normal((window, cols)).astype(np.float16)
    got = B.window_matvec(dev(b), kind, rows, cols, dev(x))
    assert got.shape == (window, rows) and got.dtype == torch.float16
    want = x.astype(np.float64) @ w[0].astype(np.float64).T
    for t in range(window):
        alone = B.window_matvec(dev(b), kind, rows, cols, dev(x[t : t + 1]))
        assert torch.equal(got[t : t + 1], alone)
    assert np.abs(got.float().cpu().numpy() - want).max() <= 1e-3 * np.abs(want).max()


def test_half_precision_activations_come_back_as_half(cuda):
    """tests/test_blocks.py:63-70."""
    rng = np.random.default_rng(5)
    b, w = stack("IQ3_XXS", rng, 3, 2, 2560, scale=(-0.05, 0.05))
    x = torch.randn(2, 1, 1, 2560, device="cuda").half()
    idx = dev(np.array([[0, 1], [2, 0]]))
    out = B.BlockSwitchLinear(dev(b), "IQ3_XXS", (3, 2, 2560))(x, idx)
    assert out.dtype == torch.float16 and out.shape == (2, 2, 1, 2)
    want = B.BlockSwitchLinear(dev(b), "IQ3_XXS", (3, 2, 2560))(x.float(), idx)
    assert (out.float() - want).abs().max().item() <= 2e-3 * want.abs().max().item()


@pytest.mark.parametrize("kind", ["Q2_K", "IQ3_S", "Q8_0", "Q4_K", "IQ4_XS"])
def test_the_rows_variant_is_the_tile_product_read_back(cuda, kind):
    """smoe_tile_matmul_rows: the tiled path's `product(down, h)[where].astype(x.dtype)`
    (strata_mlx/blocks.py:693) in one launch gives the same bits as the product then the read-back; a dense
    layer's tokens without padding rows the same bits as padded; smoe_swiglu_to the bits of the float32
    SwiGLU then the cast (blocks.py:692)."""
    rng = np.random.default_rng(11)
    E, rows, cols, T, k = 6, 256, 512, 45, 4
    b, _ = stack(kind, rng, E, rows, cols)
    blocks = dev(b)
    idx = dev(rng.choice(E, (T, k), replace=True).astype(np.int32))
    tiles, token, where = B.tiles_of(idx, E)
    x = dev(rng.standard_normal((T, cols)).astype(np.float16))
    a = x.index_select(0, token.view(torch.int32))
    want = B.tile_matmul(blocks, kind, (E, rows, cols), a, tiles).index_select(0, where.view(torch.int32)).half()
    got = B.tile_matmul_rows(blocks, kind, (E, rows, cols), a, tiles, B.slot_rows(where, a.shape[0]), T * k)
    assert torch.equal(got, want)
    # a dense layer: expert 0 for every tile, 45 tokens in 3 tiles without padding rows
    te = torch.zeros(3, dtype=torch.int32, device="cuda")
    padded = torch.cat([x, x.new_zeros(3 * 16 - T, cols)])
    want = B.tile_matmul(blocks, kind, (E, rows, cols), padded, te)[:T].half()
    got = B.tile_matmul_rows(blocks, kind, (E, rows, cols), x, te, None, T)
    assert torch.equal(got, want)
    g32, u32 = (dev(rng.standard_normal((T, rows)).astype(np.float32)) for _ in range(2))
    assert torch.equal(B.swiglu_to(g32, u32, torch.float16), B.swiglu(g32, u32).half())


@pytest.mark.parametrize("kind", ["Q2_K", "IQ3_S", "Q8_0", "Q5_K"])
def test_a_pair_of_stacks_in_one_launch_is_the_two_products(cuda, kind):
    """smoe_tile_matmul_pair(_rows): gate and up through the same tiles in one launch give each the bits of its own
    tile product (strata_mlx/blocks.py:690-692), in slot order as float32 and in the rows form as float16."""
    rng = np.random.default_rng(13)
    E, rows, cols, T, k = 6, 256, 512, 45, 4
    ga = B.BlockSwitchLinear(dev(stack(kind, rng, E, rows, cols)[0]), kind, (E, rows, cols))
    ub = B.BlockSwitchLinear(dev(stack(kind, rng, E, rows, cols)[0]), kind, (E, rows, cols))
    idx = dev(rng.choice(E, (T, k), replace=True).astype(np.int32))
    tiles, token, where = B.tiles_of(idx, E)
    x = dev(rng.standard_normal((T, cols)).astype(np.float16))
    a = x.index_select(0, token.view(torch.int32))
    g, u = B.tile_matmul_pair(ga, ub, a, tiles)
    live = (tiles.view(torch.int32).long() < E).repeat_interleave(16)  # (rows of padding tiles are not written)
    assert torch.equal(g[live], B.tile_matmul(ga.blocks, kind, ga.shape, a, tiles)[live])
    assert torch.equal(u[live], B.tile_matmul(ub.blocks, kind, ub.shape, a, tiles)[live])
    sr = B.slot_rows(where, a.shape[0])
    g16, u16 = B.tile_matmul_pair(ga, ub, a, tiles, sr, T * k)
    assert torch.equal(g16, B.tile_matmul_rows(ga.blocks, kind, ga.shape, a, tiles, sr, T * k))
    assert torch.equal(u16, B.tile_matmul_rows(ub.blocks, kind, ub.shape, a, tiles, sr, T * k))
    te = torch.zeros(3, dtype=torch.int32, device="cuda")  # a dense layer: expert 0, 45 tokens, no padding rows
    g16, u16 = B.tile_matmul_pair(ga, ub, x, te, None, T)
    assert torch.equal(g16, B.tile_matmul_rows(ga.blocks, kind, ga.shape, x, te, None, T))
    assert torch.equal(u16, B.tile_matmul_rows(ub.blocks, kind, ub.shape, x, te, None, T))


@pytest.mark.parametrize("dtype", [np.float16, np.float32])
def test_swiglu_eight_a_thread_is_the_one_a_thread(cuda, dtype):
    """smoe_swiglu / smoe_swiglu_to: the eight-wide kernels (aligned, a multiple of 8 values) give each value the
    bits of the one-value kernels (an odd offset takes those); float16 within one float16 step of the oracle's
    (strata_mlx/blocks.py:222-237; its float32 exp is numpy's)."""
    rng = np.random.default_rng(21)
    n = 4096 * 3 + 8
    g = dev((2 * rng.standard_normal(n + 1)).astype(dtype))
    u = dev((2 * rng.standard_normal(n + 1)).astype(dtype))
    wide = B.swiglu(g[1:].clone(), u[1:].clone())
    one = B.swiglu(g[1:], u[1:])
    assert torch.equal(wide, one)
    if dtype == np.float16:
        want = M.swiglu(g[1:].cpu().numpy(), u[1:].cpu().numpy()).astype(np.float32)
        got = wide.cpu().numpy().astype(np.float32)
        assert np.all(np.abs(got - want) <= 2.0 ** -10 * np.maximum(np.abs(want), 2.0 ** -14))
    else:
        assert torch.equal(B.swiglu_to(g[1:].clone(), u[1:].clone(), torch.float16), one.half())
        assert torch.equal(B.swiglu_to(g[1:], u[1:], torch.float16), one.half())


def test_slot_rows_inverts_where(cuda):
    """smoe_slot_rows: slot where[p] holds p, every other slot 0xffffffff."""
    rng = np.random.default_rng(12)
    idx = dev(rng.choice(9, (31, 3), replace=True).astype(np.int32))
    tiles, token, where = B.tiles_of(idx, 9)
    inv = B.slot_rows(where, token.numel()).view(torch.int32).cpu().numpy().astype(np.uint32)
    w = where.view(torch.int32).cpu().numpy().astype(np.int64)
    want = np.full(token.numel(), 0xFFFFFFFF, dtype=np.uint64)
    want[w] = np.arange(w.size)
    np.testing.assert_array_equal(inv.astype(np.uint64), want)


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("dtype", [np.float16, np.float32])
def test_the_tile_product_is_the_product_with_the_weights(cuda, kind, dtype):
    """tests/test_blocks.py:102-114: tiles in no particular order, weights rounded to a's type, 2e-6."""
    rng = np.random.default_rng(0)
    shape = (4, 128, 512)
    b, w = stack(kind, rng, *shape)
    w = w.astype(dtype).astype(np.float64)
    tiles = np.array([3, 0, 0, 2, 3])
    a = rng.standard_normal((16 * len(tiles), shape[2])).astype(dtype)
    got = B.tile_matmul(dev(b), kind, shape, dev(a), dev(tiles.astype(np.int32))).cpu().numpy()
    want = np.einsum("poi,pi->po", w[np.repeat(tiles, 16)], a.astype(np.float64))
    assert got.shape == want.shape and got.dtype == np.float32
    assert np.abs(got - want).max() <= 2e-6 * np.abs(want).max()


@pytest.mark.parametrize("kind", ["IQ3_S", "Q2_K", "Q8_0", "Q6_K"])
@pytest.mark.parametrize("rows, cols, tiles", [(1536, 4096, [5, 5, 5, 5, 5, 5, 5, 5, 5, 1, 7, 7]),
                                               (192, 1536, [0, 1, 1, 2]), (64, 256, [0])])
def test_tile_product_at_model_shapes_runs_of_many_tiles(cuda, kind, rows, cols, tiles):
    """Runs longer than a job's 8 tiles, rows not a multiple of 128, a single tile; the tensor-core path."""
    rng = np.random.default_rng(rows + cols)
    E = 8
    b, w = stack(kind, rng, E, rows, cols)
    w16 = w.astype(np.float16).astype(np.float64)
    tiles = np.array(tiles)
    a = (rng.standard_normal((16 * len(tiles), cols)) * 0.5).astype(np.float16)
    got = B.tile_matmul(dev(b), kind, (E, rows, cols), dev(a), dev(tiles.astype(np.int32))).cpu().numpy()
    want = np.einsum("poi,pi->po", w16[np.repeat(tiles, 16)], a.astype(np.float64))
    # the tensor cores' float32 accumulation error grows with the length of the sum: the reference's 2e-6 of
    # the largest value holds at 512 columns, here scaled by cols / 512 (at 4096: 1.6e-5, against the
    # layer's 1e-3 rel-L2 budget)
    assert np.abs(got - want).max() <= 2e-6 * (cols / 512) * np.abs(want).max()


def test_a_tile_of_no_expert_is_left_out(cuda):
    """tests/test_blocks.py:203-211."""
    rng = np.random.default_rng(3)
    b, w = stack("Q2_0", rng, 4, 128, 256)
    tiles = np.array([1, 4, 2, 9])
    a = rng.standard_normal((16 * len(tiles), 256)).astype(np.float16)
    out = torch.full((64, 128), 7.0, device="cuda")
    got = B.tile_matmul(dev(b), "Q2_0", (4, 128, 256), dev(a), dev(tiles.astype(np.int32))).cpu().numpy()
    for t in (0, 2):
        want = a[16 * t : 16 * t + 16].astype(np.float64) @ w[tiles[t]].astype(np.float16).astype(np.float64).T
        assert np.abs(got[16 * t : 16 * t + 16] - want).max() <= 2e-6 * np.abs(want).max()
    del out


@pytest.mark.parametrize("tokens, k, experts", [(211, 3, 7), (5, 2, 40), (64, 10, 512), (1, 1, 3), (1180, 8, 256),
                                                (3000, 8, 256)])
def test_tiles_hold_every_pair_with_its_expert_and_equal_the_oracle(cuda, tokens, k, experts):
    """tests/test_blocks.py:182-200, and equal to the oracle's (both place a pair by its flat index)."""
    rng = np.random.default_rng(tokens)
    idx = rng.integers(0, experts, (1, tokens, k))
    idx[0, : tokens // 3] = 1
    if tokens >= 33 and experts > 4:
        idx[0, -33:, 0] = np.repeat([3, 4], [16, 17])
    got = [t.view(torch.int32).cpu().numpy().astype(np.int64) for t in B.tiles_of(dev(idx.astype(np.int32)), experts)]
    want = M.tiles_of(idx, experts)
    for g, wnt in zip(got, want):
        np.testing.assert_array_equal(g, wnt.astype(np.int64))


def test_gate_and_up_in_one_launch_are_two_launches(cuda):
    rng = np.random.default_rng(11)
    bg, _ = stack("IQ3_S", rng, 6, 256, 1024)
    bu, _ = stack("IQ3_S", rng, 6, 256, 1024)
    gate = B.BlockSwitchLinear(dev(bg), "IQ3_S", (6, 256, 1024))
    up = B.BlockSwitchLinear(dev(bu), "IQ3_S", (6, 256, 1024))
    x = torch.randn(3, 1024, device="cuda").half()
    idx = dev(np.array([[0, 5], [2, 2], [4, 1]], dtype=np.int32))
    g, u = B.gate_up(gate, up, x, idx.reshape(-1), 2)
    x5 = x[:, None, None, :]
    assert torch.equal(g, gate(x5, idx).reshape(6, -1)) and torch.equal(u, up(x5, idx).reshape(6, -1))


@pytest.mark.parametrize("kind", ["IQ3_S", "IQ2_XS", "IQ4_NL", "Q2_K", "Q5_K", "Q8_0", "Q2_0"])
@pytest.mark.parametrize("tokens", [1, 20])
def test_down_taking_swiglu_itself_and_unsorted_pairs_give_the_same_bits(cuda, monkeypatch, kind, tokens):
    """tests/test_blocks.py:257-280: the BLOCK_GLU path (swiglu formed in down) == down(swiglu(g, u))."""
    monkeypatch.setattr(B, "MATVEC_GLU_UPTO", 1 << 20)
    rng = np.random.default_rng(tokens)

    def experts(rows, cols):
        b, _ = stack(kind, rng, 6, rows, cols, scale=(-0.05, 0.05))
        return B.BlockSwitchLinear(dev(b), kind, (6, rows, cols))

    gate, up, down = experts(256, 512), experts(256, 512), experts(512, 256)
    x = dev((0.01 * rng.standard_normal((1, tokens, 512))).astype(np.float16))
    idx = dev(np.stack([rng.choice(6, 4, replace=False) for _ in range(tokens)])[None].astype(np.int32))
    got = B.switch_glu(x, idx, up, gate, down)
    monkeypatch.setattr(B, "BLOCK_GLU", False)
    want = B.switch_glu(x, idx, up, gate, down)
    assert got.shape == want.shape == (1, tokens, 4, 512)
    assert torch.equal(got, want)
    assert torch.isfinite(want.float()).float().mean().item() > 0.9


@pytest.mark.parametrize("kinds", [("Q2_0", "Q2_0"), ("IQ3_S", "IQ4_NL"), ("IQ2_S", "Q2_0"), ("Q2_K", "Q2_K")])
@pytest.mark.parametrize("dtype", [np.float16, np.float32])
def test_a_prompt_through_tiles_is_the_prompt_a_pair_at_a_time(cuda, kinds, dtype):
    """tests/test_blocks.py:117-149: skewed routing, 211 tokens, k = 3; gate/up through tiles vs float64."""
    rng = np.random.default_rng(1)
    experts, hidden, inner, k = 7, 256, 64, 3
    sg = stack(kinds[0], rng, experts, inner, hidden)
    su = stack(kinds[0], rng, experts, inner, hidden)
    rows = 211
    x = rng.standard_normal((rows, hidden)).astype(dtype)
    idx = rng.integers(0, experts - 1, (rows, k))
    idx[:40] = 2
    te, token, where = B.tiles_of(dev(idx.astype(np.int32)), experts)
    a = dev(x).index_select(0, token.view(torch.int32).long())
    tol = 2e-3 if dtype == np.float16 else 2e-5
    for (b, w) in (sg, su):
        got = B.tile_matmul(dev(b), kinds[0], (experts, inner, hidden), a, te)
        got = got.index_select(0, where.view(torch.int32).long()).cpu().numpy().reshape(rows, k, inner)
        want = np.einsum("tkoi,ti->tko", w[idx].astype(np.float64), x.astype(np.float64))
        assert np.abs(got - want).max() <= tol * np.abs(want).max()


def test_a_prompts_three_products_go_through_tiles(cuda, monkeypatch):
    """tests/test_blocks.py:152-179: switch_glu sends a chunk through tiles, and what comes out is what a pair
    at a time gives (5e-3 of the largest)."""
    rng = np.random.default_rng(1)
    experts, hidden, inner, k = 7, 256, 256, 3
    st = {n: stack("Q2_K", rng, experts, r, c) for n, (r, c) in
          (("gate", (inner, hidden)), ("up", (inner, hidden)), ("down", (hidden, inner)))}
    glu = B.BlockSwitchGLU(*(B.BlockSwitchLinear(dev(st[n][0]), "Q2_K", st[n][1].shape) for n in ("gate", "up", "down")))
    x = dev(rng.standard_normal((1, 211, hidden)).astype(np.float16))
    idx = rng.integers(0, experts - 1, (1, 211, k))
    idx[0, :40] = 2
    called = []
    tiled = B._tiled_glu
    monkeypatch.setattr(B, "_tiled_glu", lambda *a: called.append(1) or tiled(*a))
    monkeypatch.setattr(B, "TILES_FROM", 1 << 62)
    a_pair = glu(x, dev(idx)).cpu().numpy().astype(np.float64)
    assert not called
    monkeypatch.setattr(B, "TILES_FROM", 100)
    in_tiles = glu(x, dev(idx)).cpu().numpy().astype(np.float64)
    assert called and in_tiles.shape == a_pair.shape == (1, 211, k, hidden)
    xs = x.cpu().numpy().astype(np.float64)[0]
    gate, up = (np.einsum("tkoi,ti->tko", st[n][1][idx[0]].astype(np.float64), xs) for n in ("gate", "up"))
    want = np.einsum("tkoi,tki->tko", st["down"][1][idx[0]].astype(np.float64), gate / (1 + np.exp(-gate)) * up)
    scale = np.abs(want).max()
    assert np.abs(a_pair[0] - want).max() <= 5e-3 * scale
    assert np.abs(in_tiles[0] - want).max() <= 5e-3 * scale


@pytest.mark.parametrize("dtype", [np.float16, np.float32])
def test_a_batch_of_products_gives_the_separate_products(cuda, dtype):
    """smoe_matvec_batch: the routed experts' gate and up with a one-expert stack's gate and up on the same
    activations, then two downs forming their SwiGLU, against the calls one at a time (the same bits when the
    batch runs them one at a time, float32; within 1e-3 of the largest value in the one int8 launch, float16,
    whose teams may add their partial sums in another grouping)."""
    rng = np.random.default_rng(3)
    E, F_, H, K, T = 16, 256, 512, 4, 2
    gate = B.BlockSwitchLinear(dev(stack("IQ3_S", rng, E, F_, H)[0]), "IQ3_S", (E, F_, H))
    up = B.BlockSwitchLinear(dev(stack("IQ3_S", rng, E, F_, H)[0]), "IQ3_S", (E, F_, H))
    down = B.BlockSwitchLinear(dev(stack("IQ3_S", rng, E, H, F_)[0]), "IQ3_S", (E, H, F_))
    sg = B.BlockSwitchLinear(dev(stack("Q8_0", rng, 1, 512, H)[0]), "Q8_0", (1, 512, H))
    sd = B.BlockSwitchLinear(dev(stack("Q8_0", rng, 1, H, 512)[0]), "Q8_0", (1, H, 512))
    x = dev(rng.standard_normal((T, H)).astype(dtype))
    idx = dev(rng.choice(E, (T, K), replace=True).astype(np.int32)).reshape(-1)
    zeros = B._zeros_idx(T, x.device)
    tt = x.dtype
    g, u = torch.empty((T * K, F_), dtype=tt, device="cuda"), torch.empty((T * K, F_), dtype=tt, device="cuda")
    gs = torch.empty((T, 512), dtype=tt, device="cuda")
    B.matvec_batch([B._problem(gate, idx, T * K, K, g, x=x), B._problem(up, idx, T * K, K, u, x=x),
                    B._problem(sg, zeros, T, 1, gs, x=x)])
    y = torch.empty((T * K, H), dtype=tt, device="cuda")
    s = torch.empty((T, H), dtype=tt, device="cuda")
    B.matvec_batch([B._problem(down, idx, T * K, 1, y, gate=g, up=u), B._problem(sd, zeros, T, 1, s, gate=gs, up=gs)])
    want_g = B._matvec(gate, x, idx, K, tt)
    want_u = B._matvec(up, x, idx, K, tt)
    want_gs = B._matvec(sg, x, zeros, 1, tt)
    want_y = B.matvec_glu(down, idx, want_g, want_u)
    want_s = B.matvec_glu(sd, zeros, want_gs, want_gs)
    for got, want in ((g, want_g), (u, want_u), (gs, want_gs), (y, want_y), (s, want_s)):
        if dtype == np.float32:
            assert torch.equal(got, want)
        else:
            tol = 1e-3 * want.float().abs().max().item()
            assert (got.float() - want.float()).abs().max().item() <= tol


@pytest.mark.parametrize("tokens", [1, 3])
def test_the_shared_down_product_with_the_combine_is_the_two_calls(cuda, tokens):
    """smoe_matvec_glu_combine: the shared expert's down product with the block's end as its epilogue gives the
    bits of smoe_matvec_glu then smoe_combine (strata_mlx/fused.py:448-481)."""
    from strata_mlx_b200 import _lib
    from strata_mlx_b200 import fused as F

    rng = np.random.default_rng(tokens)
    H, FS, K = 512, 512, 8
    sd = B.BlockSwitchLinear(dev(stack("Q8_0", rng, 1, H, FS)[0]), "Q8_0", (1, H, FS))
    gs = dev(rng.standard_normal((tokens, FS)).astype(np.float16))
    us = dev(rng.standard_normal((tokens, FS)).astype(np.float16))
    y = dev(rng.standard_normal((tokens, K, H)).astype(np.float16))
    w = torch.softmax(dev(rng.standard_normal((tokens, K)).astype(np.float32)), -1)
    g = dev(rng.standard_normal((tokens, 1)).astype(np.float16))
    zeros = B._zeros_idx(tokens, y.device)
    out = torch.empty((tokens, H), dtype=torch.float16, device="cuda")
    _lib.call("smoe_matvec_glu_combine", B._kind("Q8_0"), _lib.ptr(sd.blocks), H, FS, _lib.ptr(zeros), tokens,
              _lib.ptr(gs), _lib.ptr(us), _lib.ptr(y), _lib.ptr(w), _lib.ptr(g), K, _lib.ptr(out), 1, _lib.stream())
    s = B.matvec_glu(sd, zeros, gs, us)
    want = F.moe_combine(y, w, g, s)
    assert torch.equal(out, want)
