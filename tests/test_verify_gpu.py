"""Benchmark configuration 4, a speculative verify pass: 5 tokens (1 accepted + 4 drafted) through MoE layers
whose three routed stacks cycle through the nine block types (layer l, tensor j of gate/up/down has type
TYPES[(3 l + j) % 9]), top-8 of the experts, the Q8_0 shared expert of ffn 4096, at the benchmark's hidden 4096
and ffn 1536. Layers 0-2 hold every type once. Bars: each layer's output within rel-L2 1e-3 of the oracle, its
expert indices exact; a CUDA graph of the mixed-type layer replays the eager bits. The pairs go through the
decode products (gate and up in one launch, SwiGLU inside down) as in the reference's BLOCK_GLU path
(strata_mlx/blocks.py:958-986)."""

import numpy as np
import pytest

from oracle import moe as M

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
from strata_mlx_b200 import fused as F  # noqa: E402

from test_moe_gpu import build_block, dev, make_layer, rel_l2  # noqa: E402

TYPES = ("Q8_0", "Q4_K", "Q5_K", "Q6_K", "Q2_K", "Q3_K", "IQ3_S", "IQ3_XXS", "IQ4_XS")
H, F_, FS, K, TOKENS = 4096, 1536, 4096, 8, 5
E = 32  # the benchmark has 256; fewer experts keep the oracle's random bytes small, the shapes stay


def kinds_of(layer):
    return tuple(TYPES[(3 * layer + j) % 9] for j in range(3))


@pytest.mark.parametrize("layer", [0, 1, 2])
def test_a_verify_window_through_each_layer_is_the_oracles(cuda, layer):
    rng = np.random.default_rng(40 + layer)
    routed, shared, router, sgate = make_layer(rng, H, F_, E, FS, kinds_of(layer), "Q8_0")
    block = build_block(routed, shared, router, sgate, K)
    x = rng.standard_normal((TOKENS, H)).astype(np.float16)
    got = block(dev(x)).cpu().numpy()
    logits = block.gate(dev(x)).cpu().numpy()
    want, idx, _, _ = M.moe_block(x, router, K, routed, shared, sgate, logits=logits)
    np.testing.assert_array_equal(F.top_k(dev(logits), K).cpu().numpy().astype(np.int64), idx.astype(np.int64))
    assert np.isfinite(got).all()
    assert rel_l2(got, want) <= 1e-3


def test_a_graph_of_the_mixed_layer_replays_the_eager_bits(cuda):
    rng = np.random.default_rng(47)
    routed, shared, router, sgate = make_layer(rng, H, F_, E, FS, kinds_of(1), "Q8_0")
    block = build_block(routed, shared, router, sgate, K)
    xs = [dev(rng.standard_normal((TOKENS, H)).astype(np.float16)) for _ in range(2)]
    eager = [block(x).clone() for x in xs]
    gb = F.GraphedBlock(block, TOKENS, H, torch.float16, cuda)
    for _ in range(2):
        for x, want in zip(xs, eager):
            got = gb(x)
            torch.cuda.synchronize()
            assert torch.equal(got, want)
