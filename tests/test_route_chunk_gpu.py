"""The route of a prompt chunk (more than 32 tokens: route_chunk_kernel) against the same tokens routed eight at
a time (route_kernel): the same logits, choice, weights, shared gate and rank's view, bit for bit, since both
take each token's sums in the same order; the logits within float32 rounding of the float64 product, the
choice the oracle's on those logits.

The route restates `_Routed.__call__`'s start (strata_mlx/fused.py:487-491) and the router product
`_WindowLinear` (strata_mlx/fused.py:357-390).
"""

import numpy as np
import pytest

from oracle import moe as M

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
from strata_mlx_b200 import fused as F  # noqa: E402


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("tokens,experts", [(33, 256), (200, 320), (1180, 256)])
@pytest.mark.parametrize("dtype", [np.float16, np.float32])
@pytest.mark.parametrize("local", [None, (64, 96)])
def test_a_prompt_chunk_routes_as_its_tokens_eight_at_a_time(cuda, tokens, experts, dtype, local):
    rng = np.random.default_rng(tokens + experts)
    H, k = 4096, 8
    router = F.WindowLinear(dev((0.02 * rng.standard_normal((experts, H))).astype(np.float16)))
    sgate = F.WindowLinear(dev((0.02 * rng.standard_normal((1, H))).astype(np.float16)))
    x = dev(rng.standard_normal((tokens, H)).astype(dtype))
    whole = F.route(router, sgate, x, k, local=local)
    logits = router(x)
    parts = [F.route(router, sgate, x[t : t + 8], k, local=local) for t in range(0, tokens, 8)]
    for i, got in enumerate(whole):
        assert torch.equal(got, torch.cat([p[i] for p in parts]))
    assert torch.equal(logits, torch.cat([router(x[t : t + 8]) for t in range(0, tokens, 8)]))
    want = M.router_logits(router.weight.cpu().numpy(), x.cpu().numpy())
    lg = logits.cpu().numpy()
    assert np.abs(lg - want).max() <= 1e-5 * np.abs(want).max()
    np.testing.assert_array_equal(whole[0].cpu().numpy().astype(np.int64), M.top_k(lg, k).astype(np.int64))
    np.testing.assert_allclose(whole[1].cpu().numpy(), M.softmax_chosen(lg, M.top_k(lg, k)), rtol=1e-6, atol=1e-7)


def test_a_prompt_chunk_route_reuses_its_counters(cuda):
    """The counters come back to zero after each launch: routes of several prompt chunks in a row, then decode
    windows on the same counters, each the same as alone."""
    rng = np.random.default_rng(9)
    H, E, k = 1024, 256, 8
    router = F.WindowLinear(dev((0.02 * rng.standard_normal((E, H))).astype(np.float16)))
    sgate = F.WindowLinear(dev((0.02 * rng.standard_normal((1, H))).astype(np.float16)))
    xs = [dev(rng.standard_normal((t, H)).astype(np.float16)) for t in (100, 64, 1, 5, 300)]
    first = [F.route(router, sgate, x, k) for x in xs]
    for _ in range(2):
        for x, want in zip(xs, first):
            got = F.route(router, sgate, x, k)
            assert all(torch.equal(a, b) for a, b in zip(got, want))
