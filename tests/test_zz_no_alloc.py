"""smoe_tiles_of_noalloc against smoe_tiles_of, through the C ABI.

smoe_tiles_of_noalloc is for callers that cannot allocate device memory where they call the library (a host
framework that owns every device allocation and gives a plugin only its inputs and outputs, or a loop that
must not call cudaMalloc because it can synchronize the device): it keeps its scratch in a fixed array in the
library's device image instead of a caller's workspace. Its results must be those of smoe_tiles_of exactly
(integer work), on two calls in a row, the second smaller than the first so that anything the first left in
the shared array would show. This file is collected last so that a failure here comes after every other test.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
from strata_mlx_b200 import _lib  # noqa: E402


def with_workspace(idx, k, experts):
    pairs = idx.numel()
    most = pairs // 16 + min(experts, pairs)
    outs = [torch.empty(most, dtype=torch.int32, device="cuda"), torch.empty(most * 16, dtype=torch.int32, device="cuda"),
            torch.empty(pairs, dtype=torch.int32, device="cuda")]
    ws = torch.empty(int(_lib.lib().smoe_tiles_of_workspace_size(pairs, experts)), dtype=torch.uint8, device="cuda")
    _lib.call("smoe_tiles_of", _lib.ptr(idx), pairs, k, experts, *(_lib.ptr(o) for o in outs), _lib.ptr(ws), ws.numel(),
              _lib.stream())
    return outs


def without_allocation(idx, k, experts):
    pairs = idx.numel()
    most = pairs // 16 + min(experts, pairs)
    # outputs start as garbage: the entry point must write every element itself
    outs = [torch.full((most,), -7, dtype=torch.int32, device="cuda"),
            torch.full((most * 16,), -7, dtype=torch.int32, device="cuda"),
            torch.full((pairs,), -7, dtype=torch.int32, device="cuda")]
    _lib.call("smoe_tiles_of_noalloc", _lib.ptr(idx), pairs, k, experts, *(_lib.ptr(o) for o in outs), _lib.stream())
    return outs


def routing(rng, tokens, k, experts):
    """Zipf-skewed expert choices (s = 1.1), distinct within a token, like a prompt chunk's router."""
    p = 1.0 / np.arange(1, experts + 1) ** 1.1
    p /= p.sum()
    perm = rng.permutation(experts)
    idx = np.stack([perm[rng.choice(experts, k, replace=False, p=p)] for _ in range(tokens)])
    return torch.from_numpy(idx.astype(np.int32)).cuda()


def test_no_alloc_tiles_equal_the_workspace_tiles_on_two_calls_in_a_row(cuda):
    rng = np.random.default_rng(7)
    for tokens, k, experts in ((1180, 8, 256), (300, 3, 40)):
        idx = routing(rng, tokens, k, experts)
        got = without_allocation(idx, k, experts)
        want = with_workspace(idx, k, experts)
        torch.cuda.synchronize()
        for g, w in zip(got, want):
            assert torch.equal(g, w)


def test_no_alloc_tiles_reject_what_does_not_fit_their_array(cuda):
    # 262,144 pairs over 1,024 experts need 2 MiB of scratch: refused on the host, nothing launched (the
    # buffers are full-size all the same)
    pairs, k, experts = 262144, 8, 1024
    most = pairs // 16 + experts
    idx = torch.zeros(pairs, dtype=torch.int32, device="cuda")
    outs = [torch.empty(most, dtype=torch.int32, device="cuda"), torch.empty(most * 16, dtype=torch.int32, device="cuda"),
            torch.empty(pairs, dtype=torch.int32, device="cuda")]
    with pytest.raises(ValueError, match="fixed array"):
        _lib.call("smoe_tiles_of_noalloc", _lib.ptr(idx), pairs, k, experts, *(_lib.ptr(o) for o in outs), _lib.stream())


def test_no_alloc_tiles_at_the_array_limit_and_one_pair_past_it(cuda):
    # 131,072 pairs over 1,024 experts: the histograms and ranks fill the 1 MiB array exactly
    rng = np.random.default_rng(11)
    pairs, k, experts = 131072, 8, 1024
    need = int(_lib.lib().smoe_tiles_of_workspace_size(pairs, experts))
    assert need == (1 << 20) + 256
    idx = torch.from_numpy(rng.integers(0, experts, size=pairs).astype(np.int32)).cuda()
    got = without_allocation(idx, k, experts)
    want = with_workspace(idx, k, experts)
    torch.cuda.synchronize()
    for g, w in zip(got, want):
        assert torch.equal(g, w)
    # one pair more (k = 1) needs a chunk's histogram more: refused on the host
    more = torch.zeros(pairs + 1, dtype=torch.int32, device="cuda")
    with pytest.raises(ValueError, match="fixed array"):
        without_allocation(more, 1, experts)
