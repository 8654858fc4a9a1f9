"""The decode step's exchange over peer memory (`smoe_ep_reduce_combine`) against the oracle: one rank, several
ranks emulated in one cooperative launch on one GPU (the arithmetic and the order of the multi-rank exchange),
a wait that runs out, and CUDA graph replays. Two real ranks over NVLink are in test_parallel_gpu.py."""

import ctypes

import numpy as np
import pytest

from oracle import moe as M

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _exchange_buffer(lib, ranks, max_tokens, d):
    nbytes = int(lib.smoe_ep_exchange_bytes(ranks, max_tokens, d))
    buf, handle = ctypes.c_void_p(), (ctypes.c_uint8 * 64)()
    assert lib.smoe_ep_exchange_alloc(nbytes, ctypes.byref(buf), handle) == 0
    return buf.value


def _rank_inputs(rng, tokens, k, d, experts, ranks, dtype=np.float16):
    """A token's k choices among `experts` split over `ranks`: every rank's y (its own pairs' rows meaningful),
    lidx (its local experts, `per` for another rank's), w, its slice of the shared expert, and the gate."""
    per = experts // ranks
    idx = np.stack([rng.choice(experts, size=k, replace=False) for _ in range(tokens)]).astype(np.int64)
    w = rng.random((tokens, k)).astype(np.float32)
    w /= w.sum(1, keepdims=True)
    g = rng.standard_normal(tokens).astype(dtype)
    ys, lidxs, ss = [], [], []
    for r in range(ranks):
        mine = (idx >= r * per) & (idx < (r + 1) * per)
        lidxs.append(np.where(mine, idx - r * per, per).astype(np.uint32))
        y = rng.standard_normal((tokens, k, d)).astype(dtype)
        y[~mine] = np.nan  # another rank's pairs: never read
        ys.append(y)
        ss.append(rng.standard_normal((tokens, d)).astype(dtype))
    return ys, w, lidxs, ss, g, per


def _specs(lib, peers, ranks, t, y, w, lidx, per, s, g, out, capacity, polls=0):
    from strata_mlx_b200 import _lib

    tokens, k = w.shape
    return _lib.SmoeEpReduce(
        0 if ranks == 1 else t, ranks, (ctypes.c_void_p * 16)(*peers), y.data_ptr(), w.data_ptr(), lidx.data_ptr(),
        per, s.data_ptr() if s is not None else None, g.data_ptr(), tokens, k, out.shape[-1], capacity,
        out.data_ptr(), _lib.dtype_code(out.dtype), polls)


@pytest.mark.parametrize("ranks", [2, 4, 8])
@pytest.mark.parametrize("tokens", [1, 3, 8])
def test_emulated_ranks_exchange_is_the_oracles(cuda, ranks, tokens):
    """Every emulated rank's output equals the oracle's rank-order sum and combine, bit for bit, and all ranks'
    outputs are the same bits; within rel-L2 1e-3 of the one-device combine of the same products."""
    from strata_mlx_b200 import _lib

    lib = _lib.lib()
    rng = np.random.default_rng(ranks * 10 + tokens)
    k, d, experts, cap = 8, 4096, 256, 8
    ys, w, lidxs, ss, g, per = _rank_inputs(rng, tokens, k, d, experts, ranks)
    bufs = [_exchange_buffer(lib, ranks, cap, d) for _ in range(ranks)]
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    w_d, g_d = t(w), t(g)
    dev = [(t(ys[r]), t(lidxs[r]), t(ss[r])) for r in range(ranks)]
    outs = [torch.full((tokens, d), float("nan"), dtype=torch.float16, device=cuda) for _ in range(ranks)]
    for rep in range(3):  # the sequence numbers and both halves of the double buffer
        specs = (_lib.SmoeEpReduce * ranks)(*[_specs(lib, bufs, ranks, r, dev[r][0], w_d, dev[r][1], per, dev[r][2], g_d,
                                                       outs[r], cap * d) for r in range(ranks)])
        _lib.call("smoe_ep_reduce_combine_emulated", ranks, specs, _lib.stream())
        torch.cuda.synchronize()
        partials = [M.partial_sums(np.nan_to_num(ys[r]), w, lidxs[r], per, ss[r]) for r in range(ranks)]
        want = M.ep_reduce_combine(partials, g)
        for r in range(ranks):
            np.testing.assert_array_equal(outs[r].cpu().numpy().view(np.int16), want.view(np.int16))
    # against the one-device combine of the same experts' outputs
    y_all = np.zeros((tokens, k, d), dtype=np.float16)
    for r in range(ranks):
        mine = lidxs[r] < per
        y_all[mine] = ys[r][mine]
    s_all = sum(ss[r].astype(np.float32) for r in range(ranks)).astype(np.float16)
    one = M.combine(y_all, w, g.reshape(tokens), s_all).astype(np.float64)
    got = outs[0].cpu().numpy().astype(np.float64)
    assert np.linalg.norm(got - one) / np.linalg.norm(one) <= 1e-3
    for b in bufs:
        flag = ctypes.c_int(1)
        assert lib.smoe_ep_exchange_status(ctypes.c_void_p(b), ctypes.byref(flag), 1) == 0 and flag.value == 0
        assert lib.smoe_ep_exchange_free(ctypes.c_void_p(b)) == 0


def test_one_rank_exchange_is_partial_sums_and_combine_sums(cuda):
    """With one rank the exchange is smoe_partial_sums then smoe_combine_sums, bit for bit; from a CUDA graph
    too (each replay counts itself in the buffer)."""
    from strata_mlx_b200 import _lib

    lib = _lib.lib()
    rng = np.random.default_rng(3)
    tokens, k, d, experts = 2, 8, 4096, 32
    ys, w, lidxs, ss, g, per = _rank_inputs(rng, tokens, k, d, experts, 4)  # this rank: the first of four's pairs
    y = np.nan_to_num(ys[0])
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    y_d, w_d, l_d, s_d, g_d = t(y), t(w), t(lidxs[0]), t(ss[0]), t(g)
    sums = torch.empty((tokens, 2 * d), dtype=torch.float32, device=cuda)
    want = torch.empty((tokens, d), dtype=torch.float16, device=cuda)
    _lib.call("smoe_partial_sums", _lib.ptr(y_d), _lib.ptr(w_d), _lib.ptr(l_d), per, _lib.ptr(s_d), tokens, k, d,
              _lib.ptr(sums), _lib.F16, _lib.stream())
    _lib.call("smoe_combine_sums", _lib.ptr(sums), _lib.ptr(g_d), tokens, d, _lib.ptr(want), _lib.F16, _lib.stream())
    buf = _exchange_buffer(lib, 1, 4, d)
    out = torch.empty((tokens, d), dtype=torch.float16, device=cuda)
    spec = _specs(lib, [buf], 1, 0, y_d, w_d, l_d, per, s_d, g_d, out, 4 * d)
    _lib.call("smoe_ep_reduce_combine", ctypes.byref(spec), _lib.stream())
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), want.view(torch.int16))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        _lib.call("smoe_ep_reduce_combine", ctypes.byref(spec), _lib.stream())
    for _ in range(5):
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), want.view(torch.int16))
    del graph
    flag = ctypes.c_int(1)
    assert lib.smoe_ep_exchange_status(ctypes.c_void_p(buf), ctypes.byref(flag), 1) == 0 and flag.value == 0
    assert lib.smoe_ep_exchange_free(ctypes.c_void_p(buf)) == 0


def test_a_rank_that_never_arrives_gives_a_status_not_a_hang(cuda):
    """Two ranks, the second's buffer in this process and never written by anyone: this rank's wait for it runs
    out after its poll limit, the status says SMOE_ETIMEOUT, the outputs are left as they were, and the device
    stays usable (a one-rank call right after is exact)."""
    from strata_mlx_b200 import _lib

    lib = _lib.lib()
    rng = np.random.default_rng(4)
    tokens, k, d, experts = 1, 8, 4096, 256
    ys, w, lidxs, ss, g, per = _rank_inputs(rng, tokens, k, d, experts, 2)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    y_d, w_d, l_d, s_d, g_d = t(np.nan_to_num(ys[0])), t(w), t(lidxs[0]), t(ss[0]), t(g)
    mine, silent = _exchange_buffer(lib, 2, 1, d), _exchange_buffer(lib, 2, 1, d)
    out = torch.full((tokens, d), 7.0, dtype=torch.float16, device=cuda)
    spec = _specs(lib, [mine, silent], 2, 0, y_d, w_d, l_d, per, s_d, g_d, out, d, polls=2000)
    _lib.call("smoe_ep_reduce_combine", ctypes.byref(spec), _lib.stream())
    flag = ctypes.c_int(0)
    assert lib.smoe_ep_exchange_status(ctypes.c_void_p(mine), ctypes.byref(flag), 1) == 0
    assert flag.value == _lib.ETIMEOUT
    assert bool((out == 7.0).all())
    assert lib.smoe_ep_exchange_status(ctypes.c_void_p(mine), ctypes.byref(flag), 0) == 0 and flag.value == 0
    # the context is fine: a one-rank exchange right after
    one = _exchange_buffer(lib, 1, 1, d)
    spec1 = _specs(lib, [one], 1, 0, y_d, w_d, l_d, per, s_d, g_d, out, d)
    _lib.call("smoe_ep_reduce_combine", ctypes.byref(spec1), _lib.stream())
    torch.cuda.synchronize()
    want = M.ep_reduce_combine([M.partial_sums(np.nan_to_num(ys[0]), w, lidxs[0], per, ss[0])], g)
    np.testing.assert_array_equal(out.cpu().numpy().view(np.int16), want.view(np.int16))
    for b in (mine, silent, one):
        assert lib.smoe_ep_exchange_free(ctypes.c_void_p(b)) == 0


def test_the_exchange_refuses_what_it_was_not_made_for(cuda):
    from strata_mlx_b200 import _lib

    lib = _lib.lib()
    assert lib.smoe_ep_exchange_bytes(17, 1, 4096) == 0 and lib.smoe_ep_exchange_bytes(2, 0, 4096) == 0
    buf = _exchange_buffer(lib, 2, 1, 64)
    z = torch.zeros(64, dtype=torch.float16, device=cuda)
    w = torch.ones((2, 1), dtype=torch.float32, device=cuda)
    l = torch.zeros((2, 1), dtype=torch.int32, device=cuda)
    spec = _specs(lib, [buf, buf], 2, 0, z, w, l, 1, None, z, torch.empty((2, 64), dtype=torch.float16, device=cuda),
                  64)
    with pytest.raises(ValueError, match="more tokens"):
        _lib.call("smoe_ep_reduce_combine", ctypes.byref(spec), _lib.stream())
    assert lib.smoe_ep_exchange_free(ctypes.c_void_p(buf)) == 0
