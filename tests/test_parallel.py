"""Expert parallelism, host side (no GPU): the sharding helpers and the split of the MoE block at its combine,
run as two `gloo` ranks on the CPU with the oracle doing each rank's products."""

import datetime
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import moe as M
from oracle import quants as Q
from strata_mlx_b200 import parallel as P

H, F_, E, FS, K = 512, 256, 8, 512, 2


def layer(seed):
    rng = np.random.default_rng(seed)

    def blocks(kind, rows, cols, experts=1):
        return Q.random_blocks(kind, experts * rows * cols // Q.TYPES[kind][1], rng, normal=0.001).reshape(-1)

    routed = [(blocks("IQ3_S", F_, H, E), "IQ3_S", (E, F_, H)), (blocks("IQ3_S", F_, H, E), "IQ3_S", (E, F_, H)),
              (blocks("IQ3_S", H, F_, E), "IQ3_S", (E, H, F_))]
    shared = [(blocks("Q8_0", FS, H), "Q8_0", (FS, H)), (blocks("Q8_0", FS, H), "Q8_0", (FS, H)),
              (blocks("Q8_0", H, FS), "Q8_0", (H, FS))]
    router = (0.02 * rng.standard_normal((E, H))).astype(np.float16)
    sgate = (0.02 * rng.standard_normal((1, H))).astype(np.float16)
    x = rng.standard_normal((3, H)).astype(np.float16)
    return routed, shared, router, sgate, x


def test_expert_ranges_cover_the_experts_once():
    seen = []
    for r in range(4):
        lo, n = P.expert_range(r, 4, 256)
        seen += list(range(lo, lo + n))
    assert seen == list(range(256))
    with pytest.raises(ValueError):
        P.expert_range(0, 3, 256)


def test_shards_and_slices_hold_the_right_weights():
    routed, shared, *_ = layer(1)
    b, kind, shape = routed[0]
    full = Q.dequantize(b, kind, shape)
    for r in range(2):
        lb, ls = P.shard_stack(torch.from_numpy(b), kind, shape, r, 2)
        np.testing.assert_array_equal(Q.dequantize(lb.numpy(), kind, ls), full[r * 4 : r * 4 + 4])
    db, dk, (rows, cols) = shared[2]
    full = Q.dequantize(db, dk, (rows, cols))
    part = P.slice_cols(torch.from_numpy(db), dk, (rows, cols), 128, 256).numpy()
    np.testing.assert_array_equal(Q.dequantize(part, dk, (rows, 128)), full[:, 128:256])
    gb, gk, (rows, cols) = shared[0]
    part = P.slice_rows(torch.from_numpy(gb), gk, (rows, cols), 64, 192).numpy()
    np.testing.assert_array_equal(Q.dequantize(part, gk, (128, cols)), Q.dequantize(gb, gk, (rows, cols))[64:192])


def _rank(rank, world, port, seed, q):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        routed, shared, router, sgate, x = layer(seed)
        # the rank's shards, cut by the product's helpers
        local = []
        for b, kind, shape in routed:
            lb, ls = P.shard_stack(torch.from_numpy(b), kind, shape, rank, world)
            local.append((lb.numpy(), kind, ls))
        lo, n = P.expert_range(rank, world, FS)
        (gb, gk, gs), (ub, uk, us), (db, dk, ds) = shared
        sh = [(P.slice_rows(torch.from_numpy(gb), gk, gs, lo, lo + n).numpy(), gk, (n, H)),
              (P.slice_rows(torch.from_numpy(ub), uk, us, lo, lo + n).numpy(), uk, (n, H)),
              (P.slice_cols(torch.from_numpy(db), dk, ds, lo, lo + n).numpy(), dk, (H, n))]
        # what the rank's kernels compute, done by the oracle: routing (replicated), its pairs, its slice
        logits = M.router_logits(router, x)
        idx = M.top_k(logits, K)
        w = M.softmax_chosen(logits, idx)
        elo, ecount = P.expert_range(rank, world, E)
        lidx = np.where((idx >= elo) & (idx < elo + ecount), idx - elo, ecount)
        y = np.zeros((x.shape[0], K, H), dtype=np.float16)
        for t in range(x.shape[0]):
            for j in range(K):
                if lidx[t, j] < ecount:
                    y[t, j] = M.switch_glu(x[t : t + 1], lidx[t : t + 1, j : j + 1], *local)[0, 0]
        s = M.dense_mlp(x, *sh)
        sums = torch.from_numpy(M.partial_sums(y, w, lidx, ecount, s))
        dist.all_reduce(sums)  # the one collective of the step
        g = (x.astype(np.float64) @ sgate.astype(np.float64).reshape(-1)).astype(np.float16)
        out = M.combine_sums(sums.numpy(), g)
        want, *_ = M.moe_block(x, router, K, routed, shared, sgate)
        err = np.linalg.norm(out.astype(np.float64) - want) / np.linalg.norm(want.astype(np.float64))
        q.put((rank, float(err)))
    finally:
        dist.destroy_process_group()


def test_two_ranks_over_gloo_give_the_single_block():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, 3, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    errs = sorted(q.get() for _ in range(2))
    assert all(e <= 1e-3 for _, e in errs), errs


def test_the_send_plan_keeps_pair_order_within_each_destination():
    """oracle ep_plan against a direct statement: destinations in rank order, pairs in order within each."""
    rng = np.random.default_rng(11)
    idx = rng.integers(0, 66, size=(37, 8))  # 64 experts; 64 and 65 are out of range and stay home
    counts, where, send_expert, order = M.ep_plan(idx, 64, 4)
    flat = idx.reshape(-1)
    want = [i for r in range(4) for i in range(flat.size) if flat[i] < 64 and flat[i] // 16 == r]
    np.testing.assert_array_equal(order, want)
    np.testing.assert_array_equal(counts, [sum(1 for i in want if flat[i] // 16 == r) for r in range(4)])
    assert all(where[i] == -1 for i in range(flat.size) if flat[i] >= 64)
    np.testing.assert_array_equal(where[order], np.arange(len(want)))
    np.testing.assert_array_equal(send_expert, flat[order] % 16)


def _prompt_rank(rank, world, port, seed, split, q):
    """One rank of a prompt chunk: its tokens routed, the pairs sent by the product's exchange helpers, the
    received pairs' products and the combine done by the oracle."""
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        routed, shared, router, sgate, _ = layer(seed)
        rng = np.random.default_rng(seed + 1)
        x_all = rng.standard_normal((sum(split), H)).astype(np.float16)
        x = x_all[sum(split[:rank]) : sum(split[: rank + 1])]
        local = []
        for b, kind, shape in routed:
            lb, ls = P.shard_stack(torch.from_numpy(b), kind, shape, rank, world)
            local.append((lb.numpy(), kind, ls))
        logits = M.router_logits(router, x)
        idx = M.top_k(logits, K)
        w = M.softmax_chosen(logits, idx)
        counts, where, send_expert, order = M.ep_plan(idx, E, world)
        send_x = x[order // K]
        recv_counts = P.exchange_counts(torch.from_numpy(counts))
        send, recv = counts.tolist(), recv_counts.tolist()
        rows = P.exchange_rows(torch.from_numpy(send_x), send, recv).numpy()
        experts = P.exchange_rows(torch.from_numpy(send_expert), send, recv).numpy()
        y = np.zeros((rows.shape[0], H), dtype=np.float16)
        for i in range(rows.shape[0]):
            y[i] = M.switch_glu(rows[i : i + 1], experts[i : i + 1].reshape(1, 1).astype(np.int64), *local)[0, 0]
        back = P.exchange_rows(torch.from_numpy(y), recv, send).numpy()
        s = M.dense_mlp(x, *shared)
        g = (x.astype(np.float64) @ sgate.astype(np.float64).reshape(-1)).astype(np.float16)
        out = M.combine_rows(back, where, w, g, s)
        if x.shape[0]:
            want, *_ = M.moe_block(x, router, K, routed, shared, sgate)
            err = np.linalg.norm(out.astype(np.float64) - want) / np.linalg.norm(want.astype(np.float64))
        else:
            err = 0.0
        q.put((rank, float(err), int(rows.shape[0])))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("split", [(4, 3), (5, 0)])
def test_a_prompt_chunk_over_two_gloo_ranks_gives_each_ranks_tokens_the_single_block(split):
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    procs = [ctx.Process(target=_prompt_rank, args=(r, 2, port, 6, split, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    got = sorted(q.get() for _ in range(2))
    assert all(e <= 1e-3 for _, e, _ in got), got
    assert sum(n for *_, n in got) == sum(split) * K  # every pair computed once, somewhere


class _OracleLayer:
    """A rank's layer whose products are the oracle's, on CPU tensors: stands in for the CUDA kernels so that
    `ExpertParallelPrompt.__call__` itself (its exchanges, the empty-rank case) runs on gloo ranks."""

    def __init__(self, router, local, shared, sgate, k):
        self.router, self.local, self.shared, self.sgate, self.top_k = router, local, shared, sgate, k
        self.gate = lambda x: torch.from_numpy(M.router_logits(self.router, x.numpy()).astype(np.float32))
        self.shared_expert_gate = lambda x: torch.from_numpy(
            (x.numpy().astype(np.float64) @ self.sgate.astype(np.float64).reshape(-1, 1)).astype(np.float16))
        self.shared_expert = lambda x: torch.from_numpy(M.dense_mlp(x.numpy(), *self.shared))

    def switch_mlp(self, rows, local):
        e = local.view(torch.int32).numpy().astype(np.int64)
        y = np.stack([M.switch_glu(rows[i : i + 1].numpy(), e[i : i + 1], *self.local)[0] for i in range(rows.shape[0])])
        return torch.from_numpy(y)


def _oracle_top_k_softmax(logits, k):
    lg = logits.numpy()
    idx = M.top_k(lg, k)
    return torch.from_numpy(idx.astype(np.int64)).to(torch.int32).view(torch.uint32), torch.from_numpy(
        M.softmax_chosen(lg, idx).astype(np.float32))


def _oracle_dispatch(idx, x, experts, world):
    pairs = idx.numel()
    counts, where, send_expert, order = M.ep_plan(idx.view(torch.int32).numpy(), experts, world)
    k = idx.shape[-1]
    sx = np.zeros((pairs, x.shape[-1]), dtype=np.float16)
    sx[: order.size] = x.numpy()[order // k]
    se = np.zeros(pairs, dtype=np.int32)
    se[: order.size] = send_expert.astype(np.int32)
    return (torch.from_numpy(counts), torch.from_numpy(where), torch.from_numpy(se).view(torch.uint32),
            torch.from_numpy(sx))


def _oracle_combine_rows(y, where, w, g, s):
    return torch.from_numpy(M.combine_rows(y.numpy(), where.numpy(), w.numpy(), g.numpy().reshape(-1), s.numpy()))


def _class_rank(rank, world, port, seed, split, q):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        P.top_k_softmax, P.dispatch, P.combine_rows = _oracle_top_k_softmax, _oracle_dispatch, _oracle_combine_rows
        routed, shared, router, sgate, _ = layer(seed)
        rng = np.random.default_rng(seed + 1)
        x_all = rng.standard_normal((sum(split), H)).astype(np.float16)
        x = x_all[sum(split[:rank]) : sum(split[: rank + 1])]
        local = []
        for b, kind, shape in routed:
            lb, ls = P.shard_stack(torch.from_numpy(b), kind, shape, rank, world)
            local.append((lb.numpy(), kind, ls))
        block = P.ExpertParallelPrompt(_OracleLayer(router, local, shared, sgate, K), rank, world, E)
        got = block(torch.from_numpy(x)).numpy()
        assert got.shape == x.shape
        err = 0.0
        if x.shape[0]:
            want, *_ = M.moe_block(x, router, K, routed, shared, sgate)
            err = float(np.linalg.norm(got.astype(np.float64) - want) / np.linalg.norm(want.astype(np.float64)))
        q.put((rank, err, int(block.received)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("split", [(4, 3), (5, 0), (0, 6)])
def test_the_prompt_class_over_two_gloo_ranks_with_oracle_products(split):
    """`ExpertParallelPrompt.__call__` on two gloo ranks, its kernels replaced by the oracle: every rank's
    tokens get the single block's output, a rank without tokens routes one zero token and returns none."""
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    procs = [ctx.Process(target=_class_rank, args=(r, 2, port, 7, split, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    got = sorted(q.get() for _ in range(2))
    assert all(e <= 1e-3 for _, e, _ in got), got
    # every pair computed once; the empty rank's zero token adds its K pairs
    assert sum(n for *_, n in got) == sum(split) * K + K * sum(1 for t in split if t == 0)
