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
