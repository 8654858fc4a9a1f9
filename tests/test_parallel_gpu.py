"""Expert parallelism on the GPU: `ExpertParallelMoE` against the oracle's MoE block (one rank here; two ranks
over NCCL when the machine has two GPUs), through the C ABI kernels."""

import datetime
import socket

import numpy as np
import pytest

from oracle import moe as M
from oracle import quants as Q

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

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
    x = rng.standard_normal((5, H)).astype(np.float16)
    return routed, shared, router, sgate, x


def run_rank(rank, world, device, seed, exchange=False, graph=False):
    """rel-L2 of the expert-parallel block on this rank against the oracle's whole block (and, with the peer
    exchange, the bits of every rank's output: a checksum the caller compares across ranks)."""
    from strata_mlx_b200 import fused as F
    from strata_mlx_b200 import parallel as P

    routed, shared, router, sgate, x = layer(seed)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)  # noqa: E731
    part = P.shard_layer(dev(router), *((dev(b), k, s) for b, k, s in routed),
                         [(dev(b), k, s) for b, k, s in shared], dev(sgate), K, rank, world)
    ex = P.PeerExchange(rank, world, H, max_tokens=8, device=device) if exchange else None
    block = P.ExpertParallelMoE(part, rank, world, E, exchange=ex)
    if graph:
        gb = F.GraphedBlock(block, x.shape[0], H, torch.float16, device)
        for _ in range(3):
            out = gb(dev(x))
        got = out.cpu().numpy()
        del gb
    else:
        got = block(dev(x)).cpu().numpy()
    failed = ex.failed() if ex is not None else False
    logits = part.gate(dev(x)).cpu().numpy()
    want, *_ = M.moe_block(x, router, K, routed, shared, sgate, logits=logits)
    err = float(np.linalg.norm(got.astype(np.float64) - want) / np.linalg.norm(want.astype(np.float64)))
    if ex is not None:
        torch.cuda.synchronize()
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        ex.close()
    return err, int(got.view(np.uint16).astype(np.int64).sum()), failed


def test_one_rank_expert_parallel_block_is_the_oracles(cuda):
    assert run_rank(0, 1, cuda, 4)[0] <= 1e-3


@pytest.mark.parametrize("graph", [False, True])
def test_one_rank_peer_exchange_block_is_the_oracles(cuda, graph):
    err, _, failed = run_rank(0, 1, cuda, 4, exchange=True, graph=graph)
    assert err <= 1e-3 and not failed


def _nccl_rank(rank, world, port, q, exchange=False, graph=False):
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank), timeout=datetime.timedelta(seconds=60))
    try:
        q.put((rank,) + run_rank(rank, world, torch.device("cuda", rank), 5, exchange, graph))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _spawn(target, world, *args):
    import torch.multiprocessing as mp

    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    procs = [ctx.Process(target=target, args=(r, world, port, q) + args) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    return sorted(q.get() for _ in range(world))


def test_two_ranks_over_nccl_give_the_single_block(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    got = _spawn(_nccl_rank, 2)
    assert all(e <= 1e-3 for _, e, _, _ in got), got


@pytest.mark.parametrize("graph", [False, True])
def test_two_ranks_over_the_peer_exchange_give_the_single_block(cuda, graph):
    """The decode step with its one exchange over NVLink peer memory: within rel-L2 1e-3 of the oracle on both
    ranks, the same bits on both (the partials are added in rank order everywhere), no wait gave up."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    got = _spawn(_nccl_rank, 2, True, graph)
    assert all(e <= 1e-3 and not failed for _, e, _, failed in got), got
    assert got[0][2] == got[1][2], got


# ---------------------------------------------------------------- a prompt chunk, tokens split over the ranks


@pytest.mark.parametrize("ranks", [1, 2, 4, 8])
@pytest.mark.parametrize("tokens", [1, 37, 2048])
def test_the_send_plan_and_rows_are_the_oracles(cuda, ranks, tokens):
    """smoe_ep_dispatch: counts, places, experts and rows bit for bit those of the oracle's plan (indices
    past the experts included: they are not sent)."""
    from strata_mlx_b200 import parallel as P

    rng = np.random.default_rng(tokens + ranks)
    experts, k, hidden = 256, 8, 4096
    idx = rng.integers(0, experts + 3, size=(tokens, k)).astype(np.uint32)
    x = rng.standard_normal((tokens, hidden)).astype(np.float16)
    counts, where, send_expert, send_x = P.dispatch(torch.from_numpy(idx).to(cuda), torch.from_numpy(x).to(cuda),
                                                   experts, ranks)
    c, wh, se, order = M.ep_plan(idx, experts, ranks)
    n = len(order)
    np.testing.assert_array_equal(counts.cpu().numpy(), c)
    np.testing.assert_array_equal(where.cpu().numpy(), wh)
    np.testing.assert_array_equal(send_expert[:n].cpu().numpy(), se)
    np.testing.assert_array_equal(send_x[:n].cpu().numpy(), x[order // k])


@pytest.mark.parametrize("k", [1, 8, 10])
def test_the_combine_through_places_is_the_combine(cuda, k):
    """smoe_combine_rows reading y at the places equals smoe_combine of the gathered y, bit for bit."""
    from strata_mlx_b200 import fused as F
    from strata_mlx_b200 import parallel as P

    rng = np.random.default_rng(k)
    tokens, d = 29, 1000
    places = rng.permutation(tokens * k).astype(np.int32)
    places[3] = -1  # a pair that was not sent adds nothing
    y_rows = rng.standard_normal((tokens * k, d)).astype(np.float16)
    w = rng.random((tokens, k)).astype(np.float32)
    g = rng.standard_normal(tokens).astype(np.float16)
    s = rng.standard_normal((tokens, d)).astype(np.float16)
    t = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    got = P.combine_rows(t(y_rows), t(places), t(w), t(g), t(s)).cpu().numpy()
    y = y_rows[np.maximum(places, 0)].reshape(tokens, k, d)
    y[places.reshape(tokens, k) < 0] = 0
    want = F.moe_combine(t(y), t(w), t(g.reshape(tokens, 1)), t(s)).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.int16), want.view(np.int16))
    np.testing.assert_array_equal(got.view(np.int16), M.combine_rows(y_rows, places, w, g, s).view(np.int16))


def run_prompt_rank(rank, world, device, seed, split):
    from strata_mlx_b200 import parallel as P

    routed, shared, router, sgate, _ = layer(seed)
    rng = np.random.default_rng(seed + 1)
    x_all = rng.standard_normal((sum(split), H)).astype(np.float16)
    x = x_all[sum(split[:rank]) : sum(split[: rank + 1])]
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)  # noqa: E731
    part = P.shard_layer(dev(router), *((dev(b), k, s) for b, k, s in routed),
                         [(dev(b), k, s) for b, k, s in shared], dev(sgate), K, rank, world, whole_shared=True)
    block = P.ExpertParallelPrompt(part, rank, world, E)
    got = block(dev(x)).cpu().numpy()
    if not x.shape[0]:
        return 0.0, block.received
    logits = part.gate(dev(x)).cpu().numpy()
    want, *_ = M.moe_block(x, router, K, routed, shared, sgate, logits=logits)
    return float(np.linalg.norm(got.astype(np.float64) - want) / np.linalg.norm(want.astype(np.float64))), block.received


@pytest.mark.parametrize("tokens", [3, 900])
def test_one_rank_prompt_chunk_is_the_oracles(cuda, tokens):
    """900 tokens x 2 pairs reach the tile products (TILES_FROM); 3 tokens stay on the matvec."""
    err, received = run_prompt_rank(0, 1, cuda, 8, (tokens,))
    assert err <= 1e-3 and received == tokens * K


def _nccl_prompt_rank(rank, world, port, split, q):
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank), timeout=datetime.timedelta(seconds=60))
    try:
        q.put((rank,) + run_prompt_rank(rank, world, torch.device("cuda", rank), 9, split))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("split", [(1200, 500)])  # ~1700 pairs a rank: tiles
def test_a_prompt_chunk_over_two_nccl_ranks_is_the_oracles(cuda, split):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    procs = [ctx.Process(target=_nccl_prompt_rank, args=(r, 2, port, split, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    got = sorted(q.get() for _ in range(2))
    assert all(e <= 1e-3 for _, e, _ in got), got
    assert sum(n for *_, n in got) == sum(split) * K
