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


def run_rank(rank, world, device, seed):
    from strata_mlx_b200 import parallel as P

    routed, shared, router, sgate, x = layer(seed)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)  # noqa: E731
    part = P.shard_layer(dev(router), *((dev(b), k, s) for b, k, s in routed),
                         [(dev(b), k, s) for b, k, s in shared], dev(sgate), K, rank, world)
    block = P.ExpertParallelMoE(part, rank, world, E)
    got = block(dev(x)).cpu().numpy()
    logits = part.gate(dev(x)).cpu().numpy()
    want, *_ = M.moe_block(x, router, K, routed, shared, sgate, logits=logits)
    return np.linalg.norm(got.astype(np.float64) - want) / np.linalg.norm(want.astype(np.float64))


def test_one_rank_expert_parallel_block_is_the_oracles(cuda):
    assert run_rank(0, 1, cuda, 4) <= 1e-3


def _nccl_rank(rank, world, port, q):
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank), timeout=datetime.timedelta(seconds=60))
    try:
        q.put((rank, float(run_rank(rank, world, torch.device("cuda", rank), 5))))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_ranks_over_nccl_give_the_single_block(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    procs = [ctx.Process(target=_nccl_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    errs = sorted(q.get() for _ in range(2))
    assert all(e <= 1e-3 for _, e in errs), errs
