"""Benchmark of the MoE hot path: the headline configuration 2, one MoE layer decoding one token (batch 1).

Workload (the benchmark's configs[1]): hidden 4096 float16 ~N(0,1); router float16 [256 x 4096] ~N(0,0.02); top-8 with
the softmax over the chosen; 256 experts with gate/up [1536 x 4096] and down [4096 x 1536] in IQ3_S blocks
(uniform random bytes, float16 super-scale |N(0,0.02)|); a shared expert of ffn 4096 in Q8_0 with its float16
sigmoid gate; SwiGLU; weighted combine. A step is one token through one such layer. Steps cycle through
`--layers` independent layers (default 8, 2.13 GB each) so that no step finds its weights in the 126 MB L2.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

value    token-layers/s with the token already in HBM (device-timed with CUDA events, max over ranks)
e2e      the same through the public API (`GraphedBlock.__call__` in its host_io mode) with every step copying
         its token from pinned host memory and its result back to pinned host memory
roofline the dominant kernel (the step's batched gate/up: 16 IQ3_S matrices of 1536 x 4096 and the shared
         expert's two Q8_0 4096 x 4096 in one launch) against the measured HBM copy bandwidth: algorithmic
         bytes per launch / its CUDA-event time
cpu_baseline  the oracle port (numpy: decode of the chosen experts' blocks + products) on the host's cores
prefill  configuration 3: a 1,180-token prompt chunk through a Q2_K layer, Zipf-routed, and its tile products
verify   configuration 4: a 5-token verify pass through 8 layers cycling the nine block types
stack    configuration 5: 26 IQ3_S layers, a 32,768-token prompt in 2,048-token chunks, decode at batch 1 and 8

With --gpus N > 1 (torchrun, one process per GPU, NCCL) the experts are sharded 256/N per rank and the
shared expert's ffn N ways; every rank routes the token, computes its own experts' weighted sum and its slice
of the shared expert, and one NCCL all-reduce of the [1, 4096] float32 partial sums ends the step;
`--ep-prefill` and `--stack` add configurations 3 and 5 over the ranks (all-to-all dispatch of prompt pairs).
`--impl reference` times the reference's CPU path (the oracle port, all host cores) on the same workload.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H, F_, E, FS, K = 4096, 1536, 256, 4096, 8
KIND, SHARED_KIND = "IQ3_S", "Q8_0"
SIGMA = 0.02


def _args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--layers", type=int, default=8)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--cpu-steps", type=int, default=2, help="decode steps of the CPU baseline sample")
    p.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline (profiling runs)")
    p.add_argument("--no-prefill", action="store_true", help="skip the config-3 prefill measurement")
    p.add_argument("--only-prefill", action="store_true", help="only the config-3 prefill measurement (profiling)")
    p.add_argument("--no-verify", action="store_true", help="skip the config-4 verify-pass measurement")
    p.add_argument("--no-stack", action="store_true", help="skip the config-5 stack measurement")
    p.add_argument("--only-stack", action="store_true", help="only the config-5 stack measurement")
    p.add_argument("--stack-layers", type=int, default=26)
    p.add_argument("--only-verify", action="store_true", help="only the config-4 verify-pass measurement")
    p.add_argument("--only-matvec", metavar="KIND", help="profiling: the decode matvec of config 4's down "
                   "product (40 pairs of 5 tokens, 64 experts of 4096 x 1536 KIND blocks), a few launches")
    return p.parse_args()


# ---------------------------------------------------------------- CPU baseline (oracle port)

def _cpu_matrix(job):
    """One matrix-vector product the CPU way: decode the blocks with the oracle, then a BLAS product."""
    import numpy as np

    from oracle import quants as Q

    blocks, kind, rows, cols, x = job
    w = Q.dequantize(blocks, kind, (rows, cols))
    # the config's scales make the down product's input overflow float16 (inf times zero weights is NaN):
    # expected, as on the GPU, and no concern of the timing
    with np.errstate(invalid="ignore", over="ignore"):
        return w @ x.astype(np.float32)


def cpu_step_inputs(seed):
    """The host-side inputs of one decode step (the 8 chosen experts' blocks and the shared expert's)."""
    import numpy as np

    from oracle import quants as Q

    rng = np.random.default_rng(seed)

    def blocks(kind, rows, cols):
        per = Q.TYPES[kind][1]
        return Q.random_blocks(kind, rows * cols // per, rng, normal=SIGMA).reshape(-1)

    routed = [(blocks(KIND, F_, H), blocks(KIND, F_, H), blocks(KIND, H, F_)) for _ in range(K)]
    shared = (blocks(SHARED_KIND, FS, H), blocks(SHARED_KIND, FS, H), blocks(SHARED_KIND, H, FS))
    router = (0.02 * rng.standard_normal((E, H))).astype(np.float16)
    sgate = (0.02 * rng.standard_normal(H)).astype(np.float16)
    x = rng.standard_normal(H).astype(np.float16)
    return routed, shared, router, sgate, x


def cpu_decode_step(pool, inputs):
    """The reference's CPU path for one token through one layer: router product, top-k, softmax, the chosen
    experts decoded from their blocks and multiplied (gate/up, then down), the shared expert, the combine."""
    import numpy as np

    from oracle import moe as M

    routed, shared, router, sgate, x = inputs
    logits = M.router_logits(router, x[None])
    idx = M.top_k(logits, K)[0]
    w = M.softmax_chosen(logits, idx[None])[0]
    x32 = x.astype(np.float32)
    gu = pool.map(_cpu_matrix, [(routed[j][p], KIND, F_, H, x32) for j in range(K) for p in (0, 1)]
                  + [(shared[p], SHARED_KIND, FS, H, x32) for p in (0, 1)])
    hs = [M.swiglu(gu[2 * j], gu[2 * j + 1]) for j in range(K + 1)]
    down = pool.map(_cpu_matrix, [(routed[j][2], KIND, H, F_, hs[j]) for j in range(K)]
                    + [(shared[2], SHARED_KIND, H, FS, hs[K])])
    y = np.stack(down[:K]).astype(np.float16)[None]
    g = np.float16(x32 @ sgate.astype(np.float32))
    return M.combine(y, w[None], np.array([g]), down[K].astype(np.float16)[None])


def cpu_baseline(steps, seed, warmup=1):
    """Time `steps` decode steps of the CPU path with a spawn pool over all host cores (bounded sample), each
    step decoding the chosen experts' blocks; then the same steps with the weights decoded beforehand."""
    import multiprocessing as mp

    cores = os.cpu_count() or 1
    ctx = mp.get_context("spawn")
    inputs = cpu_step_inputs(seed)
    with ctx.Pool(cores) as pool:
        for _ in range(max(1, warmup)):
            cpu_decode_step(pool, inputs)  # (the first also warms the workers)
        t0 = time.perf_counter()
        for _ in range(steps):
            cpu_decode_step(pool, inputs)
        dt = time.perf_counter() - t0
    out = {"value": steps / dt, "unit": "token-layers/s", "cores": cores, "kind": "port",
           "sample": f"{steps} decode steps of config 2 (8 IQ3_S experts decoded from blocks + Q8_0 shared expert, "
                     f"numpy oracle, {cores}-process pool), {dt:.1f} s"}
    out["product_only"] = cpu_product_only(inputs, 50)
    return out


def cpu_product_only(inputs, steps):
    """The CPU path with the weights decoded beforehand (float32 arrays of the 8 chosen experts and the shared
    expert, made outside the timing): per step the router, top-k, softmax, the 27 matrix-vector products (numpy
    BLAS with every host core), SwiGLU and the combine."""
    import numpy as np

    from oracle import moe as M
    from oracle import quants as Q

    routed, shared, router, sgate, x = inputs
    wr = [[Q.dequantize(routed[j][p], KIND, (F_, H) if p < 2 else (H, F_)) for p in range(3)] for j in range(K)]
    ws = [Q.dequantize(shared[p], SHARED_KIND, (FS, H) if p < 2 else (H, FS)) for p in range(3)]
    cores = os.cpu_count() or 1

    def step():
        with np.errstate(invalid="ignore", over="ignore"):
            logits = M.router_logits(router, x[None])
            idx = M.top_k(logits, K)[0]
            w = M.softmax_chosen(logits, idx[None])[0]
            x32 = x.astype(np.float32)
            hs = [M.swiglu(wr[j][0] @ x32, wr[j][1] @ x32) for j in range(K)]
            y = np.stack([wr[j][2] @ hs[j] for j in range(K)]).astype(np.float16)[None]
            s = ws[2] @ M.swiglu(ws[0] @ x32, ws[1] @ x32)
            g = np.float16(x32 @ sgate.astype(np.float32))
            return M.combine(y, w[None], np.array([g]), s.astype(np.float16)[None])

    from threadpoolctl import threadpool_limits

    with threadpool_limits(cores):
        step()
        t0 = time.perf_counter()
        for _ in range(steps):
            step()
        dt = time.perf_counter() - t0
    return {"value": steps / dt, "unit": "token-layers/s", "threads": cores,
            "sample": f"{steps} decode steps of config 2 with the 8 chosen experts' and the shared expert's weights "
                      f"decoded to float32 beforehand (numpy BLAS), {dt:.2f} s"}


# ---------------------------------------------------------------- GPU workload

def make_layers(n_layers, seed, device, rank=0, world=1, sigma=SIGMA):
    """`n_layers` independent layers of random blocks on the device, as configuration 2 of the benchmark describes
    them. Every rank draws the same layers (the seed does not depend on the rank); with world > 1 each rank then
    keeps its experts [rank E/world, (rank+1) E/world) of every stack and its slice of the shared expert's ffn,
    so the ranks' parts add up to the one-GPU layer (the router and the shared gate whole on every rank)."""
    import torch

    from strata_mlx_b200 import blocks as B
    from strata_mlx_b200 import fused as Fz
    from strata_mlx_b200 import parallel as P

    g = torch.Generator(device=device)
    g.manual_seed(seed)

    def random_blocks(kind, n_weights):
        per, nbytes = B.BLOCK[kind]
        n = n_weights // per
        b = torch.randint(0, 256, (n, nbytes), dtype=torch.uint8, device=device, generator=g)
        scale = (torch.randn(n, device=device, generator=g) * sigma).abs().half()
        b[:, 0:2] = scale.view(torch.uint8).view(n, 2)
        return b.reshape(-1)

    layers = []
    for _ in range(n_layers):
        stacks = [(random_blocks(KIND, E * F_ * H), KIND, (E, F_, H)), (random_blocks(KIND, E * F_ * H), KIND, (E, F_, H)),
                  (random_blocks(KIND, E * H * F_), KIND, (E, H, F_))]
        shared = [(random_blocks(SHARED_KIND, FS * H), SHARED_KIND, (FS, H)),
                  (random_blocks(SHARED_KIND, FS * H), SHARED_KIND, (FS, H)),
                  (random_blocks(SHARED_KIND, H * FS), SHARED_KIND, (H, FS))]
        router = (torch.randn(E, H, device=device, generator=g) * 0.02).half()
        sgate = (torch.randn(1, H, device=device, generator=g) * 0.02).half()
        if world == 1:
            layers.append(Fz.SparseMoeBlock(router, B.BlockSwitchGLU(*(B.BlockSwitchLinear(*st) for st in stacks)),
                                            B.BlockMLP(*(B.BlockLinear(*sh) for sh in shared)), sgate, K))
            continue
        part = P.shard_layer(router, *stacks, shared, sgate, K, rank, world)
        # own copies of this rank's bytes, so that the whole layer's are freed
        for lin in (part.switch_mlp.gate_proj, part.switch_mlp.up_proj, part.switch_mlp.down_proj):
            lin.blocks = lin.blocks.clone()
        for lin in (part.shared_expert.gate_proj, part.shared_expert.up_proj, part.shared_expert.down_proj):
            lin.stack.blocks = lin.stack.blocks.clone()
        layers.append(part)
        del stacks, shared
    return layers


def parity_ep(device, seed, rank, world, exchange, tokens=1):
    """rel-L2 of the expert-parallel block (this rank's part, through the exchange) against the same layer
    whole on this GPU, at |N(0, 0.001)| super-scales (where every output is finite): configuration 2's shapes."""
    import torch

    from strata_mlx_b200 import blocks as B
    from strata_mlx_b200 import fused as Fz
    from strata_mlx_b200 import parallel as P

    g = torch.Generator(device=device)
    g.manual_seed(seed)

    def random_blocks(kind, n_weights):
        per, nbytes = B.BLOCK[kind]
        n = n_weights // per
        b = torch.randint(0, 256, (n, nbytes), dtype=torch.uint8, device=device, generator=g)
        b[:, 0:2] = (torch.randn(n, device=device, generator=g) * 0.001).abs().half().view(torch.uint8).view(n, 2)
        return b.reshape(-1)

    stacks = [(random_blocks(KIND, E * F_ * H), KIND, (E, F_, H)), (random_blocks(KIND, E * F_ * H), KIND, (E, F_, H)),
              (random_blocks(KIND, E * H * F_), KIND, (E, H, F_))]
    shared = [(random_blocks(SHARED_KIND, FS * H), SHARED_KIND, (FS, H)),
              (random_blocks(SHARED_KIND, FS * H), SHARED_KIND, (FS, H)),
              (random_blocks(SHARED_KIND, H * FS), SHARED_KIND, (H, FS))]
    router = (torch.randn(E, H, device=device, generator=g) * 0.02).half()
    sgate = (torch.randn(1, H, device=device, generator=g) * 0.02).half()
    x = torch.randn(tokens, H, device=device, generator=g).half()
    whole = Fz.SparseMoeBlock(router, B.BlockSwitchGLU(*(B.BlockSwitchLinear(*st) for st in stacks)),
                              B.BlockMLP(*(B.BlockLinear(*sh) for sh in shared)), sgate, K)
    want = whole(x).double()
    ep = P.ExpertParallelMoE(P.shard_layer(router, *stacks, shared, sgate, K, rank, world), rank, world, E,
                             exchange=exchange)
    got = ep(x).double()
    torch.cuda.synchronize()
    return float((got - want).norm() / want.norm())


def run_prefill(device, seed, steps=5, warmup=2, rank=0, world=1):
    """Configuration 3 of the benchmark: the same layer shapes in Q2_K (gate/up 1536 x 4096, down 4096 x 1536, 256 experts), a
    prompt chunk of 1180 tokens ~N(0,1), router logits biased so expert load is Zipf-skewed (s = 1.1): the
    router weight carries log p_e along a unit direction u that every token has a component 1 along. Times the
    whole block (router, top-k, tiles_of, three tensor-core tile products, SwiGLU, the shared expert on the
    tile product, combine) and the three routed tile products alone.

    With world > 1 every rank makes the same layer and chunk, keeps its experts (E / world) and the whole
    shared expert, and takes a contiguous share of the tokens; the block is `ExpertParallelPrompt` (all-to-all
    dispatch and return over NCCL), timed on every rank with CUDA events, the maximum over ranks reported."""
    import torch

    from strata_mlx_b200 import blocks as B
    from strata_mlx_b200 import fused as Fz

    T, kind = 1180, "Q2_K"
    g = torch.Generator(device=device)
    g.manual_seed(seed)

    def random_blocks(kd, n_weights):
        per, nbytes = B.BLOCK[kd]
        n = n_weights // per
        b = torch.randint(0, 256, (n, nbytes), dtype=torch.uint8, device=device, generator=g)
        for at in ((80, 82) if kd == "Q2_K" else (0,)):
            b[:, at : at + 2] = (torch.randn(n, device=device, generator=g) * SIGMA).abs().half().view(torch.uint8).view(n, 2)
        return b.reshape(-1)

    gate = B.BlockSwitchLinear(random_blocks(kind, E * F_ * H), kind, (E, F_, H))
    up = B.BlockSwitchLinear(random_blocks(kind, E * F_ * H), kind, (E, F_, H))
    down = B.BlockSwitchLinear(random_blocks(kind, E * H * F_), kind, (E, H, F_))
    shared = B.BlockMLP(B.BlockLinear(random_blocks(SHARED_KIND, FS * H), SHARED_KIND, (FS, H)),
                        B.BlockLinear(random_blocks(SHARED_KIND, FS * H), SHARED_KIND, (FS, H)),
                        B.BlockLinear(random_blocks(SHARED_KIND, H * FS), SHARED_KIND, (H, FS)))
    zipf = torch.empty(E, device=device)  # each expert's place in the Zipf order
    zipf[torch.randperm(E, device=device, generator=g)] = torch.arange(1, E + 1, device=device, dtype=torch.float32)
    logp = -1.1 * torch.log(zipf)
    logp -= torch.logsumexp(logp, 0)
    u = torch.randn(H, device=device, generator=g)
    u /= u.norm()
    router = (torch.randn(E, H, device=device, generator=g) * 0.02 + logp[:, None] * u[None, :]).half()
    sgate = (torch.randn(1, H, device=device, generator=g) * 0.02).half()
    block = Fz.SparseMoeBlock(router, B.BlockSwitchGLU(gate, up, down), shared, sgate, K)
    x = torch.randn(T, H, device=device, generator=g)
    x = (x - (x @ u)[:, None] * u[None, :] + u[None, :]).half()
    if world > 1:
        return _prefill_ep(block, x, steps, warmup, rank, world)

    for _ in range(warmup):
        block(x)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        block(x)
    e1.record()
    torch.cuda.synchronize()
    layer_ms = e0.elapsed_time(e1) / steps

    # the routed tile products alone, on this chunk's tiles, as the layer launches them: gate and up in one
    # launch (float32 sums), down in the rows form (float16 in pair order)
    idx = Fz.top_k(block.gate(x), K)
    tiles, token, where = B.tiles_of(idx, E)
    a = x.index_select(0, token.view(torch.int32).long())
    hsz = torch.empty(a.shape[0], F_, dtype=torch.float16, device=device).normal_()
    srow = B.slot_rows(where, a.shape[0])

    def products():
        B.tile_matmul_pair(gate, up, a, tiles)
        B.tile_matmul_rows(down.blocks, down.kind, down.shape, hsz, tiles, srow, T * K)

    products()
    torch.cuda.synchronize()
    e0.record()
    for _ in range(steps):
        products()
    e1.record()
    torch.cuda.synchronize()
    gemm_ms = e0.elapsed_time(e1) / steps
    pairs = T * K
    counts = torch.bincount(idx.view(torch.int32).reshape(-1).long(), minlength=E)
    flops = 2.0 * pairs * 3 * F_ * H
    return {"workload": "config 3: one MoE layer, prefill chunk of 1180 tokens, 256 Q2_K experts, top-8, Zipf s=1.1 "
                        "routing, shared expert ffn 4096 Q8_0",
            "layer_ms": layer_ms, "tokens_per_s": T / (layer_ms * 1e-3),
            "routed_gemm_ms": gemm_ms, "routed_gemm_tflops": flops / (gemm_ms * 1e-3) / 1e12,
            "routed_gflop": flops / 1e9, "experts_hit": int((counts > 0).sum().item()),
            "max_pairs_per_expert": int(counts.max().item())}


def run_config1(device, seed, steps=200, cpu_steps=3):
    """Configuration 1 of the benchmark: one expert's matrix-vector product, W [1536 x 4096] in IQ3_S blocks
    (2,703,360 bytes), x float16 [4096] ~N(0,1). The GPU takes W from a stack of 256 such experts (692 MB, more
    than L2), a different expert each step, through `BlockSwitchLinear` (the int8 tensor-core decode matvec);
    the CPU decodes the same blocks with the oracle port and multiplies with numpy (all host threads), and the
    product alone with the weights decoded beforehand."""
    import numpy as np
    import torch

    from oracle import quants as Q
    from strata_mlx_b200 import blocks as B

    experts, rows, cols = 256, F_, H
    rng = np.random.default_rng(seed)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    per, nbytes = B.BLOCK[KIND]
    n = experts * rows * cols // per
    b = torch.randint(0, 256, (n, nbytes), dtype=torch.uint8, device=device, generator=g)
    b[:, 0:2] = (torch.randn(n, device=device, generator=g) * SIGMA).abs().half().view(torch.uint8).view(n, 2)
    lin = B.BlockSwitchLinear(b.reshape(-1), KIND, (experts, rows, cols))
    x = torch.randn(1, 1, cols, device=device, generator=g).half()
    idxs = [torch.tensor([[e]], dtype=torch.int32, device=device) for e in range(experts)]
    for i in range(5):
        lin(x, idxs[i])
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        lin(x, idxs[(37 * i) % experts])
    e1.record()
    torch.cuda.synchronize()
    eager_us = e0.elapsed_time(e1) / steps * 1e3
    # the same launches replayed from a CUDA graph: the product's own latency without the host's per-call
    # Python work; 96 different experts a graph (260 MB, more than L2), so every replay reads them from HBM
    per_graph = 96
    seq = [idxs[(37 * i) % experts] for i in range(per_graph)]
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for idx in seq:
            lin(x, idx)
    torch.cuda.current_stream(device).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for idx in seq:
            lin(x, idx)
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    reps = max(1, steps // per_graph)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    gpu_us = e0.elapsed_time(e1) / (reps * per_graph) * 1e3
    del graph
    mbytes = rows * B.row_bytes(KIND, cols)
    # the CPU: one expert's blocks decoded and multiplied, then the product alone
    blocks = b[: rows * cols // per].cpu().numpy().reshape(-1)
    xc = x.reshape(-1).float().cpu().numpy()
    Q.dequantize(blocks, KIND, (rows, cols))
    t0 = time.perf_counter()
    for _ in range(cpu_steps):
        w = Q.dequantize(blocks, KIND, (rows, cols))
        w @ xc
    cpu_s = (time.perf_counter() - t0) / cpu_steps
    from threadpoolctl import threadpool_limits

    with threadpool_limits(os.cpu_count() or 1):
        w @ xc
        t0 = time.perf_counter()
        for _ in range(50):
            w @ xc
        prod_s = (time.perf_counter() - t0) / 50
    return {"workload": "config 1: one expert's matvec, W [1536 x 4096] IQ3_S blocks, x float16 [4096]",
            "gpu_us_per_matvec": gpu_us, "gpu_gbs": mbytes / (gpu_us * 1e-6) / 1e9,
            "gpu_note": "one launch per matvec (its latency included), a different expert of a 692 MB stack each, "
                        "replayed from a CUDA graph of 96 such launches",
            "gpu_us_per_matvec_eager": eager_us,
            "eager_note": "the same calls one at a time from Python (BlockSwitchLinear.__call__), host work included",
            "cpu_ms_decode_and_product": cpu_s * 1e3, "cpu_ms_product_only": prod_s * 1e3,
            "cpu_threads": os.cpu_count(), "bytes_per_matvec": mbytes}


VERIFY_TYPES = ("Q8_0", "Q4_K", "Q5_K", "Q6_K", "Q2_K", "Q3_K", "IQ3_S", "IQ3_XXS", "IQ4_XS")
# the float16 scale fields of each type's block (byte offsets), overwritten with |N(0, SIGMA)|
SCALE_AT = {"Q8_0": (0,), "Q4_K": (0, 2), "Q5_K": (0, 2), "Q6_K": (208,), "Q2_K": (80, 82), "Q3_K": (108,),
            "IQ3_S": (0,), "IQ3_XXS": (0,), "IQ4_XS": (0,), "Q2_0": (0,)}


def run_verify(device, seed, steps=50, warmup=5, n_layers=8, tokens=5):
    """Configuration 4 of the benchmark, a speculative verify pass: 5 tokens (1 accepted + 4 drafted) through 8
    MoE layers of 256 experts, top-8, whose routed tensors cycle through the nine block types (layer l's
    gate/up/down have VERIFY_TYPES[(3 l + j) % 9]), each with the Q8_0 shared expert of ffn 4096. Every layer is
    one CUDA graph (`GraphedBlock`); a step replays the 8 in order. Every layer takes the same window (the
    layers are random, so a chained window would overflow float16 and route by inf): the routing stays that
    of N(0,1) tokens. The layers hold 22 GB, so a step reads its experts from HBM. `bytes` counts each layer's
    distinct chosen experts' three stacks, the shared expert and the router, once per step."""
    import torch

    from strata_mlx_b200 import blocks as B
    from strata_mlx_b200 import fused as Fz

    g = torch.Generator(device=device)
    g.manual_seed(seed)

    def random_blocks(kind, n_weights):
        per, nbytes = B.BLOCK[kind]
        n = n_weights // per
        b = torch.randint(0, 256, (n, nbytes), dtype=torch.uint8, device=device, generator=g)
        for at in SCALE_AT[kind]:
            b[:, at : at + 2] = (torch.randn(n, device=device, generator=g) * SIGMA).abs().half().view(torch.uint8).view(n, 2)
        return b.reshape(-1)

    x = torch.randn(tokens, H, device=device, generator=g).half()
    graphs, total_bytes = [], 0
    for layer in range(n_layers):
        kinds = [VERIFY_TYPES[(3 * layer + j) % 9] for j in range(3)]
        gate = B.BlockSwitchLinear(random_blocks(kinds[0], E * F_ * H), kinds[0], (E, F_, H))
        up = B.BlockSwitchLinear(random_blocks(kinds[1], E * F_ * H), kinds[1], (E, F_, H))
        down = B.BlockSwitchLinear(random_blocks(kinds[2], E * H * F_), kinds[2], (E, H, F_))
        shared = B.BlockMLP(B.BlockLinear(random_blocks(SHARED_KIND, FS * H), SHARED_KIND, (FS, H)),
                            B.BlockLinear(random_blocks(SHARED_KIND, FS * H), SHARED_KIND, (FS, H)),
                            B.BlockLinear(random_blocks(SHARED_KIND, H * FS), SHARED_KIND, (H, FS)))
        router = (torch.randn(E, H, device=device, generator=g) * 0.02).half()
        sgate = (torch.randn(1, H, device=device, generator=g) * 0.02).half()
        block = Fz.SparseMoeBlock(router, B.BlockSwitchGLU(gate, up, down), shared, sgate, K)
        hit = int(torch.unique(Fz.top_k(block.gate(x), K).view(torch.int32)).numel())
        per_expert = F_ * B.row_bytes(kinds[0], H) + F_ * B.row_bytes(kinds[1], H) + H * B.row_bytes(kinds[2], F_)
        total_bytes += hit * per_expert + 3 * FS * B.row_bytes(SHARED_KIND, H) + (E + 1) * H * 2
        graphs.append(Fz.GraphedBlock(block, tokens, H, torch.float16, device))
    for _ in range(warmup):
        for gb in graphs:
            gb(x)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        for gb in graphs:
            gb(x)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    peak = 6462.0
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        peak = json.load(open(path)).get("hbm_gbs", peak)
    gbs = total_bytes / (ms * 1e-3) / 1e9
    return {"workload": f"config 4: verify pass of {tokens} tokens through {n_layers} MoE layers cycling the nine "
                        "block types, 256 experts top-8, shared expert ffn 4096 Q8_0, one CUDA graph per layer",
            "ms_per_pass": ms, "tokens_per_s": tokens / (ms * 1e-3),
            "token_layers_per_s": tokens * n_layers / (ms * 1e-3), "bytes_per_pass": total_bytes,
            "achieved_gbs": gbs, "hbm_peak_gbs": peak, "frac": gbs / peak}


def run_stack(args, rank, world, local_rank, prompt=32768, chunk=2048, decode_steps=20):
    """Configuration 5 of the benchmark: the expert-parallel stack. `--stack-layers` (26) MoE layers of 256 IQ3_S
    experts (2.08 GB of routed blocks a layer), experts sharded E / world per rank, the Q8_0 shared expert of ffn
    4096, router N(0, 0.02); a prompt of 32,768 tokens in chunks of 2,048 (each rank takes its share of every
    chunk: `ExpertParallelPrompt`, all-to-all dispatch and return; one GPU: `SparseMoeBlock`), then decoding at
    batch 1 and 8 (each layer one CUDA graph; several GPUs: `ExpertParallelMoE`, one all-reduce a layer).
    Every layer takes the same chunk / tokens (random layers chained would overflow float16). Times are CUDA
    events, the maximum over ranks. Prefill tokens/s counts the prompt's tokens (all ranks); decode tokens/s
    counts the batch's tokens through the whole stack."""
    import torch

    from strata_mlx_b200 import blocks as B
    from strata_mlx_b200 import fused as Fz
    from strata_mlx_b200 import parallel as P

    device = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist  # noqa: F811
    # a rank's experts are its own draws (random either way); the shared expert, the router and the shared gate
    # are the same draws on every rank
    g = torch.Generator(device=device)
    g.manual_seed(args.seed + 4099 + 7919 * rank)
    g_same = torch.Generator(device=device)
    g_same.manual_seed(args.seed + 4099)
    e_loc = E // world

    def random_blocks(kind, n_weights, gen=g):
        per, nbytes = B.BLOCK[kind]
        n = n_weights // per
        b = torch.randint(0, 256, (n, nbytes), dtype=torch.uint8, device=device, generator=gen)
        b[:, 0:2] = (torch.randn(n, device=device, generator=gen) * SIGMA).abs().half().view(torch.uint8).view(n, 2)
        return b.reshape(-1)

    exchange = P.PeerExchange(rank, world, H, max_tokens=64, device=device) if world > 1 else None
    prompt_blocks, decode_blocks = [], []
    for _ in range(args.stack_layers):
        sw = B.BlockSwitchGLU(B.BlockSwitchLinear(random_blocks(KIND, e_loc * F_ * H), KIND, (e_loc, F_, H)),
                              B.BlockSwitchLinear(random_blocks(KIND, e_loc * F_ * H), KIND, (e_loc, F_, H)),
                              B.BlockSwitchLinear(random_blocks(KIND, e_loc * H * F_), KIND, (e_loc, H, F_)))
        shared = [(random_blocks(SHARED_KIND, FS * H, g_same), SHARED_KIND, (FS, H)),
                  (random_blocks(SHARED_KIND, FS * H, g_same), SHARED_KIND, (FS, H)),
                  (random_blocks(SHARED_KIND, H * FS, g_same), SHARED_KIND, (H, FS))]
        router = (torch.randn(E, H, device=device, generator=g_same) * 0.02).half()
        sgate = (torch.randn(1, H, device=device, generator=g_same) * 0.02).half()
        whole = B.BlockMLP(*(B.BlockLinear(b, k, s) for b, k, s in shared))
        prompt_layer = Fz.SparseMoeBlock(router, sw, whole, sgate, K)
        if world == 1:
            prompt_blocks.append(prompt_layer)
            decode_blocks.append(prompt_layer)
            continue
        lo, n = P.expert_range(rank, world, FS)
        (gb, gk, gs), (ub, uk, us), (db, dk, ds) = shared
        sliced = B.BlockMLP(B.BlockLinear(P.slice_rows(gb, gk, gs, lo, lo + n), gk, (n, H)),
                            B.BlockLinear(P.slice_rows(ub, uk, us, lo, lo + n), uk, (n, H)),
                            B.BlockLinear(P.slice_cols(db, dk, ds, lo, lo + n), dk, (H, n)))
        prompt_blocks.append(P.ExpertParallelPrompt(prompt_layer, rank, world, E))
        decode_blocks.append(P.ExpertParallelMoE(Fz.SparseMoeBlock(router, sw, sliced, sgate, K), rank, world, E,
                                                 exchange=exchange))

    gx = torch.Generator(device=device)
    gx.manual_seed(args.seed + 5)
    chunk_x = torch.randn(chunk, H, device=device, generator=gx).half()
    mine = chunk_x[rank * chunk // world : (rank + 1) * chunk // world].contiguous()

    def world_max(v):
        t = torch.tensor([v], device=device)
        if dist:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # prefill: every chunk through every layer
    for blk in prompt_blocks[:2]:
        blk(mine)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(prompt // chunk):
        for blk in prompt_blocks:
            blk(mine)
    e1.record()
    torch.cuda.synchronize()
    prefill_ms = world_max(e0.elapsed_time(e1))
    received = None
    if world > 1:  # each rank's pair count of the last chunk, per layer
        mine_r = torch.tensor([blk.received for blk in prompt_blocks], device=device)
        every = [torch.zeros_like(mine_r) for _ in range(world)]
        dist.all_gather(every, mine_r)
        received = [t.tolist() for t in every]

    out = {"workload": f"config 5: {args.stack_layers} MoE layers x 256 IQ3_S experts sharded over {world} GPU(s), "
                       f"shared expert ffn 4096 Q8_0; prefill {prompt} tokens in chunks of {chunk}, then decode at "
                       "batch 1 and 8, one CUDA graph a layer",
           "prefill_ms": prefill_ms, "prefill_tokens_per_s": prompt / (prefill_ms * 1e-3)}
    if received is not None:
        out["prefill_pairs_per_rank_last_chunk_layer0"] = [r[0] for r in received]
        out["prefill_pairs_per_rank_max_over_layers"] = [max(r) for r in received]
    for batch in (1, 8):
        xb = torch.randn(batch, H, device=device, generator=gx).half()
        if dist:
            dist.broadcast(xb, 0)
        graphs = [Fz.GraphedBlock(blk, batch, H, torch.float16, device) for blk in decode_blocks]
        for gb in graphs:
            gb.x.copy_(xb)
        for gb in graphs:
            gb.graph.replay()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        e0.record()
        for _ in range(decode_steps):
            for gb in graphs:
                gb.graph.replay()
        e1.record()
        torch.cuda.synchronize()
        ms = world_max(e0.elapsed_time(e1) / decode_steps)
        out[f"decode_bs{batch}_ms_per_token_step"] = ms
        out[f"decode_bs{batch}_tokens_per_s"] = batch / (ms * 1e-3)
        del graphs
        torch.cuda.synchronize()
    if exchange is not None:
        if exchange.failed():
            out["error"] = "a wait of the peer exchange gave up"
        dist.barrier()
        exchange.close()
    return out


def run_matvec(kind, seed, steps=3, warmup=3, experts=64, tokens=5):
    """One product of config 4's shape on the decode matvec the type takes: `tokens` x top-8 pairs through a
    stack of `experts` (4096 x 1536) of `kind`, 283 MB for Q5_K (more than L2), small enough for a profiler's
    replays."""
    import torch

    from strata_mlx_b200 import blocks as B

    device = torch.device("cuda", 0)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    per, nbytes = B.BLOCK[kind]
    n = experts * H * F_ // per
    b = torch.randint(0, 256, (n, nbytes), dtype=torch.uint8, device=device, generator=g)
    for at in SCALE_AT[kind]:
        b[:, at : at + 2] = (torch.randn(n, device=device, generator=g) * SIGMA).abs().half().view(torch.uint8).view(n, 2)
    lin = B.BlockSwitchLinear(b.reshape(-1), kind, (experts, H, F_))
    x = torch.randn(tokens, 1, 1, F_, device=device, generator=g).half()  # one row shared by a token's 8 pairs
    idx = torch.randperm(experts, device=device, generator=g)[: tokens * K].to(torch.int32).reshape(tokens, K)
    for _ in range(warmup):
        lin(x, idx)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        lin(x, idx)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) / steps * 1e3
    nbytes_read = tokens * K * H * B.row_bytes(kind, F_)
    return {"kind": kind, "pairs": tokens * K, "us": us, "gbs": nbytes_read / (us * 1e-6) / 1e9}


def _prefill_ep(block, x, steps, warmup, rank, world):
    """Configuration 3 over `world` ranks: rank r's experts and tokens [r T / world, (r+1) T / world)."""
    import torch
    import torch.distributed as dist

    from strata_mlx_b200 import parallel as P

    T = x.shape[0]
    sw = block.switch_mlp
    stacks = [(lin.blocks, lin.kind, lin.shape) for lin in (sw.gate_proj, sw.up_proj, sw.down_proj)]
    sh = block.shared_expert
    shared = [(lin.blocks, lin.kind, (lin.output_dims, lin.input_dims)) for lin in (sh.gate_proj, sh.up_proj, sh.down_proj)]
    part = P.shard_layer(block.gate.weight, *stacks, shared, block.shared_expert_gate.weight, K, rank, world,
                         whole_shared=True)
    ep = P.ExpertParallelPrompt(part, rank, world, E)
    xr = x[rank * T // world : (rank + 1) * T // world].contiguous()
    for _ in range(warmup):
        ep(xr)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        ep(xr)
    e1.record()
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1) / steps], device=x.device)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    received = torch.tensor([ep.received], device=x.device)
    per_rank = [torch.zeros_like(received) for _ in range(world)]
    dist.all_gather(per_rank, received)
    layer_ms = float(ms.item())
    return {"workload": f"config 3 over {world} GPUs: one MoE layer, prefill chunk of 1180 tokens split over the "
                        "ranks, 256 Q2_K experts sharded E/N, top-8, Zipf s=1.1 routing, the shared expert ffn 4096 "
                        "Q8_0 on every rank; all-to-all dispatch and return over NCCL",
            "layer_ms": layer_ms, "tokens_per_s": T / (layer_ms * 1e-3),
            "pairs_per_rank": [int(t.item()) for t in per_rank]}


class Clocks:
    """SM clocks and throttle reasons sampled with NVML every few milliseconds from a thread while the timed
    region runs (reading counters only; nothing about the GPU is changed)."""

    NAMES = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4}

    def __init__(self, index):
        import threading

        self.samples, self.stop_flag = [], threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            dev = int(os.environ.get("CUDA_VISIBLE_DEVICES", str(index)).split(",")[index]) \
                if "CUDA_VISIBLE_DEVICES" in os.environ else index
            self.h = pynvml.nvmlDeviceGetHandleByIndex(dev)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - no NVML: report no clock record
            self.nv = None
            return
        self.t = threading.Thread(target=self._run, daemon=True)
        self.t.start()

    def _run(self):
        while not self.stop_flag.is_set():
            try:
                mhz = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                reasons = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((mhz, reasons))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.005)

    def stop(self):
        if self.nv is None:
            return None
        self.stop_flag.set()
        self.t.join(timeout=5)
        if not self.samples:
            return None
        reasons = sorted(name for name, bit in self.NAMES.items() if any(r & bit for _, r in self.samples))
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": float(self.max_mhz),
                "reasons": reasons, "samples": len(self.samples), "source": "NVML, 5 ms"}


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return d["hbm_gbs"], "measured"
    return 6650.0, "fallback"


def traffic_from_profiles():
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary, if there is one."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        try:
            return json.load(open(path)).get("decode_gate_up_bytes_per_launch")
        except (OSError, ValueError):
            return None
    return None


def run_ours(args, rank, world, local_rank):
    import torch

    from strata_mlx_b200 import blocks as B

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dist = None
    if world > 1:
        import torch.distributed as dist  # noqa: F811

    # every rank draws the same layers and keeps its part of each (world > 1)
    layers = make_layers(args.layers, args.seed, device, rank, world)
    gx = torch.Generator(device=device)
    gx.manual_seed(args.seed + 1)
    xs = [torch.randn(1, H, device=device, generator=gx).half() for _ in range(args.layers)]
    exchange, parity = None, None
    if world > 1:
        from strata_mlx_b200.parallel import ExpertParallelMoE, PeerExchange

        exchange = PeerExchange(rank, world, H, max_tokens=64, device=device)
        blocks = [ExpertParallelMoE(layer, rank, world, E, exchange=exchange) for layer in layers]
        parity = parity_ep(device, args.seed + 17, rank, world, exchange)
    else:
        blocks = layers
    stream = torch.cuda.current_stream()
    from strata_mlx_b200 import _lib
    from strata_mlx_b200 import fused as Fz
    from strata_mlx_b200.fused import GraphedBlock, route, top_k_softmax

    # one CUDA graph per layer: a decode engine's step, with the token already in its static input
    graphs = []
    for i in range(args.layers):
        gb = GraphedBlock(blocks[i], 1, H, torch.float16, device)
        gb.x.copy_(xs[i])
        graphs.append(gb)
    n0 = _lib.launches
    blocks[0](xs[0])
    launches = _lib.launches - n0  # our kernels in one step

    def align():
        """Line the ranks' timed regions up on the device: a barrier on the host, then a small all-reduce on the
        timing stream whose end every rank reaches together."""
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
            torch.cuda.synchronize()
            dist.all_reduce(torch.ones(1, device=device))

    for i in range(args.warmup):
        graphs[i % args.layers].graph.replay()
    clocks = Clocks(local_rank)
    align()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        graphs[i % args.layers].graph.replay()
    t_end.record(stream)
    torch.cuda.synchronize()
    ms = t_start.elapsed_time(t_end)
    clk = clocks.stop()
    if exchange is not None and exchange.failed():
        raise RuntimeError("a wait of the peer exchange gave up during the timed steps")

    # the dominant kernel alone: a graph of its launches over the rotating layers, with each layer's routing: the
    # step's batched gate / up launch (the routed experts' of this rank and the shared expert's products in one
    # int8 tensor-core kernel; with FUSED_ROUTE the route with this rank's view of it in the same launch)
    fuse = Fz.FUSED_ROUTE
    routes, gu_bytes = [], 0
    for i in range(args.layers):
        blk = blocks[i]
        layer = blk if world == 1 else blk.layer
        idx, _ = top_k_softmax(layer.gate(xs[i]), K)
        if world > 1:
            idx = blk.local_indices(idx)
        fi = idx.reshape(-1).contiguous()
        sw, sh = layer.switch_mlp, layer.shared_expert
        valid = int((fi.view(torch.int32) < sw.gate_proj.num_experts).sum().item())
        gu_bytes += (2 * valid * F_ * B.row_bytes(KIND, H)
                     + 2 * sh.gate_proj.output_dims * B.row_bytes(SHARED_KIND, H) + ((E + 1) * H * 2 if fuse else 0))
        if fuse:
            r = route(layer.gate, layer.shared_expert_gate, xs[i], K, defer=True,
                      local=(blk.lo, blk.count) if world > 1 else None)
            step_r, ri = r[-1], (r[3] if world > 1 else r[0]).reshape(-1)
        else:
            step_r, ri = None, fi
        outs = [torch.empty((K, F_), dtype=torch.float16, device=device) for _ in range(2)]
        souts = [torch.empty((1, sh.gate_proj.output_dims), dtype=torch.float16, device=device) for _ in range(2)]
        z = B._zeros_idx(1, device)
        probs = [B._problem(sw.gate_proj, ri, K, K, outs[0], x=xs[i]), B._problem(sw.up_proj, ri, K, K, outs[1], x=xs[i]),
                 B._problem(sh.gate_proj.stack, z, 1, 1, souts[0], x=xs[i]),
                 B._problem(sh.up_proj.stack, z, 1, 1, souts[1], x=xs[i])]
        routes.append((probs, outs + souts, step_r))
    gu_bytes /= args.layers  # per launch, averaged over the layers' routings
    reps = max(1, 64 // args.layers)
    for probs, _, step_r in routes:
        B.matvec_batch(probs, route=step_r)
    torch.cuda.synchronize()
    gu_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gu_graph):
        for _ in range(reps):
            for probs, _, step_r in routes:
                B.matvec_batch(probs, route=step_r)
    gu_graph.replay()
    torch.cuda.synchronize()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record(stream)
    n_rep = max(1, args.steps // (reps * args.layers))
    for _ in range(n_rep):
        gu_graph.replay()
    g1.record(stream)
    torch.cuda.synchronize()
    gu = g0.elapsed_time(g1) / (n_rep * reps * args.layers)

    # end to end through the public API (GraphedBlock.__call__ with host_io): each step copies its token from
    # pinned host memory to the device and its result back to pinned host memory, both inside the step's graph
    del graphs
    host_graphs = [GraphedBlock(blocks[i], 1, H, torch.float16, device, host_io=True) for i in range(args.layers)]
    host_in = [x.cpu().pin_memory() for x in xs]
    for i in range(args.warmup):
        host_graphs[i % args.layers](host_in[i % args.layers])
    align()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        host_graphs[i % args.layers](host_in[i % args.layers])
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    del host_graphs, gu_graph
    if exchange is not None and exchange.failed():
        raise RuntimeError("a wait of the peer exchange gave up during the end-to-end steps")

    def world_max(v):
        if not dist:
            return v
        t = torch.tensor([v], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    ms, e2e_ms, gu, gu_bytes = world_max(ms), world_max(e2e_ms), world_max(gu), world_max(gu_bytes)
    if parity is not None:
        parity = world_max(parity)
    if exchange is not None:
        torch.cuda.synchronize()
        dist.barrier()
        exchange.close()
    if rank != 0:
        return None
    peak, peak_kind = peaks()
    achieved = gu_bytes / (gu * 1e-3) / 1e9
    # bytes a rank reads per step: its share of the routed experts (8 of 256 spread evenly), its slice of the
    # shared expert, the whole router
    per_step_bytes = (3 * K * F_ * B.row_bytes(KIND, H) + 3 * FS * B.row_bytes(SHARED_KIND, H)) / world + (E + 1) * H * 2
    step_gbs = per_step_bytes / (ms / args.steps * 1e-3) / 1e9
    line = {
        "metric": "MoE layer tokens/s (decode bs1) + achieved HBM GB/s vs roofline",
        "value": args.steps / (ms * 1e-3),
        "unit": "token-layers/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f16 activations, IQ3_S/Q8_0 blocks, f32 accumulation",
        "data": "synthetic (seeded random blocks and activations, BASELINE config 2 distributions)",
        "config": dict(CONFIG2),
        "setup": {"layers_rotated": args.layers, "l2": f"inputs > L2: {args.layers} layers x "
                  f"{(3 * E * F_ * B.row_bytes(KIND, H) + 3 * FS * B.row_bytes(SHARED_KIND, H)) / 1e9:.2f} GB cycled",
                  "parallelism": f"ep{world}: experts {E // world} a rank, shared ffn {FS // world} a rank, one "
                                 "exchange of partial sums over NVLink peer memory a step" if world > 1 else "single",
                  "bytes_per_rank_per_step": per_step_bytes},
        "hbm_gbs_step": step_gbs,
        "step_roofline": {"bound": "hbm", "achieved": step_gbs, "peak": peak, "unit": "GB/s", "frac": step_gbs / peak,
                          "bytes": "per rank per step: its share of the routed and shared bytes, the router"},
        "gpu_launches": launches * args.steps,
        "e2e": {"value": args.steps / (e2e_ms * 1e-3), "unit": "token-layers/s",
                "h2d_bytes_per_step": H * 2, "d2h_bytes_per_step": H * 2},
        "roofline": {"kernel": ("mv8_kernel (the route with the batched gate+up: the router's 257 x 4096 float16 rows, "
                                "this rank's IQ3_S 1536 x 4096 pairs, the Q8_0 shared expert's gate and up rows)") if fuse
                     else ("mv8_kernel (batched gate+up: this rank's IQ3_S 1536 x 4096 pairs + the Q8_0 shared "
                           "expert's gate and up rows)"),
                     "bound": "hbm",
                     "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_source": peak_kind,
                     "algorithmic_bytes_per_launch": gu_bytes, "launch_ms": gu,
                     "traffic": traffic_from_profiles() if world == 1 else None},
        "clocks": clk,
    }
    if parity is not None:
        line["parity_rel_l2"] = parity
        line["parity"] = ("max over ranks of rel-L2(expert-parallel block, the same layer whole on one GPU), one "
                          "token, super-scales |N(0, 0.001)|")
    return line


CONFIG2 = {"workload": "config 2: one MoE layer, decode batch 1, hidden 4096, 256 IQ3_S experts (gate/up 1536x4096, "
                       "down 4096x1536), top-8, shared expert ffn 4096 Q8_0"}


def main():
    args = _args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank != 0:
            return
        # the reference's CPU path: each step a whole decode step (about a second on 16 cores); at most 40 steps
        steps, warmup = min(args.steps, 40), min(args.warmup, 3)
        cb = cpu_baseline(steps, args.seed, warmup=warmup)
        line = {"impl": "reference", "metric": "MoE layer tokens/s (decode bs1) + achieved HBM GB/s vs roofline",
                "value": cb["value"], "unit": cb["unit"], "n_gpus": world, "steps": steps, "warmup": warmup,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "f32 (numpy; blocks decoded by the oracle port of the reference's decoders)",
                "data": "synthetic (seeded random blocks and activations, BASELINE config 2 distributions)",
                "config": dict(CONFIG2),
                "setup": {"cpu": f"oracle port of the reference's block decoders + numpy products, {cb['cores']} "
                                 "processes"},
                "cpu_baseline": cb, "e2e": {"value": cb["value"], "unit": cb["unit"], "h2d_bytes_per_step": 0,
                                            "d2h_bytes_per_step": 0}}
        if steps != args.steps:
            line["sample"] = f"{steps} of the {args.steps} steps asked for (each a whole decode step on the CPU)"
        print(json.dumps(line))
        return
    if args.only_matvec:
        print(json.dumps({"matvec": run_matvec(args.only_matvec, args.seed + 299, steps=args.steps,
                                               warmup=args.warmup)}))
        return
    if args.only_stack and world == 1:
        print(json.dumps({"stack": run_stack(args, 0, 1, local_rank)}))
        return
    if args.only_verify:
        import torch

        print(json.dumps({"verify": run_verify(torch.device("cuda", local_rank), args.seed + 199)}))
        return
    if args.only_prefill:
        import torch

        print(json.dumps({"prefill": run_prefill(torch.device("cuda", local_rank), args.seed + 99, steps=args.steps,
                                                 warmup=args.warmup)}))
        return
    cb = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cb = cpu_baseline(args.cpu_steps, args.seed)  # before any CUDA work: the pool is spawned
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        line = run_ours(args, rank, world, local_rank)
        # several GPUs: configurations 3 and 5 over the ranks too (every rank takes the same steps, so an error
        # is raised on every rank and ends the job)
        if world > 1 and not args.no_prefill:
            import torch

            pf = run_prefill(torch.device("cuda", local_rank), args.seed + 99, rank=rank, world=world)
            if line is not None:
                line["prefill"] = pf
        if world > 1 and not args.no_stack:
            st = run_stack(args, rank, world, local_rank)
            if line is not None:
                line["stack"] = st
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
            dist.destroy_process_group()
    if line is not None:
        line["cpu_baseline"] = cb
        if world == 1 and not args.no_prefill:
            import torch

            pf = run_prefill(torch.device("cuda", local_rank), args.seed + 99)
            peak_tf = 1672.6
            path = os.path.join(ROOT, "MEASURED_PEAKS.json")
            if os.path.exists(path):
                peak_tf = json.load(open(path)).get("bf16_tflops", peak_tf)
            pf["roofline"] = {"kernel": "gemm_tc_kernel<Q2_K> (the three routed tile products: gate + up in one "
                                        "launch, down)", "bound": "tensor",
                              "achieved": pf["routed_gemm_tflops"], "peak": peak_tf, "unit": "TFLOP/s",
                              "frac": pf["routed_gemm_tflops"] / peak_tf}
            line["prefill"] = pf
        # the headline line is printed whatever becomes of the extra measurements below (one process, one GPU:
        # an error there leaves no rank waiting)
        if world == 1 and not args.no_verify:
            import torch

            try:
                line["config1"] = run_config1(torch.device("cuda", local_rank), args.seed + 149)
            except Exception as exc:  # noqa: BLE001
                line["config1"] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
            try:
                line["verify"] = run_verify(torch.device("cuda", local_rank), args.seed + 199)
            except Exception as exc:  # noqa: BLE001
                line["verify"] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
        if world == 1 and not args.no_stack:
            import torch

            try:
                torch.cuda.empty_cache()
                line["stack"] = run_stack(args, rank, world, local_rank)
            except Exception as exc:  # noqa: BLE001
                line["stack"] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
        print(json.dumps(line))


if __name__ == "__main__":
    main()
