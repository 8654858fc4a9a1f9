// Grouped GEMM of a prompt's expert-sorted tiles on GGUF blocks: `tile_matmul` (strata_mlx/blocks.py:583-654)
// on the 5th-generation tensor cores.
//
// out[p, r] = W[expert of p's tile][r, :] . a[p, :] with the weights rounded to float16 (a's type) and float32
// sums. The tensor-core product is taken "swap AB": 128 weight rows are the M side of a tcgen05 MMA and a
// run of up to 8 tiles (128 tokens) of one expert is the N side, so a weight row is decoded once for every
// token of that expert in the run.
//
// Per CTA (persistent over jobs = (run of tiles, block of 128 rows)):
//   warps 0-7  loaders + decoders: cp.async the raw block bytes of a 256-column stage of the 128 rows and the
//              run's activations (canonical K-major core-matrix layout, no swizzle) into a double buffer; then
//              each thread decodes 128 weights of one row (its TMEM lane) and stores them as float16 pairs
//              into a TMEM A slot (3 slots); after the last stage they read the float32 accumulators back
//              (tcgen05.ld) and write out.
//   warp 8     one thread issues tcgen05.mma kind::f16 with A from TMEM and B from shared memory, 16 MMAs of
//              K = 16 per stage, and tcgen05.commit releases the A slot, the activation buffer and, after a
//              job's last stage, the accumulator.
// Every wait is bounded; a CTA whose wait gives up records SMOE_ETIMEOUT in the workspace status word and
// leaves its remaining jobs.
#include "blocks.cuh"
#include "tc05.cuh"

namespace smoe {

constexpr int kGmDecoders = 8;                 // decoder warps
constexpr int kGmThreads = 32 * (kGmDecoders + 1);
constexpr int kGmM = 128;                      // weight rows per job
constexpr int kGmKStage = 256;                 // columns per pipeline stage
constexpr int kGmMaxTiles = 8;                 // tiles of 16 tokens per job -> N <= 128
constexpr int kGmMaxN = 16 * kGmMaxTiles;
constexpr int kGmASlots = 3;
constexpr uint32_t kGmTmemCols = 512;          // D: [0,128), A slots: 128 + 128 i
constexpr uint32_t kWaitLimit = 1u << 22;      // polls of try_wait before a wait gives up

struct GemmPlanHeader {
    int32_t count;   // jobs' tile runs
    int32_t status;  // 0, or SMOE_ETIMEOUT if a wait gave up
    int32_t pad[14];
};
struct TileRun {
    int32_t first_tile, tiles, expert, pad;
};

// ---- plan: maximal runs of equal tile_expert split into runs of at most kGmMaxTiles tiles

__device__ __forceinline__ int block_scan_max(int v, int* warp_buf) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v = max(v, u);
    }
    if (lane == 31) warp_buf[w] = v;
    __syncthreads();
    if (w == 0) {
        int t = warp_buf[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t = max(t, u);
        }
        warp_buf[lane] = t;
    }
    __syncthreads();
    const int r = w > 0 ? max(v, warp_buf[w - 1]) : v;
    __syncthreads();
    return r;
}

__device__ __forceinline__ int block_scan_sum(int v, int* warp_buf, int& total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += u;
    }
    if (lane == 31) warp_buf[w] = x;
    __syncthreads();
    if (w == 0) {
        int t = warp_buf[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += u;
        }
        warp_buf[lane] = t;
    }
    __syncthreads();
    const int incl = x + (w > 0 ? warp_buf[w - 1] : 0);
    total = warp_buf[31];
    __syncthreads();
    return incl - v;  // exclusive
}

__global__ void __launch_bounds__(1024) gemm_plan_kernel(const uint32_t* __restrict__ tile_expert, int64_t ntiles,
                                                        int64_t experts, GemmPlanHeader* __restrict__ hdr,
                                                        TileRun* __restrict__ runs) {
    __shared__ int warp_buf[32];
    int carry_start = -1, carry_count = 0;
    for (int64_t c0 = 0; c0 < ntiles; c0 += 1024) {
        const int64_t t = c0 + threadIdx.x;
        const bool in = t < ntiles;
        const uint32_t e = in ? tile_expert[t] : 0xffffffffu;
        const uint32_t prev = (in && t > 0) ? tile_expert[t - 1] : 0xfffffffeu;
        const bool start = in && e != prev;
        int rs = block_scan_max(start ? static_cast<int>(t) : -1, warp_buf);
        rs = max(rs, carry_start);
        const bool lead = in && e < uint64_t(experts) && ((t - rs) % kGmMaxTiles) == 0;
        int total;
        const int pos = block_scan_sum(lead ? 1 : 0, warp_buf, total) + carry_count;
        if (lead) {
            int n = 1;
            while (n < kGmMaxTiles && t + n < ntiles && tile_expert[t + n] == e) ++n;
            runs[pos] = TileRun{static_cast<int32_t>(t), n, static_cast<int32_t>(e), 0};
        }
        // carry the last run start of this chunk into the next
        __shared__ int last_rs;
        if (threadIdx.x == 1023) last_rs = rs;
        __syncthreads();
        carry_start = last_rs;
        carry_count += total;
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        hdr->count = carry_count;
        hdr->status = 0;
    }
}

// ---- the tensor-core kernel

struct GemmArgs {
    const uint8_t* blocks;
    const uint8_t* end;
    const __half* a;
    float* out;
    const GemmPlanHeader* hdr;
    const TileRun* runs;
    int* status;
    int64_t rows, cols, row_bytes;
    int stage_bytes;  // raw bytes of one row's 256-column stage
    int rawb;         // smem stride of a row's raw stage (>= stage_bytes + 15, an odd multiple of 16)
    int mblocks;
};

struct GemmSmem {
    uint64_t afull[kGmASlots], afree[kGmASlots], bfree[2], dfull, dfree, drain;
    uint32_t tmem_base;
    int abort;
};

template <class B>
__global__ void __launch_bounds__(kGmThreads, 1) gemm_tc_kernel(const GemmArgs g) {
    extern __shared__ __align__(128) uint8_t smem[];
    GemmSmem& S = *reinterpret_cast<GemmSmem*>(smem);
    uint8_t* raw = smem + 128;                                            // 2 x 128 rows x rawb
    uint8_t* bbuf = raw + 2 * kGmM * g.rawb;                              // 2 x (kGmMaxN x 256) float16
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int njobs = g.hdr->count * g.mblocks;
    const int nk = static_cast<int>(g.cols / kGmKStage);

    if (threadIdx.x == 0) {
        for (int i = 0; i < kGmASlots; ++i) {
            tc::mbar_init(&S.afull[i], kGmDecoders);
            tc::mbar_init(&S.afree[i], 1);
        }
        tc::mbar_init(&S.bfree[0], 1);
        tc::mbar_init(&S.bfree[1], 1);
        tc::mbar_init(&S.dfull, 1);
        tc::mbar_init(&S.dfree, kGmDecoders);
        tc::mbar_init(&S.drain, 1);
        S.abort = 0;
        tc::fence_barrier_init();
    }
    if (warp == kGmDecoders) {
        tc::tmem_alloc(&S.tmem_base, kGmTmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = S.tmem_base;

    if (warp == kGmDecoders) {
        // ---------------- MMA issuer (lane 0 issues; the warp waits together and agrees on every outcome)
        uint32_t gstage = 0, jobs = 0;
        bool ok = true;
        for (int job = blockIdx.x; job < njobs && ok; job += gridDim.x, ++jobs) {
            const TileRun run = g.runs[job / g.mblocks];
            const int n = 16 * run.tiles;
            const uint32_t idesc = tc::idesc_f16_f32(kGmM, n);
            const uint32_t lbo = static_cast<uint32_t>(n) * 16u;
            if (jobs > 0) ok = __all_sync(0xffffffffu, tc::mbar_wait(&S.dfree, (jobs - 1) & 1, kWaitLimit));
            if (!ok) break;
            tc::fence_after_sync();
            for (int s = 0; s < nk; ++s, ++gstage) {
                const uint32_t as = gstage % kGmASlots, bs = gstage & 1;
                ok = __all_sync(0xffffffffu, tc::mbar_wait(&S.afull[as], (gstage / kGmASlots) & 1, kWaitLimit));
                if (!ok) break;
                tc::fence_after_sync();
                if (lane == 0) {
                    const uint32_t bbase = static_cast<uint32_t>(__cvta_generic_to_shared(bbuf + bs * (kGmMaxN * 512)));
#pragma unroll 4
                    for (int j = 0; j < kGmKStage / 16; ++j) {
                        const uint64_t bd = tc::smem_desc(bbase + 2u * j * lbo, lbo, 128);
                        tc::mma_f16_ts(tmem, tmem + 128u + 128u * as + 8u * j, bd, idesc, (s > 0 || j > 0) ? 1u : 0u);
                    }
                    tc::mma_commit(&S.afree[as]);
                    tc::mma_commit(&S.bfree[bs]);
                    if (s == nk - 1) tc::mma_commit(&S.dfull);
                }
                __syncwarp();
            }
        }
        if (!ok && lane == 0) {
            S.abort = 1;
            atomicExch(g.status, SMOE_ETIMEOUT);
        }
    } else {
        // ---------------- loaders, decoders, epilogue (256 threads). Every wait's outcome is and-reduced over
        // the 256 threads by the named barrier that follows it, so they leave a job together or not at all.
        const int t = threadIdx.x;             // 0..255
        const int m = 32 * (warp & 3) + lane;  // TMEM lane = weight row within the block
        const int h = warp >> 2;               // which 128 columns of a stage this thread decodes
        uint32_t gstage = 0, jobs = 0;
        bool ok = true;
        for (int job = blockIdx.x; job < njobs && ok; job += gridDim.x, ++jobs) {
            const int ri = job / g.mblocks, mb = job % g.mblocks;
            const TileRun run = g.runs[ri];
            const int n = 16 * run.tiles;
            const int64_t row0 = int64_t(mb) * kGmM;
            const int mrows = static_cast<int>(min(int64_t(kGmM), g.rows - row0));
            const uint8_t* wbase = g.blocks + (int64_t(run.expert) * g.rows + row0) * g.row_bytes;
            const __half* abase = g.a + int64_t(run.first_tile) * 16 * g.cols;

            auto issue = [&](uint32_t gs, int s) {
                const int slot = gs & 1;
                uint8_t* rdst = raw + slot * (kGmM * g.rawb);
                // raw bytes: the 16-byte chunks covering each row's stage
                for (int r = t >> 3; r < mrows; r += 32) {
                    const uint8_t* src = wbase + r * g.row_bytes + int64_t(s) * g.stage_bytes;
                    stage_bytes(rdst + r * g.rawb, src, g.stage_bytes, g.end, t & 7, 8);
                }
                // activations: n rows x 256 columns -> chunk (row i, k-chunk c) at c * (n * 16) + i * 16
                uint8_t* bdst = bbuf + slot * (kGmMaxN * 512);
                for (int q = t; q < n * 32; q += 256) {
                    const int i = q >> 5, c = q & 31;
                    cp_async16(bdst + c * (n * 16) + i * 16, abase + int64_t(i) * g.cols + int64_t(s) * kGmKStage + 8 * c, 16);
                }
            };
            auto wait_bfree = [&](uint32_t gs) -> bool {
                return gs < 2 || tc::mbar_wait(&S.bfree[gs & 1], ((gs - 2) >> 1) & 1, kWaitLimit);
            };

            ok = tc::bar_and(1, 256, wait_bfree(gstage));
            if (!ok) break;
            issue(gstage, 0);
            cp_async_commit();
            for (int s = 0; s < nk; ++s, ++gstage) {
                // (this barrier also means everyone is done decoding the stage whose buffers are refilled next)
                const bool more = s + 1 < nk;
                ok = tc::bar_and(1, 256, more ? wait_bfree(gstage + 1) : true);
                if (!ok) break;
                if (more) issue(gstage + 1, s + 1);
                cp_async_commit();
                cp_async_wait<1>();
                tc::fence_proxy_async_smem();
                const uint32_t as = gstage % kGmASlots;
                ok = tc::bar_and(1, 256, gstage < kGmASlots ||
                                             tc::mbar_wait(&S.afree[as], ((gstage - kGmASlots) / kGmASlots) & 1, kWaitLimit));
                if (!ok) break;
                tc::fence_after_sync();
                // decode 4 runs (128 weights) of row m into TMEM lane m, columns 128 + 128 as + 64 h + 16 i
                const uint8_t* rsrc = raw + (gstage & 1) * (kGmM * g.rawb) + m * g.rawb;
                const int off = static_cast<int>((reinterpret_cast<uintptr_t>(wbase + int64_t(m) * g.row_bytes +
                                                                              int64_t(s) * g.stage_bytes)) & 15);
                const uint32_t tbase = tmem + (uint32_t(32 * (warp & 3)) << 16) + 128u + 128u * as + 64u * h;
#pragma unroll 1
                for (int i = 0; i < 4; ++i) {
                    uint32_t v[16];
                    if (m < mrows) {
                        float w[32];
                        B::run(rsrc + off, 4 * h + i, w);
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] = tc::pack_half2(w[2 * j], w[2 * j + 1]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] = 0u;
                    }
                    tc::tmem_st16(tbase + 16u * i, v);
                }
                tc::tmem_wait_st();
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&S.afull[as]);
            }
            if (!ok) break;
            // epilogue: accumulators of rows m, tokens [n/2 * h, n/2 * (h+1))
            ok = tc::bar_and(1, 256, tc::mbar_wait(&S.dfull, jobs & 1, kWaitLimit));
            if (!ok) break;
            tc::fence_after_sync();
            const int half_n = n >> 1;
            float* obase = g.out + int64_t(run.first_tile) * 16 * g.rows + row0 + m;
            for (int c0 = h * half_n; c0 < (h + 1) * half_n; c0 += 8) {
                uint32_t v[8];
                tc::tmem_ld8(tmem + (uint32_t(32 * (warp & 3)) << 16) + uint32_t(c0), v);
                tc::tmem_wait_ld();
                if (m < mrows) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) obase[int64_t(c0 + j) * g.rows] = __uint_as_float(v[j]);
                }
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&S.dfree);
        }
        cp_async_wait<0>();
        if (!ok && t == 0) {
            S.abort = 1;
            atomicExch(g.status, SMOE_ETIMEOUT);
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == kGmDecoders) {
        if (S.abort) {
            // let any MMA still in flight finish before the TMEM it writes is released (bounded wait)
            if (lane == 0) tc::mma_commit(&S.drain);
            __syncwarp();
            tc::mbar_wait(&S.drain, 0, kWaitLimit);
        }
        tc::tmem_dealloc(tmem, kGmTmemCols);
    }
}

// ---- CUDA-core path for what the tensor-core kernel does not take (float32 activations, stages that do not
// divide into 256 columns): a CTA per (tile, 64 rows), weights decoded per thread, float32 throughout.

template <class B, typename T>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const uint8_t* __restrict__ blocks, const T* __restrict__ a,
                                                        const uint32_t* __restrict__ tile_expert, int64_t experts,
                                                        int64_t rows, int64_t cols, int64_t row_bytes,
                                                        float* __restrict__ out) {
    constexpr int kChunk = 512;           // columns of a staged in shared memory at a time
    __shared__ __align__(16) float as[16 * kChunk];
    const int64_t tile = blockIdx.y;
    const uint32_t e = tile_expert[tile];
    if (e >= experts) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r = int64_t(blockIdx.x) * 8 + warp;  // a warp per weight row
    const uint8_t* row = blocks + (int64_t(e) * rows + (r < rows ? r : 0)) * row_bytes;
    float acc[16];
#pragma unroll
    for (int p = 0; p < 16; ++p) acc[p] = 0.0f;
    for (int64_t c0 = 0; c0 < cols; c0 += kChunk) {
        const int width = static_cast<int>(min(int64_t(kChunk), cols - c0));
        __syncthreads();
        for (int i = threadIdx.x; i < 16 * width; i += 256) {
            const int p = i / width, c = i % width;
            as[p * kChunk + c] = to_f32(a[(tile * 16 + p) * cols + c0 + c]);
        }
        __syncthreads();
        if (r < rows) {
            for (int n = lane; n < width / 32; n += 32) {
                float w[32];
                B::run(row, static_cast<int>(c0 / 32) + n, w);
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    // the weights are rounded to a's type before the product
                    const float wj = to_f32(from_f32<T>(w[j]));
#pragma unroll
                    for (int p = 0; p < 16; ++p) acc[p] = fmaf(wj, as[p * kChunk + 32 * n + j], acc[p]);
                }
            }
        }
    }
    if (r < rows) {
#pragma unroll
        for (int p = 0; p < 16; ++p) {
            const float s = warp_sum(acc[p]);
            if (lane == 0) out[(tile * 16 + p) * rows + r] = s;
        }
    }
}

}  // namespace smoe

using namespace smoe;

extern "C" int smoe_tileable(int kind, int64_t rows, int64_t cols) {
    int per, bytes;
    if (!block_info(kind, per, bytes)) return 0;
    return rows > 0 && cols > 0 && rows % 64 == 0 && cols % 64 == 0 && cols % per == 0;
}

extern "C" size_t smoe_tile_matmul_workspace_size(int64_t p16) {
    const int64_t ntiles = p16 / 16;
    return sizeof(GemmPlanHeader) + sizeof(TileRun) * static_cast<size_t>(ntiles > 0 ? ntiles : 1);
}

static int g_num_sms = 0;

extern "C" int smoe_tile_matmul(int kind, const uint8_t* blocks, int64_t experts, int64_t rows, int64_t cols,
                                const void* a, int a_dtype, int64_t p16, const uint32_t* tile_expert, float* out,
                                void* workspace, size_t workspace_bytes, void* stream) {
    if (p16 == 0) return SMOE_OK;
    int per, bytes;
    if (!block_info(kind, per, bytes)) return fail(SMOE_EKIND, "block type " + std::to_string(kind) + " has no decoder");
    SMOE_REQUIRE(smoe_tileable(kind, rows, cols), SMOE_ESHAPE, "stack not tileable: rows and cols must divide by 64 and cols by the block");
    SMOE_REQUIRE(blocks && a && tile_expert && out && p16 > 0 && experts > 0, SMOE_EARG, "null pointer or empty stack");
    SMOE_REQUIRE(p16 % 16 == 0, SMOE_ESHAPE, "a's rows must be a multiple of 16");
    SMOE_REQUIRE((reinterpret_cast<uintptr_t>(a) & 15) == 0, SMOE_EARG, "a must be 16-byte aligned");
    cudaStream_t st = as_stream(stream);
    const int64_t ntiles = p16 / 16;
    const int64_t row_bytes = cols / per * bytes;
    if (a_dtype == SMOE_F16 && cols % kGmKStage == 0) {
        SMOE_REQUIRE(workspace && workspace_bytes >= smoe_tile_matmul_workspace_size(p16), SMOE_EWORKSPACE,
                     "tile_matmul workspace too small");
        GemmArgs g{};
        g.blocks = blocks;
        g.row_bytes = row_bytes;
        g.end = blocks + experts * rows * row_bytes;
        g.a = static_cast<const __half*>(a);
        g.out = out;
        g.hdr = static_cast<const GemmPlanHeader*>(workspace);
        g.runs = reinterpret_cast<const TileRun*>(static_cast<uint8_t*>(workspace) + sizeof(GemmPlanHeader));
        g.status = &static_cast<GemmPlanHeader*>(workspace)->status;
        g.rows = rows;
        g.cols = cols;
        g.stage_bytes = static_cast<int>(kGmKStage / per * bytes);
        int rawb = (g.stage_bytes + 15 + 15) & ~15;
        if ((rawb / 16) % 2 == 0) rawb += 16;  // an odd number of 16-byte chunks: rows fall on different banks
        g.rawb = rawb;
        g.mblocks = static_cast<int>((rows + kGmM - 1) / kGmM);
        gemm_plan_kernel<<<1, 1024, 0, st>>>(tile_expert, ntiles, experts, static_cast<GemmPlanHeader*>(workspace),
                                             const_cast<TileRun*>(g.runs));
        if (int s = launch_status("tile_matmul plan")) return s;
        if (g_num_sms == 0) {
            int dev = 0;
            cudaGetDevice(&dev);
            cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
            if (g_num_sms <= 0) g_num_sms = 148;
        }
        const int64_t max_jobs = ntiles * g.mblocks;
        const unsigned grid = static_cast<unsigned>(std::min<int64_t>(max_jobs, g_num_sms));
        const size_t smem = 128 + size_t(2) * kGmM * rawb + size_t(2) * kGmMaxN * 512;
        int status = dispatch_kind(kind, [&](auto blk) {
            using B = decltype(blk);
            max_smem(gemm_tc_kernel<B>, static_cast<int>(smem));
            gemm_tc_kernel<B><<<grid, kGmThreads, smem, st>>>(g);
        });
        if (status) return fail(status, "block type has no decoder");
        return launch_status("tile_matmul");
    }
    SMOE_REQUIRE(a_dtype == SMOE_F16 || a_dtype == SMOE_F32, SMOE_EDTYPE, "a must be float16 or float32");
    SMOE_REQUIRE(ntiles <= 65535, SMOE_ESHAPE, "too many tiles for one tile_matmul call");
    dim3 grid(static_cast<unsigned>((rows + 7) / 8), static_cast<unsigned>(ntiles));
    int status = dispatch_kind(kind, [&](auto blk) {
        using B = decltype(blk);
        if (a_dtype == SMOE_F16)
            gemm_simt_kernel<B, __half><<<grid, 256, 0, st>>>(blocks, static_cast<const __half*>(a), tile_expert, experts,
                                                              rows, cols, row_bytes, out);
        else
            gemm_simt_kernel<B, float><<<grid, 256, 0, st>>>(blocks, static_cast<const float*>(a), tile_expert, experts,
                                                             rows, cols, row_bytes, out);
    });
    if (status) return fail(status, "block type has no decoder");
    return launch_status("tile_matmul simt");
}
