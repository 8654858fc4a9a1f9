// Grouped GEMM of a prompt's expert-sorted tiles on GGUF blocks: `tile_matmul` (strata_mlx/blocks.py:583-654)
// on the 5th-generation tensor cores.
//
// out[p, r] = W[expert of p's tile][r, :] . a[p, :] with the weights rounded to float16 (a's type) and float32
// sums. The tensor-core product is taken "swap AB": 128 weight rows are the M side of a tcgen05 MMA and a
// run of up to 8 tiles (128 tokens) of one expert is the N side, so a weight row is decoded once for every
// token of that expert in the run.
//
// Per CTA (persistent over jobs = (run of tiles, block of 128 rows)), warp-specialized, every hand-off an
// mbarrier:
//   warp 17    raw producer: per 256-column stage, the 16-byte aligned cover of each of the 128 rows' block
//              bytes by tiled TMA over the stack seen as groups of q rows (q = 16 / gcd(row bytes, 16), one
//              copy per residue class of rows) into a ring of raw slots (rows an odd number of 16-byte chunks
//              apart).
//   warp 18    activation producer: the run's rows of the stage by TMA (boxes of 128/64/32/16 rows x 64
//              columns, 128-byte swizzle) into a ring of activation slots.
//   warps 0-15 decoders: each thread reads its row's stage from shared memory, decodes 64 weights (a quarter
//              of the stage) to float16 pairs and stores them into its TMEM lane of an A slot (3 slots); after
//              a job's last stage they read the float32 accumulators back (tcgen05.ld) and write out.
//   warp 16    one thread issues tcgen05.mma kind::f16 with A from TMEM and B from shared memory, 16 MMAs of
//              K = 16 per stage, and tcgen05.commit releases the A slot, the activation slot and, after a
//              job's last stage, the accumulator.
// Every wait is bounded; a CTA whose wait gives up records SMOE_ETIMEOUT in the workspace status word and
// leaves its remaining jobs.
#include <cuda.h>

#include <mutex>
#include <type_traits>
#include <utility>

#include "blocks.cuh"
#include "gemm_dec.cuh"
#include "tc05.cuh"

namespace smoe {

constexpr int kGmDecoders = 16;                // decoder warps: 4 per TMEM lane quarter, each a quarter of a stage
constexpr int kGmThreads = 32 * (kGmDecoders + 3);  // + the MMA warp and two producer warps
constexpr int kGmM = 128;                      // weight rows per job
constexpr int kGmKStage = 256;                 // columns per pipeline stage
constexpr int kGmMaxTiles = 8;                 // tiles of 16 tokens per job -> N <= 128
constexpr int kGmMaxN = 16 * kGmMaxTiles;
constexpr int kGmASlots = 3;
constexpr int kGmMaxRaw = 4;                   // raw block stage slots in shared memory
constexpr int kGmMaxB = 3;                     // activation stage slots in shared memory
constexpr int kGmAtomBytes = kGmMaxN * 128;    // one 64-column K atom of up to 128 activation rows (128-byte swizzle)
constexpr int kGmBSlotBytes = (kGmKStage / 64) * kGmAtomBytes;
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
    // the rows variant: slot s's row goes to row slot_row[s] of out16 / out (float16 when out16 is set; rows at or
    // past out_rows are not written); without slot_row, slot s to row s
    __half* out16;
    const uint32_t* slot_row;
    int64_t out_rows;
    // a pair (blocks2 set): the same tiles and activations through a second stack of the same type and shape,
    // its jobs after the first stack's, its results in out2 / out16_2 as the first's go to out / out16
    const uint8_t* blocks2;
    float* out2;
    __half* out16_2;
    const GemmPlanHeader* hdr;
    const TileRun* runs;
    int* status;
    int64_t rows, cols, row_bytes;
    int stage_bytes;  // raw bytes of one row's 256-column stage
    int rawb;         // smem stride of a row's raw stage (>= stage_bytes + 15, an odd multiple of 16)
    int mblocks;
    int nb, nr;          // activation and raw stage slots
    int q;               // rows per 16-byte aligned group of rows (16 / gcd(row_bytes, 16)): raw TMA copies per stage
    int region_bytes;    // bytes of the raw rows of one residue class (128 / q rows) in a raw slot
};

// The tensor maps of one launch: the stack's bytes as 32-bit words in groups of q rows, and the activations
// in boxes of 16, 32, 64 and 128 rows x 64 columns (128-byte swizzle).
struct alignas(64) GemmMaps {
    CUtensorMap w;
    CUtensorMap a[4];
    CUtensorMap w2;  // a pair's second stack
};

// job -> its run of tiles, first weight row and stack: the first count x mblocks jobs take the first stack, a
// pair's next count x mblocks the second
struct GemmJob {
    TileRun run;
    int64_t row0;
    int second;
};
__device__ __forceinline__ GemmJob gemm_job(const GemmArgs& g, int job, int half) {
    const int second = job >= half ? 1 : 0;
    const int j = job - (second ? half : 0);
    return GemmJob{g.runs[j / g.mblocks], int64_t(j % g.mblocks) * kGmM, second};
}

template <class D>
struct D_lut {
    static constexpr bool value = D::kLut;
};
template <>
struct D_lut<void> {
    static constexpr bool value = false;
};


struct GemmSmem {
    uint64_t rawfull[kGmMaxRaw], rawfree[kGmMaxRaw], bfull[kGmMaxB], bfree[kGmMaxB];
    uint64_t afull[kGmASlots], afree[kGmASlots], dfull, dfree, drain;
    uint32_t tmem_base;
    int abort;
};

// Shared memory: [B slots: nb x 64 KB, 1024-aligned][IQ3_S codebook][raw slots: nr x 128 rows x rawb][mc][GemmSmem]
// (with room for rounding the q residue classes' regions up to 128 bytes and for reads a little past the
// last row)
__host__ __device__ constexpr size_t gemm_raw_slot_bytes(int rawb) { return size_t(kGmM) * rawb + 2048; }

// Offset of residue class j's rows in a raw slot. A tiled TMA copy writes to a 128-byte aligned address, so
// the regions start on 128 bytes; within a class, rows are an odd number of 16-byte chunks apart (8
// consecutive rows of one class read their 16-byte chunks on 8 different bank groups; rows of different
// classes may share one when q > 1).
__host__ __device__ constexpr int raw_region(int j, int region_bytes) { return j * ((region_bytes + 127) & ~127); }
__host__ __device__ constexpr size_t gemm_smem_bytes(int nb, int nr, int rawb, bool lut) {
    return size_t(nb) * kGmBSlotBytes + (lut ? 512 * kGmLutRep * 4 : 0) + size_t(nr) * gemm_raw_slot_bytes(rawb) +
           128 + ((sizeof(GemmSmem) + 127) & ~size_t(127));
}

// Decode quarter Q of a stage of the row staged at `row`, whose bytes start `off` bytes into it (a multiple of
// the type's offset step): false if `off` is none the type can have.
template <class D, int Q>
__device__ __forceinline__ bool decode_part(int off, const uint8_t* row, uint32_t (&out)[32], const uint32_t* lut,
                                            const uint32_t* mc) {
    const uint32_t* base = reinterpret_cast<const uint32_t*>(row + (off & ~3));
    if ((off & 3) == 0) {
        D::template decode<Q, 0>(BlockWords<0>{base}, out, lut, mc);
        return true;
    }
    if constexpr (D::kOffStep == 2) {
        if ((off & 3) == 2) {
            D::template decode<Q, 2>(BlockWords<2>{base}, out, lut, mc);
            return true;
        }
    }
    return false;
}

// B: the block type (run decoder) for the generic path; D: a specialized decoder (gemm_dec.cuh) or void
template <class B, class D>
__global__ void __launch_bounds__(kGmThreads, 1) gemm_tc_kernel(const GemmArgs g, const __grid_constant__ GemmMaps maps) {
    constexpr bool kT = !std::is_void<D>::value;
    constexpr bool kLut = kT && D_lut<D>::value;
    extern __shared__ __align__(1024) uint8_t smem[];
    const int nb = g.nb, nr = g.nr;
    const size_t raw_slot = gemm_raw_slot_bytes(g.rawb);
    uint8_t* bslots = smem;
    uint32_t* lut = reinterpret_cast<uint32_t*>(smem + size_t(nb) * kGmBSlotBytes);
    uint8_t* raw = smem + size_t(nb) * kGmBSlotBytes + (kLut ? 512 * kGmLutRep * 4 : 0);
    uint32_t* mc = reinterpret_cast<uint32_t*>(raw + size_t(nr) * raw_slot);                     // 16 x (m, c)
    GemmSmem& S = *reinterpret_cast<GemmSmem*>(reinterpret_cast<uint8_t*>(mc) + 128);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int half = g.hdr->count * g.mblocks;
    const int njobs = g.blocks2 != nullptr ? 2 * half : half;
    const int nk = static_cast<int>(g.cols / kGmKStage);

    // the 128-byte swizzle of the TMA writes and of the B descriptors needs 1024-byte aligned slots
    if (smem_addr(smem) & 1023u) {
        if (threadIdx.x == 0) atomicExch(g.status, SMOE_EARG);
        return;
    }
    if constexpr (kLut) {
        for (int i = threadIdx.x; i < 512 * kGmLutRep; i += kGmThreads) lut[i] = __ldg(&kIq3sGrid[i / kGmLutRep]);
    }
    if (threadIdx.x < 16) {
        const float mv = float(1 + 2 * threadIdx.x);
        const uint32_t mb = __half_as_ushort(__float2half_rn(mv));
        const uint32_t cb = __half_as_ushort(__float2half_rn(-1024.0f * mv));
        mc[2 * threadIdx.x] = mb | (mb << 16);
        mc[2 * threadIdx.x + 1] = cb | (cb << 16);
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < nr; ++i) {
            tc::mbar_init(&S.rawfull[i], 1);
            tc::mbar_init(&S.rawfree[i], kGmDecoders);
        }
        for (int i = 0; i < nb; ++i) {
            tc::mbar_init(&S.bfull[i], 1);
            tc::mbar_init(&S.bfree[i], 1);
        }
        for (int i = 0; i < kGmASlots; ++i) {
            tc::mbar_init(&S.afull[i], kGmDecoders);
            tc::mbar_init(&S.afree[i], 1);
        }
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
    auto give_up = [&]() {
        if (lane == 0) {
            S.abort = 1;
            atomicExch(g.status, SMOE_ETIMEOUT);
        }
    };
    // every role walks the same sequence of (job, stage); slot i of a ring of n is reused every n stages
    struct Ring {
        int slot = 0;
        uint32_t phase = 0;
        __device__ void next(int n) {
            if (++slot == n) {
                slot = 0;
                phase ^= 1;
            }
        }
    };

    if (warp == kGmDecoders + 1) {
        // ---------------- raw producer: the 16-byte aligned cover of each row's stage bytes, by TMA over the
        // stack seen as rows of q rows (a multiple of 16 bytes), one copy per residue class of rows
        Ring rr;
        uint32_t gs = 0;
        bool ok = true;
        for (int job = blockIdx.x; job < njobs && ok; job += gridDim.x) {
            const GemmJob jb = gemm_job(g, job, half);
            const TileRun run = jb.run;
            const int64_t row0 = jb.row0;
            const int64_t y0 = (int64_t(run.expert) * g.rows + row0) / g.q;
            const CUtensorMap* wmap = jb.second ? &maps.w2 : &maps.w;
            for (int s = 0; s < nk; ++s, ++gs, rr.next(nr)) {
                if (gs >= uint32_t(nr)) {
                    ok = __all_sync(0xffffffffu, tc::mbar_wait(&S.rawfree[rr.slot], rr.phase ^ 1, kWaitLimit));
                    if (!ok) break;
                }
                // q tiled copies, one per residue class of rows: rows j, j + q, ... of the job's 128
                if (lane == 0) tc::mbar_arrive_expect_tx(&S.rawfull[rr.slot], static_cast<uint32_t>(kGmM * g.rawb));
                __syncwarp();
                if (lane < g.q) {
                    const int64_t x = ((int64_t(lane) * g.row_bytes + int64_t(s) * g.stage_bytes) & ~int64_t(15)) >> 2;
                    const uint32_t dst = smem_addr(raw + size_t(rr.slot) * raw_slot + raw_region(lane, g.region_bytes));
                    if (dst & 127u) atomicExch(g.status, SMOE_EARG);  // a tiled copy's destination is 128-byte aligned
                    else tc::tma_load_2d(dst, wmap, static_cast<int>(x), static_cast<int>(y0), &S.rawfull[rr.slot]);
                }
            }
        }
        // no bulk copy may still be writing this CTA's shared memory when it exits
        for (uint32_t i = 0; i < uint32_t(nr) && i < gs; ++i) {
            const uint32_t st = gs - 1 - i;
            tc::mbar_wait(&S.rawfull[st % nr], (st / nr) & 1, kWaitLimit);
        }
        if (!ok) give_up();
    } else if (warp == kGmDecoders + 2) {
        // ---------------- activation producer: the run's rows of the stage's 256 columns by TMA into the
        // 128-byte swizzle layout (row i of atom q at q * kGmAtomBytes + 128 i)
        Ring br;
        uint32_t gs = 0;
        bool ok = true;
        for (int job = blockIdx.x; job < njobs && ok; job += gridDim.x) {
            const TileRun run = gemm_job(g, job, half).run;
            for (int s = 0; s < nk; ++s, ++gs, br.next(nb)) {
                if (gs >= uint32_t(nb)) {
                    ok = __all_sync(0xffffffffu, tc::mbar_wait(&S.bfree[br.slot], br.phase ^ 1, kWaitLimit));
                    if (!ok) break;
                }
                if (lane == 0) {
                    const uint32_t bdst = smem_addr(bslots + size_t(br.slot) * kGmBSlotBytes);
                    tc::mbar_arrive_expect_tx(&S.bfull[br.slot], static_cast<uint32_t>(run.tiles) * 16u * kGmKStage * 2u);
                    // the run's tiles as boxes of 128, 64, 32 and 16 rows (its bits), for each 64-column atom
                    int done = 0;
                    for (int b = 3; b >= 0; --b) {
                        if (!((run.tiles >> b) & 1)) continue;
                        for (int q = 0; q < kGmKStage / 64; ++q)
                            tc::tma_load_2d(bdst + q * kGmAtomBytes + done * 128, &maps.a[b], s * kGmKStage + 64 * q,
                                            run.first_tile * 16 + done, &S.bfull[br.slot]);
                        done += 16 << b;
                    }
                }
                __syncwarp();
            }
        }
        for (uint32_t i = 0; i < uint32_t(nb) && i < gs; ++i) {
            const uint32_t st = gs - 1 - i;
            tc::mbar_wait(&S.bfull[st % nb], (st / nb) & 1, kWaitLimit);
        }
        if (!ok) give_up();
    } else if (warp == kGmDecoders) {
        // ---------------- MMA issuer (the converged warp issues, one elected lane; it waits together and agrees on
        // every outcome)
        Ring br;
        uint32_t gs = 0, jobs = 0;
        bool ok = true;
        for (int job = blockIdx.x; job < njobs && ok; job += gridDim.x, ++jobs) {
            const TileRun run = gemm_job(g, job, half).run;
            const uint32_t idesc = tc::idesc_f16_f32(kGmM, 16 * run.tiles);
            if (jobs > 0) ok = __all_sync(0xffffffffu, tc::mbar_wait(&S.dfree, (jobs - 1) & 1, kWaitLimit));
            if (!ok) break;
            tc::fence_after_sync();
            for (int s = 0; s < nk; ++s, ++gs, br.next(nb)) {
                const uint32_t as = gs % kGmASlots;
                ok = __all_sync(0xffffffffu, tc::mbar_wait(&S.afull[as], (gs / kGmASlots) & 1, kWaitLimit) &&
                                                 tc::mbar_wait(&S.bfull[br.slot], br.phase, kWaitLimit));
                if (!ok) break;
                tc::fence_after_sync();
                const uint64_t bd0 = tc::smem_desc_sw128(smem_addr(bslots + size_t(br.slot) * kGmBSlotBytes));
#pragma unroll
                for (int k = 0; k < kGmKStage / 16; ++k)
                    tc::mma_f16_ts_warp(tmem, tmem + 128u + 128u * as + 8u * k,
                                        bd0 + uint64_t(((k >> 2) * kGmAtomBytes + (k & 3) * 32) >> 4), idesc,
                                        (s > 0 || k > 0) ? 1u : 0u);
                tc::mma_commit_warp(&S.afree[as]);
                tc::mma_commit_warp(&S.bfree[br.slot]);
                if (s == nk - 1) tc::mma_commit_warp(&S.dfull);
                __syncwarp();
            }
        }
        if (!ok) give_up();
    } else {
        // ---------------- decoders and epilogue (16 warps, each on its own: warp w decodes the 64 weights
        // [64 qq, 64 qq + 64) of each stage for TMEM lanes 32 (w % 4) .. + 31, qq = w / 4). TMEM lane L holds
        // weight row m = q (L % (128 / q)) + L / (128 / q) of the block: the rows of one residue class mod q
        // are 128 / q consecutive lanes, so (for q <= 4) a warp's rows share their byte offset in the stage
        // and read consecutive rows of one region of the raw slot.
        const int L = 32 * (warp & 3) + lane;
        const int per_class = kGmM / g.q;
        const int m = g.q * (L % per_class) + L / per_class;
        const int row_off = raw_region(L / per_class, g.region_bytes) + (L % per_class) * g.rawb;
        const int qq = warp >> 2;              // which 64 columns of a stage this warp decodes
        const uint32_t* lut_lane = lut + (lane % kGmLutRep);
        Ring rr;
        uint32_t gs = 0, jobs = 0;
        bool ok = true;
        for (int job = blockIdx.x; job < njobs && ok; job += gridDim.x, ++jobs) {
            const GemmJob jb = gemm_job(g, job, half);
            const TileRun run = jb.run;
            const int64_t row0 = jb.row0;
            const int mrows = static_cast<int>(min(int64_t(kGmM), g.rows - row0));
            const uint8_t* wrow = (jb.second ? g.blocks2 : g.blocks) + ((int64_t(run.expert) * g.rows + row0) + m) * g.row_bytes;
            float* const out32 = jb.second ? g.out2 : g.out;
            __half* const out16 = jb.second ? g.out16_2 : g.out16;
            for (int s = 0; s < nk; ++s, ++gs, rr.next(nr)) {
                const uint32_t as = gs % kGmASlots;
                ok = __all_sync(0xffffffffu, tc::mbar_wait(&S.rawfull[rr.slot], rr.phase, kWaitLimit) &&
                                                 (gs < kGmASlots ||
                                                  tc::mbar_wait(&S.afree[as], ((gs - kGmASlots) / kGmASlots) & 1, kWaitLimit)));
                if (!ok) break;
                tc::fence_after_sync();
                // decode 64 weights of row m into TMEM lane L, columns 128 + 128 as + 32 qq (+ 16 per 32 weights)
                const uint32_t tbase = tmem + (uint32_t(32 * (warp & 3)) << 16) + 128u + 128u * as + 32u * qq;
                const int off = static_cast<int>(reinterpret_cast<uintptr_t>(wrow + int64_t(s) * g.stage_bytes) & 15);
                const uint8_t* rrow = raw + size_t(rr.slot) * raw_slot + row_off;
                // every lane decodes (rows past the block's end decode bytes that were staged all the same and
                // only reach accumulator rows the epilogue does not write); the warp converges before the
                // .sync.aligned TMEM stores
                if constexpr (kT) {
                    uint32_t v[32];
                    bool done;
                    switch (qq) {
                        case 0: done = decode_part<D, 0>(off, rrow, v, lut_lane, mc); break;
                        case 1: done = decode_part<D, 1>(off, rrow, v, lut_lane, mc); break;
                        case 2: done = decode_part<D, 2>(off, rrow, v, lut_lane, mc); break;
                        default: done = decode_part<D, 3>(off, rrow, v, lut_lane, mc); break;
                    }
                    if (!done) atomicExch(g.status, SMOE_EARG);  // an offset the block type cannot have
                    __syncwarp();
                    tc::tmem_st16(tbase, *reinterpret_cast<const uint32_t(*)[16]>(v));
                    tc::tmem_st16(tbase + 16u, *reinterpret_cast<const uint32_t(*)[16]>(v + 16));
                } else {
#pragma unroll 1
                    for (int i = 0; i < 2; ++i) {
                        float w[32];
                        B::run(rrow + off, 2 * qq + i, w);
                        uint32_t v[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] = tc::pack_half2(w[2 * j], w[2 * j + 1]);
                        __syncwarp();
                        tc::tmem_st16(tbase + 16u * i, v);
                    }
                }
                tc::tmem_wait_st();
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) {
                    tc::mbar_arrive(&S.afull[as]);
                    tc::mbar_arrive(&S.rawfree[rr.slot]);
                }
            }
            if (!ok) break;
            // epilogue: accumulators of rows m, tokens 8 qq + 32 i .. + 7
            const int64_t s0 = int64_t(run.first_tile) * 16;
            const int ncol = 16 * run.tiles;
            // (the rows variant: lane l holds the output rows of slots s0 + l + 32 i, loaded before the wait)
            uint32_t orow[4] = {~0u, ~0u, ~0u, ~0u};
            if (g.slot_row != nullptr) {
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    if (32 * i + lane < ncol) orow[i] = __ldg(g.slot_row + s0 + 32 * i + lane);
            }
            ok = __all_sync(0xffffffffu, tc::mbar_wait(&S.dfull, jobs & 1, kWaitLimit));
            if (!ok) break;
            tc::fence_after_sync();
            if (out32 != nullptr) {
                float* obase = out32 + s0 * g.rows + row0 + m;
                for (int c0 = 8 * qq; c0 < ncol; c0 += 32) {
                    uint32_t v[8];
                    tc::tmem_ld8(tmem + (uint32_t(32 * (warp & 3)) << 16) + uint32_t(c0), v);
                    tc::tmem_wait_ld();
                    if (m < mrows) {
#pragma unroll
                        for (int j = 0; j < 8; ++j) obase[int64_t(c0 + j) * g.rows] = __uint_as_float(v[j]);
                    }
                }
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int c0 = 8 * qq + 32 * i;
                    if (c0 >= ncol) break;
                    uint32_t v[8];
                    tc::tmem_ld8(tmem + (uint32_t(32 * (warp & 3)) << 16) + uint32_t(c0), v);
                    tc::tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const uint32_t sr = __shfl_sync(0xffffffffu, orow[i], 8 * qq + j);
                        const int64_t r = g.slot_row != nullptr ? int64_t(sr) : s0 + c0 + j;
                        if (m < mrows && r < g.out_rows)
                            out16[r * g.rows + row0 + m] = __float2half_rn(__uint_as_float(v[j]));
                    }
                }
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&S.dfree);
        }
        if (!ok) give_up();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == kGmDecoders) {
        if (S.abort) {
            // let any MMA still in flight finish before the TMEM it writes is released (bounded wait)
            tc::mma_commit_warp(&S.drain);
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
constexpr int kGmSmemLimit = 227 * 1024;  // opt-in dynamic shared memory per block on sm_100

// The launch's tensor maps (GemmMaps). cuTensorMapEncodeTiled is reached through the runtime's driver entry
// point (no link against libcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encoder() {
    static std::once_flag once;
    static EncodeTiledFn encode = nullptr;
    std::call_once(once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            encode = reinterpret_cast<EncodeTiledFn>(fn);
    });
    return encode;
}

static int encode_maps(GemmMaps* maps, const uint8_t* blocks, int64_t total_rows, int64_t row_bytes, int q, int rawb,
                       const void* a, int64_t a_rows, int64_t cols) {
    EncodeTiledFn encode = encoder();
    if (!encode) return fail(SMOE_EARG, "tile_matmul: cuTensorMapEncodeTiled is not available");
    const cuuint32_t estr[2] = {1, 1};
    {
        // the stack as [total_rows / q][q * row_bytes / 4] words; a box is 128 / q groups x the stage's cover
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(q * row_bytes / 4), static_cast<cuuint64_t>(total_rows / q)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(q * row_bytes)};
        const cuuint32_t box[2] = {static_cast<cuuint32_t>(rawb / 4), static_cast<cuuint32_t>(kGmM / q)};
        const CUresult r = encode(&maps->w, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint8_t*>(blocks), dims,
                                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS)
            return fail(SMOE_EARG, "tile_matmul: block tensor map rejected (" + std::to_string(int(r)) + ")");
    }
    for (int b = 0; b < 4; ++b) {
        // (rows of the last tile past a_rows read as zeros: the copy's fill)
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(a_rows)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
        const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(16 << b)};
        const CUresult r = encode(&maps->a[b], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(a), dims, strides,
                                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (r != CUDA_SUCCESS)
            return fail(SMOE_EARG, "tile_matmul: activation tensor map rejected (" + std::to_string(int(r)) + ")");
    }
    return SMOE_OK;
}

// slot_row[where[p]] = p for every pair p; slots no pair names keep 0xffffffff
__global__ void slot_rows_kernel(const uint32_t* __restrict__ where, int64_t pairs, int64_t slots,
                                 uint32_t* __restrict__ slot_row) {
    for (int64_t p = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; p < pairs; p += int64_t(gridDim.x) * blockDim.x) {
        const uint32_t s = where[p];
        if (s < slots) slot_row[s] = static_cast<uint32_t>(p);
    }
}

// out (float32, slot order) or, the rows variant, out16 (float16) at the rows slot_row names
static int tile_matmul_impl(int kind, const uint8_t* blocks, int64_t experts, int64_t rows, int64_t cols,
                            const void* a, int a_dtype, int64_t a_rows, int64_t p16, const uint32_t* tile_expert,
                            float* out, __half* out16, const uint32_t* slot_row, int64_t out_rows, void* workspace,
                            size_t workspace_bytes, void* stream, const uint8_t* blocks2 = nullptr,
                            float* out2 = nullptr, __half* out16_2 = nullptr) {
    if (p16 == 0) return SMOE_OK;
    int per, bytes;
    if (!block_info(kind, per, bytes)) return fail(SMOE_EKIND, "block type " + std::to_string(kind) + " has no decoder");
    SMOE_REQUIRE(smoe_tileable(kind, rows, cols), SMOE_ESHAPE, "stack not tileable: rows and cols must divide by 64 and cols by the block");
    SMOE_REQUIRE(blocks && a && tile_expert && (out || out16) && p16 > 0 && experts > 0, SMOE_EARG,
                 "null pointer or empty stack");
    SMOE_REQUIRE(a_rows > 0 && a_rows <= p16, SMOE_ESHAPE, "a's rows must be 1 to the tiles' slots");
    SMOE_REQUIRE(p16 % 16 == 0, SMOE_ESHAPE, "a's rows must be a multiple of 16");
    SMOE_REQUIRE((reinterpret_cast<uintptr_t>(a) & 15) == 0, SMOE_EARG, "a must be 16-byte aligned");
    SMOE_REQUIRE((reinterpret_cast<uintptr_t>(blocks) & 15) == 0 && (reinterpret_cast<uintptr_t>(blocks2) & 15) == 0,
                 SMOE_EARG, "blocks must be 16-byte aligned");
    SMOE_REQUIRE(blocks2 == nullptr || (a_dtype == SMOE_F16 && cols % kGmKStage == 0 && (out2 || out16_2) &&
                                        (out2 != nullptr) == (out != nullptr)),
                 SMOE_EARG, "a pair of stacks takes float16 activations, columns a multiple of 256 and two outputs");
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
        g.out16 = out16;
        g.slot_row = slot_row;
        g.out_rows = out_rows;
        g.blocks2 = blocks2;
        g.out2 = out2;
        g.out16_2 = out16_2;
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
        const bool lut = kind == GdIQ3S::kKind;
        // the most raw slots (latency of the weights' DRAM reads), then the most activation slots that fit
        g.nr = kGmMaxRaw;
        g.nb = 0;
        for (int nb = kGmMaxB; nb >= 2 && !g.nb; --nb)
            if (gemm_smem_bytes(nb, g.nr, rawb, lut) <= size_t(kGmSmemLimit)) g.nb = nb;
        while (!g.nb && g.nr > 2) {
            --g.nr;
            if (gemm_smem_bytes(2, g.nr, rawb, lut) <= size_t(kGmSmemLimit)) g.nb = 2;
        }
        SMOE_REQUIRE(g.nb, SMOE_EKIND, "tile_matmul: stage does not fit in shared memory");
        const size_t smem = gemm_smem_bytes(g.nb, g.nr, rawb, lut);
        int gcd = 16;
        while (row_bytes % gcd) gcd >>= 1;
        g.q = 16 / gcd;
        g.region_bytes = (kGmM / g.q) * rawb;
        GemmMaps maps;
        if (int e = encode_maps(&maps, blocks, experts * rows, row_bytes, g.q, rawb, a, a_rows, cols)) return e;
        if (blocks2 != nullptr) {
            GemmMaps m2;
            if (int e = encode_maps(&m2, blocks2, experts * rows, row_bytes, g.q, rawb, a, a_rows, cols)) return e;
            maps.w2 = m2.w;
        }
        gemm_plan_kernel<<<1, 1024, 0, st>>>(tile_expert, ntiles, experts, static_cast<GemmPlanHeader*>(workspace),
                                             const_cast<TileRun*>(g.runs));
        if (int s = launch_status("tile_matmul plan")) return s;
        if (g_num_sms == 0) {
            int dev = 0;
            cudaGetDevice(&dev);
            cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
            if (g_num_sms <= 0) g_num_sms = 148;
        }
        const int64_t max_jobs = ntiles * g.mblocks * (blocks2 != nullptr ? 2 : 1);
        const unsigned grid = static_cast<unsigned>(std::min<int64_t>(max_jobs, g_num_sms));
        int status = SMOE_OK;
        auto launch = [&](auto kern) {
            if (int e = max_smem(kern, static_cast<int>(smem))) status = fail(e, "tile_matmul: shared memory limit");
            else kern<<<grid, kGmThreads, smem, st>>>(g, maps);
        };
        if (kind == GdQ2K::kKind) launch(gemm_tc_kernel<Q2_K, GdQ2K>);
        else if (kind == GdIQ3S::kKind) launch(gemm_tc_kernel<IQ3_S, GdIQ3S>);
        else if (kind == GdQ8_0::kKind) launch(gemm_tc_kernel<Q8_0, GdQ8_0>);
        else status = dispatch_kind(kind, [&](auto blk) { launch(gemm_tc_kernel<decltype(blk), void>); });
        if (status) return status;
        return launch_status("tile_matmul");
    }
    SMOE_REQUIRE(out != nullptr && a_rows == p16, SMOE_EDTYPE,
                 "tile_matmul_rows takes float16 activations and columns a multiple of 256");
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

extern "C" int smoe_tile_matmul(int kind, const uint8_t* blocks, int64_t experts, int64_t rows, int64_t cols,
                                const void* a, int a_dtype, int64_t p16, const uint32_t* tile_expert, float* out,
                                void* workspace, size_t workspace_bytes, void* stream) {
    return tile_matmul_impl(kind, blocks, experts, rows, cols, a, a_dtype, p16, p16, tile_expert, out, nullptr, nullptr,
                            0, workspace, workspace_bytes, stream);
}

extern "C" int smoe_tile_matmul_rows(int kind, const uint8_t* blocks, int64_t experts, int64_t rows, int64_t cols,
                                     const void* a, int64_t a_rows, int64_t p16, const uint32_t* tile_expert,
                                     const uint32_t* slot_row, int64_t out_rows, void* out, void* workspace,
                                     size_t workspace_bytes, void* stream) {
    if (p16 == 0) return SMOE_OK;
    SMOE_REQUIRE(out != nullptr && out_rows >= 0, SMOE_EARG, "null output");
    SMOE_REQUIRE(cols % kGmKStage == 0, SMOE_ESHAPE, "tile_matmul_rows takes columns a multiple of 256");
    SMOE_REQUIRE((reinterpret_cast<uintptr_t>(out) & 1) == 0, SMOE_EARG, "out must be 2-byte aligned");
    return tile_matmul_impl(kind, blocks, experts, rows, cols, a, SMOE_F16, a_rows, p16, tile_expert, nullptr,
                            static_cast<__half*>(out), slot_row, out_rows, workspace, workspace_bytes, stream);
}

extern "C" int smoe_slot_rows(const uint32_t* where, int64_t pairs, int64_t slots, uint32_t* slot_row, void* stream) {
    if (slots == 0) return SMOE_OK;
    SMOE_REQUIRE(where && slot_row && pairs >= 0 && slots > 0, SMOE_EARG, "null pointer or negative size");
    cudaStream_t st = as_stream(stream);
    if (cudaMemsetAsync(slot_row, 0xff, size_t(slots) * sizeof(uint32_t), st) != cudaSuccess)
        return launch_status("slot_rows");
    if (pairs > 0) {
        const unsigned grid = static_cast<unsigned>(std::min<int64_t>((pairs + 255) / 256, 148 * 8));
        slot_rows_kernel<<<grid, 256, 0, st>>>(where, pairs, slots, slot_row);
    }
    return launch_status("slot_rows");
}

extern "C" int smoe_tile_matmul_pair(int kind, const uint8_t* blocks_a, const uint8_t* blocks_b, int64_t experts,
                                     int64_t rows, int64_t cols, const void* a, int64_t p16,
                                     const uint32_t* tile_expert, float* out_a, float* out_b, void* workspace,
                                     size_t workspace_bytes, void* stream) {
    if (p16 == 0) return SMOE_OK;
    SMOE_REQUIRE(blocks_b != nullptr && out_a != nullptr && out_b != nullptr, SMOE_EARG, "null pointer");
    return tile_matmul_impl(kind, blocks_a, experts, rows, cols, a, SMOE_F16, p16, p16, tile_expert, out_a, nullptr,
                            nullptr, 0, workspace, workspace_bytes, stream, blocks_b, out_b, nullptr);
}

extern "C" int smoe_tile_matmul_pair_rows(int kind, const uint8_t* blocks_a, const uint8_t* blocks_b, int64_t experts,
                                          int64_t rows, int64_t cols, const void* a, int64_t a_rows, int64_t p16,
                                          const uint32_t* tile_expert, const uint32_t* slot_row, int64_t out_rows,
                                          void* out_a, void* out_b, void* workspace, size_t workspace_bytes,
                                          void* stream) {
    if (p16 == 0) return SMOE_OK;
    SMOE_REQUIRE(blocks_b != nullptr && out_a != nullptr && out_b != nullptr && out_rows >= 0, SMOE_EARG,
                 "null pointer");
    SMOE_REQUIRE(((reinterpret_cast<uintptr_t>(out_a) | reinterpret_cast<uintptr_t>(out_b)) & 1) == 0, SMOE_EARG,
                 "outputs must be 2-byte aligned");
    return tile_matmul_impl(kind, blocks_a, experts, rows, cols, a, SMOE_F16, a_rows, p16, tile_expert, nullptr,
                            static_cast<__half*>(out_a), slot_row, out_rows, workspace, workspace_bytes, stream,
                            blocks_b, nullptr, static_cast<__half*>(out_b));
}
