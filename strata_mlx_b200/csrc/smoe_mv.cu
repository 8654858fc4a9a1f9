// Decode matvec on the tensor cores for the types of the decode hot path (IQ3_S routed experts, Q8_0 shared
// expert): out[p, r] = W[idx[p], r, :] . x[p / share, :] with float16 activations.
//
// Layout (B200, one persistent CTA of 16 warps per SM):
//   - a job = (problem, pair, tile of 16 weight rows) is taken by a team of 4, 8 or 16 warps of a CTA (more
//     warps when there are few jobs) that split its columns in stages (256 columns of IQ3_S, 128 of Q8_0): warp
//     k of the team takes stages k, k + team, ... and the team adds its partial sums in shared memory in a
//     fixed order, so results do not depend on timing;
//   - each warp streams its stages' raw block bytes (16 rows) through a ring of 4 shared-memory slots with
//     cp.async, laid out so that the 32 lanes' loads of their fields hit 32 different banks: IQ3_S word-
//     transposed with 4-byte copies (word i of row r at i * 18 + r, its lanes' fields are 16 bytes apart),
//     Q8_0 row-major with 16-byte copies and a 176-byte row stride (its lanes' fields are 4 bytes apart);
//   - every lane expands its share of the weights into exact float16 integers (grid value x sign x the run's
//     odd sub-scale for IQ3_S, the int8 code for Q8_0): the A operand of mma.sync m16n8k16, whose B operand
//     is the activation column. The tensor core sums the exact products; the float16 scale d of the block
//     (IQ3_S) or run (Q8_0) multiplies each partial in float32 afterwards;
//   - the IQ3_S codebook (512 words) sits in shared memory once per bank (64 KB): lane l reads copy l, so a
//     warp's 32 lookups never conflict.
// The k index of an MMA is a permutation of the stage's columns (lane tig of a quad holds four consecutive
// weights of its row), applied the same way to A and B, so the sums are those of the plain product. All 8
// B columns hold the activation row (they would hold 8 tokens' rows when 8 tokens share an expert); only
// column 0 of D is read.
#include <utility>

#include "blocks.cuh"

namespace smoe {

constexpr int kMmWarps = 16;
constexpr int kMmThreads = 32 * kMmWarps;
constexpr int kMmStages = 4;

__device__ __forceinline__ void cp_async4(uint32_t* smem_dst, const uint8_t* gmem_src, int valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(smem_addr(smem_dst)), "l"(gmem_src),
                 "r"(valid));
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t hfma2u(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t hsub2u(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;\n" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ void bar_sync_n(int id, int threads) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ float half_lo(uint32_t w) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xffffu)));
}

// ---------------------------------------------------------------- IQ3_S
// Lane tig of a quad takes groups 16 tig .. 16 tig + 15 of the block (64 weights: runs 2 tig and 2 tig + 1),
// one group per MMA q: its qs bytes, qh bits, sign bits and sub-scale byte are contiguous.
struct MmIQ3S {
    static constexpr int kKind = 21, kStageCols = 256, kStageBytes = 110, kMmas = 16, kFlushEvery = 16;
    static constexpr bool kLut = true;
    // 4-byte copies, word-transposed: word i of row r at i * 18 + r
    static constexpr bool kCopy16 = false;
    static constexpr int kWords = 30, kRS = 18, kSlotWords = kWords * kRS;
    __device__ static uint32_t word(const uint32_t* st, int r, int p) {
        const int w = p >> 2;
        return __funnelshift_r(st[w * kRS + r], st[(w + 1) * kRS + r], 8 * (p & 3));
    }
    struct Row {
        uint32_t qs[4], qh, sg[2], m[2], c[2];
        float d;
    };
    // mc: 16 x (m, c) half2 pairs, m = 1 + 2s and c = -1024 m (shared memory)
    __device__ static void load(const uint32_t* st, int r, int off, int tig, const uint32_t* mc, Row& R) {
        const int p = off + 2 + 16 * tig;
#pragma unroll
        for (int j = 0; j < 4; ++j) R.qs[j] = word(st, r, p + 4 * j);
        R.qh = word(st, r, off + 66 + 2 * tig);
        R.sg[0] = word(st, r, off + 74 + 8 * tig);
        R.sg[1] = word(st, r, off + 78 + 8 * tig);
        const uint32_t sc = word(st, r, off + 106 + tig);
        R.d = half_lo(word(st, r, off));
        const uint2 e0 = reinterpret_cast<const uint2*>(mc)[sc & 15u];
        const uint2 e1 = reinterpret_cast<const uint2*>(mc)[(sc >> 4) & 15u];
        R.m[0] = e0.x;
        R.c[0] = e0.y;
        R.m[1] = e1.x;
        R.c[1] = e1.y;
    }
    template <int Q>
    __device__ static void frag(const Row& R, const uint32_t* lut, uint32_t& lo, uint32_t& hi) {
        const uint32_t qsb = (R.qs[Q >> 2] >> (8 * (Q & 3))) & 255u;
        const uint32_t hb = Q <= 8 ? ((R.qh << (8 - Q)) & 0x100u) : ((R.qh >> (Q - 8)) & 0x100u);
        const uint32_t g = lut[(qsb | hb) * 32];  // lut already offset by the lane
        const uint32_t t = (R.sg[Q >> 3] >> (4 * (Q & 7))) & 15u;
        const uint32_t m = R.m[Q >> 3], c = R.c[Q >> 3];
        lo = hfma2u(__byte_perm(g, 0x6464u, 0x4140), m, c) ^ ((t * 0x40008000u) & 0x80008000u);
        hi = hfma2u(__byte_perm(g, 0x6464u, 0x4342), m, c) ^ ((t * 0x10002000u) & 0x80008000u);
    }
    __device__ static float scale(const Row& R, int) { return R.d; }
    // B operand: columns 64 tig + 4 q .. + 3 for MMA q
    __device__ static void load_x(const __half* xs, int tig, uint32_t (&bx)[2 * kMmas]) {
        const uint4* v = reinterpret_cast<const uint4*>(xs + 64 * tig);
#pragma unroll
        for (int h = 0; h < 8; ++h) {
            const uint4 u = v[h];
            bx[4 * h] = u.x;
            bx[4 * h + 1] = u.y;
            bx[4 * h + 2] = u.z;
            bx[4 * h + 3] = u.w;
        }
    }
};

// ---------------------------------------------------------------- Q8_0
// Lane tig takes group 4q + tig in MMA q: four consecutive codes of run q / 2; a run's two MMAs are scaled by
// the run's d.
struct MmQ8_0 {
    static constexpr int kKind = 8, kStageCols = 128, kStageBytes = 136, kMmas = 8, kFlushEvery = 2;
    static constexpr bool kLut = false;
    // 16-byte copies, row-major, 176-byte rows (44 words: lanes' fields 4 bytes apart never share a bank)
    static constexpr bool kCopy16 = true;
    static constexpr int kChunks = 10, kRSW = 44, kSlotWords = 16 * kRSW;
    __device__ static uint32_t word(const uint32_t* st, int r, int p) {
        const int w = r * kRSW + (p >> 2);
        return __funnelshift_r(st[w], st[w + 1], 8 * (p & 3));
    }
    struct Row {
        uint32_t q[8];
        float d[4];
    };
    __device__ static void load(const uint32_t* st, int r, int off, int tig, const uint32_t*, Row& R) {
#pragma unroll
        for (int run = 0; run < 4; ++run) {
            const int p = off + 34 * run;
            R.q[2 * run] = word(st, r, p + 2 + 4 * tig);
            R.q[2 * run + 1] = word(st, r, p + 18 + 4 * tig);
            R.d[run] = half_lo(word(st, r, p));
        }
    }
    template <int Q>
    __device__ static void frag(const Row& R, const uint32_t*, uint32_t& lo, uint32_t& hi) {
        const uint32_t v = R.q[Q] ^ 0x80808080u;  // int8 -> code + 128
        lo = hsub2u(__byte_perm(v, 0x6464u, 0x4140), 0x64806480u);  // (1024 + 128 + q) - 1152 = q
        hi = hsub2u(__byte_perm(v, 0x6464u, 0x4342), 0x64806480u);
    }
    __device__ static float scale(const Row& R, int flush) { return R.d[flush]; }
    // B operand: columns 16 q + 4 tig .. + 3 for MMA q
    __device__ static void load_x(const __half* xs, int tig, uint32_t (&bx)[2 * kMmas]) {
#pragma unroll
        for (int q = 0; q < kMmas; ++q) {
            const uint2 u = *reinterpret_cast<const uint2*>(xs + 16 * q + 4 * tig);
            bx[2 * q] = u.x;
            bx[2 * q + 1] = u.y;
        }
    }
};

// One MMA of a stage: expand group Q of both rows, multiply by the activations, and after every
// kFlushEvery MMAs scale the partials by the block (or run) scale into the float32 totals.
template <class D, int Q>
__device__ __forceinline__ void mm_step(const typename D::Row& R0, const typename D::Row& R1, const uint32_t* lut,
                                        const uint32_t (&bx)[2 * D::kMmas], float (&dacc)[2][4], float (&total)[2]) {
    uint32_t lo0, hi0, lo1, hi1;
    D::template frag<Q>(R0, lut, lo0, hi0);
    D::template frag<Q>(R1, lut, lo1, hi1);
    mma16816(dacc[Q & 1], lo0, lo1, hi0, hi1, bx[2 * Q], bx[2 * Q + 1]);
    if constexpr ((Q + 1) % D::kFlushEvery == 0) {
        constexpr int f = Q / D::kFlushEvery;
        total[0] = fmaf(D::scale(R0, f), dacc[0][0] + dacc[1][0], total[0]);
        total[1] = fmaf(D::scale(R1, f), dacc[0][2] + dacc[1][2], total[1]);
#pragma unroll
        for (int c = 0; c < 4; ++c) dacc[0][c] = dacc[1][c] = 0.f;
    }
}

template <class D, int... Q>
__device__ __forceinline__ void mm_stage(const typename D::Row& R0, const typename D::Row& R1, const uint32_t* lut,
                                         const uint32_t (&bx)[2 * D::kMmas], float (&total)[2],
                                         std::integer_sequence<int, Q...>) {
    float dacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    (mm_step<D, Q>(R0, R1, lut, bx, dacc, total), ...);
}

struct MmArgs {
    const uint8_t* blocks[2];
    const uint8_t* end[2];
    __half* out[2];
    const uint32_t* idx;
    const __half* x;
    int64_t experts, rows, cols, row_bytes, pairs, share;
    int tiles;  // 16-row tiles per pair
    int jobs;   // nprob * pairs * tiles
    int team;   // warps per job: 4, 8 or 16
};

template <class D>
__global__ void __launch_bounds__(kMmThreads, 1) mv_mma_kernel(const MmArgs a) {
    extern __shared__ __align__(16) uint32_t sm[];
    uint32_t* lut = sm;                                // 512 x 32 words (IQ3_S)
    uint32_t* mc = sm + (D::kLut ? 512 * 32 : 0);     // 16 x 2 words
    float* red = reinterpret_cast<float*>(mc + 32);    // [16 warps][16 rows]
    uint32_t* ring = mc + 32 + kMmWarps * 16;          // per warp kMmStages slots
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gid = lane >> 2, tig = lane & 3;
    const int team = a.team, teams = kMmWarps / team;
    const int tid_team = warp / team, kq = warp % team;
    if constexpr (D::kLut) {
        for (int i = threadIdx.x; i < 512 * 32; i += kMmThreads) lut[i] = __ldg(&kIq3sGrid[i >> 5]);
    }
    if (threadIdx.x < 16) {
        const float mv = float(1 + 2 * threadIdx.x);
        const uint32_t mb = __half_as_ushort(__float2half_rn(mv));
        const uint32_t cb = __half_as_ushort(__float2half_rn(-1024.0f * mv));
        mc[2 * threadIdx.x] = mb | (mb << 16);
        mc[2 * threadIdx.x + 1] = cb | (cb << 16);
    }
    __syncthreads();
    uint32_t* my = ring + warp * (kMmStages * D::kSlotWords);
    const uint32_t* mylut = lut + lane;
    const int S = static_cast<int>(a.cols / D::kStageCols);
    const int my_stages = S > kq ? (S - kq + team - 1) / team : 0;  // stages kq, kq + team, ... of every job
    const int nteams = gridDim.x * teams;
    const int q0 = blockIdx.x * teams + tid_team;
    const int my_jobs = q0 < a.jobs ? (a.jobs - q0 + nteams - 1) / nteams : 0;
    const int64_t per_prob = a.pairs * a.tiles;

    int pre_job = 0, pre_k = 0, pre_prob = 0, pre_tile = 0;
    int64_t pre_pair = 0;
    uint32_t pre_e = 0;
    int cur_prob = 0, cur_tile = 0;
    int64_t cur_pair = 0;
    uint32_t cur_e = 0;
#define SMOE_LOCATE(JOB, PROB, PAIR, TILE, E)                    \
    do {                                                         \
        const int64_t j_ = int64_t(q0) + int64_t(JOB) * nteams;  \
        PROB = static_cast<int>(j_ / per_prob);                  \
        const int64_t rest_ = j_ - int64_t(PROB) * per_prob;     \
        PAIR = rest_ / a.tiles;                                  \
        TILE = static_cast<int>(rest_ - PAIR * a.tiles);         \
        E = a.idx[PAIR];                                         \
    } while (0)

    // lanes 2r, 2r + 1 copy row r of the stage the copy cursor points at, from the aligned cover of its bytes
    auto issue = [&](int slot) {
        if (pre_e >= a.experts) return;
        const int r = lane >> 1;
        const int64_t row = int64_t(pre_tile) * 16 + r;
        if (row >= a.rows) return;
        const int s = kq + team * pre_k;
        const uint8_t* src = (pre_prob ? a.blocks[1] : a.blocks[0]) + (int64_t(pre_e) * a.rows + row) * a.row_bytes +
                             int64_t(s) * D::kStageBytes;
        const uint8_t* end = pre_prob ? a.end[1] : a.end[0];
        uint32_t* slot_base = my + slot * D::kSlotWords;
        if constexpr (D::kCopy16) {
            const uint8_t* g = reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(src) & ~uintptr_t(15));
            uint32_t* dst = slot_base + r * D::kRSW;
            for (int c = lane & 1; c < D::kChunks; c += 2) {
                const uint8_t* p = g + 16 * c;
                const int valid = p < end ? static_cast<int>(end - p < 16 ? end - p : 16) : 0;
                cp_async16(dst + 4 * c, valid ? p : g, valid);
            }
        } else {
            const uint8_t* g = reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(src) & ~uintptr_t(3));
            uint32_t* dst = slot_base + r;
            if (g + 4 * D::kWords <= end) {
#pragma unroll
                for (int w = lane & 1; w < D::kWords; w += 2) cp_async4(dst + w * D::kRS, g + 4 * w, 4);
            } else {
                for (int w = lane & 1; w < D::kWords; w += 2) {
                    const uint8_t* p = g + 4 * w;
                    const int valid = p < end ? static_cast<int>(end - p < 4 ? end - p : 4) : 0;
                    cp_async4(dst + w * D::kRS, valid ? p : g, valid);
                }
            }
        }
    };
    auto advance_pre = [&]() {
        if (++pre_k == my_stages) {
            pre_k = 0;
            if (++pre_job < my_jobs) SMOE_LOCATE(pre_job, pre_prob, pre_pair, pre_tile, pre_e);
        }
    };

    const int items = my_jobs * my_stages;
    if (my_jobs > 0) SMOE_LOCATE(0, pre_prob, pre_pair, pre_tile, pre_e);
    for (int i = 0; i < kMmStages - 1; ++i) {
        if (i < items) {
            issue(i % kMmStages);
            advance_pre();
        }
        cp_async_commit();
    }
    constexpr int kAlign = D::kCopy16 ? 15 : 3;  // misalignment of a row's stage within its first copied unit
    float total[2] = {0.f, 0.f};
    for (int job = 0; job < my_jobs; ++job) {
        SMOE_LOCATE(job, cur_prob, cur_pair, cur_tile, cur_e);
        for (int k = 0; k < my_stages; ++k) {
            const int it = job * my_stages + k;
            if (it + kMmStages - 1 < items) {
                issue((it + kMmStages - 1) % kMmStages);
                advance_pre();
            }
            cp_async_commit();
            cp_async_wait<kMmStages - 1>();
            __syncwarp();
            if (cur_e < a.experts) {
                const int s = kq + team * k;
                const uint32_t* st = my + (it % kMmStages) * D::kSlotWords;
                const int64_t r0 = int64_t(cur_tile) * 16;
                const uint8_t* base = (cur_prob ? a.blocks[1] : a.blocks[0]) + (int64_t(cur_e) * a.rows + r0) * a.row_bytes +
                                      int64_t(s) * D::kStageBytes;
                const int off0 = static_cast<int>(reinterpret_cast<uintptr_t>(base + int64_t(gid) * a.row_bytes) & kAlign);
                const int off1 =
                    static_cast<int>(reinterpret_cast<uintptr_t>(base + int64_t(gid + 8) * a.row_bytes) & kAlign);
                typename D::Row R0, R1;
                D::load(st, gid, off0, tig, mc, R0);
                D::load(st, gid + 8, off1, tig, mc, R1);
                uint32_t bx[2 * D::kMmas];
                D::load_x(a.x + (cur_pair / a.share) * a.cols + int64_t(s) * D::kStageCols, tig, bx);
                mm_stage<D>(R0, R1, mylut, bx, total, std::make_integer_sequence<int, D::kMmas>{});
            }
            __syncwarp();
        }
        // the team's partial sums of this job's 16 rows, added in warp order
        float* rq = red + (tid_team * team) * 16;
        if (tig == 0) {
            rq[kq * 16 + gid] = total[0];
            rq[kq * 16 + gid + 8] = total[1];
        }
        total[0] = total[1] = 0.f;
        bar_sync_n(1 + tid_team, 32 * team);
        if (kq == 0 && lane < 16) {
            const int64_t row = int64_t(cur_tile) * 16 + lane;
            if (cur_e < a.experts && row < a.rows) {
                float v = rq[lane];
                for (int w = 1; w < team; ++w) v += rq[16 * w + lane];
                (cur_prob ? a.out[1] : a.out[0])[cur_pair * a.rows + row] = __float2half_rn(v);
            }
        }
        bar_sync_n(1 + tid_team, 32 * team);
    }
    cp_async_wait<0>();
#undef SMOE_LOCATE
}

static int g_mm_sms = 0;

// Launch the tensor-core decode matvec when it takes the problem: 0 launched, 1 not taken, else an error.
int mv_mma_try(int kind0, int kind1, const uint8_t* b0, const uint8_t* b1, int64_t experts, int64_t rows, int64_t cols,
               int64_t row_bytes, const uint32_t* idx, int64_t pairs, int64_t share, const __half* x, __half* o0,
               __half* o1, int nprob, cudaStream_t st) {
    if (kind0 != kind1) return 1;
    auto go = [&](auto dec) -> int {
        using D = decltype(dec);
        if (cols % D::kStageCols) return 1;
        if (reinterpret_cast<uintptr_t>(x) & 15) return 1;
        MmArgs a{};
        a.blocks[0] = b0;
        a.blocks[1] = b1;
        a.end[0] = b0 + experts * rows * row_bytes;
        a.end[1] = b1 + experts * rows * row_bytes;
        a.out[0] = o0;
        a.out[1] = o1;
        a.idx = idx;
        a.x = x;
        a.experts = experts;
        a.rows = rows;
        a.cols = cols;
        a.row_bytes = row_bytes;
        a.pairs = pairs;
        a.share = share;
        a.tiles = static_cast<int>((rows + 15) / 16);
        const int64_t jobs = int64_t(nprob) * pairs * a.tiles;
        if (jobs > (int64_t(1) << 30)) return 1;
        a.jobs = static_cast<int>(jobs);
        if (g_mm_sms == 0) {
            int dev = 0;
            cudaGetDevice(&dev);
            cudaDeviceGetAttribute(&g_mm_sms, cudaDevAttrMultiProcessorCount, dev);
            if (g_mm_sms <= 0) g_mm_sms = 148;
        }
        // the team: enough warps on each job that every SM's 16 warps have work, no more than there are stages
        const int S = static_cast<int>(cols / D::kStageCols);
        int team = 4;
        while (team < 16 && jobs * team < int64_t(g_mm_sms) * kMmWarps && 2 * team <= S) team *= 2;
        a.team = team;
        const int teams = kMmWarps / team;
        const int64_t want = (jobs + teams - 1) / teams;
        const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(want, g_mm_sms)));
        const size_t smem =
            size_t((D::kLut ? 512 * 32 : 0) + 32 + kMmWarps * 16 + kMmWarps * kMmStages * D::kSlotWords) * 4;
        if (int s = max_smem(mv_mma_kernel<D>, static_cast<int>(smem))) return fail(s, "matvec: shared memory limit");
        mv_mma_kernel<D><<<grid, kMmThreads, smem, st>>>(a);
        return launch_status("matvec (tensor cores)");
    };
    if (kind0 == MmIQ3S::kKind) return go(MmIQ3S{});
    if (kind0 == MmQ8_0::kKind) return go(MmQ8_0{});
    return 1;
}

}  // namespace smoe
