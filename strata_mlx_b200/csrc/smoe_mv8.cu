// Decode matvec on the int8 tensor cores for the types of the decode hot path (IQ3_S routed experts, Q8_0
// shared expert): out[p, r] = W[idx[p], r, :] . x[p / share, :] with float16 activations.
//
// Every product is exact integer arithmetic until one float32 scaling per block:
//   - the activations are split, per row and 256-column block, into two int8 vectors: x = s (hi + lo / 128)
//     with s = max|x| / 127 over the block (|error| <= s / 256, far below float16's own rounding of the
//     weights); each CTA does this for the rows it needs, into shared memory, while its first weight stages
//     load;
//   - the weights enter the MMA as int8: Q8_0 codes as stored, IQ3_S as the grid word of a group's 9-bit
//     index (16 copies of the 512-word grid in shared memory, 32 KB, so lookups rarely share a bank) with the
//     group's signs applied by xor;
//   - mma.sync m16n8k32 s8 takes one 32-weight run per MMA: column 0 of B holds hi, column 1 holds lo, so one
//     MMA gives both sums of a run; 128 hi + lo times the run's integer sub-scale (1 + 2 s for IQ3_S) adds into
//     an int32 total per row and block (|total| < 2^31 for any weights), scaled once by d s / 128 (IQ3_S), or
//     run by run by d s / 128 (Q8_0).
// Layout (B200, one persistent CTA of 16 warps per SM): a job = (problem, pair, tile of 16 weight rows) is
// taken by a team of 1 to 16 warps (the size that gives the shortest longest warp) that split its 512-
// (IQ3_S: two blocks) or 128-column (Q8_0) stages; the team adds its partial sums in shared memory in a fixed
// order.
// A tile holds rows c, c + q, c + 2q, ... of one residue class c mod q (q = 16 / gcd(row bytes, 16)), so its
// 16 rows' bytes sit at one offset within 16 bytes: every warp loads its stages with one tiled TMA copy each
// (the stack seen as groups of q rows), rows an odd number of 16-byte chunks apart, through a ring of
// shared-memory slots, and reads every field at a warp-uniform offset.
#include <cuda.h>

#include <algorithm>
#include <mutex>
#include <utility>
#include <vector>

#include "mv8.cuh"
#include "mv8_dev.cuh"
#include "router_dev.cuh"

namespace smoe {
// A wait for a weight copy that gives up (it should not: each is bounded, about a second) records SMOE_ETIMEOUT
// here; the launch's outputs are then not valid. smoe_matvec_status reads and clears it. g_mv8_polls is the
// bound in polls (each suspends up to 1 ms), settable for tests.
static __device__ int g_mv8_status = 0;
static __device__ uint32_t g_mv8_polls = kM8WaitLimit;
// Test hook: when set, each warp withholds its first weight copy (neither issued nor arrived), so the wait for
// it runs out after g_mv8_polls polls; the drain then skips that copy.
static __device__ int g_mv8_withhold = 0;

__device__ __forceinline__ void mv8_gave_up(int lane) {
    if (lane == 0) atomicExch(&g_mv8_status, SMOE_ETIMEOUT);
}

// ---------------------------------------------------------------- one stack (or a gate / up pair)
// The kernel the single entry points use: its geometry (stage, row stride) is the block type's, known at
// compile time.

struct M8Args {
    const uint32_t* idx;
    const __half* x;
    const __half *gate, *up;  // when gate is set, the activations are swiglu(gate, up) (down's input)
    __half* out[2];
    int64_t experts, rows, cols, row_bytes, pairs, share;
    int q, lq;      // rows per 16-byte aligned group of rows (a power of two) and its log2
    int tiles;      // tiles of 16 rows (of one residue class) per pair
    int jobs;       // nprob * pairs * tiles
    int team;       // warps per job: 1, 2, 4, 8 or 16
    int xrows;      // activation rows (pairs / share)
    int xwin;       // activation rows a CTA holds: its jobs' rows from the first one's on (<= xrows)
    int nslots;     // ring slots per warp
    // when cy is set, the product is the shared expert's down and out[0] receives the block's combine instead:
    // out[t, r] = half(sum_j cy[t, j, r] cw[t, j]) + half(half(sigmoid(cg[t])) half(product[t, r])) (pair t is
    // token t)
    const __half* cy;
    const float* cw;
    const __half* cg;
    int ck;
    // bit 0: idx, bit 1: the activations may be read before pdl_wait (the launch just before this one does not
    // write them), so the first weight copies and the activation split overlap that launch's end
    int early;
    // pairs a job takes: 1, or up to 4 for a one-expert stack whose pairs each have their own activation row
    // (the shared expert over several tokens: the weights are read and expanded once for all of them)
    int tok;
};
// a job's place (worked out once per job, 32-bit): problem, pair, expert, the tile's residue class and block
// of 16 q rows, the first row of its TMA box, the activation row
struct alignas(8) M8WhereS {
    int prob, cls, blk, xr, pair;
    uint32_t e;
    int y, pad;
};
constexpr int kM8SMaskRows = 1024;  // activation rows a CTA can mark as needed
constexpr int kM8WhereSBytes = kM8Warps * 4 * int(sizeof(M8WhereS)) + kM8SMaskRows / 8;

struct alignas(64) M8Maps2 {
    CUtensorMap w[2];
};

template <class D>
__global__ void __launch_bounds__(kM8Threads, 1) mv8s_kernel(const M8Args a, const __grid_constant__ M8Maps2 maps) {
    extern __shared__ __align__(128) uint8_t sm[];
    constexpr int kSlot = 16 * D::kRS;
    const int ns = a.nslots;
    uint8_t* ring = sm;                                                         // [warp][slot] 16 rows x kRS
    uint64_t* bars = reinterpret_cast<uint64_t*>(ring + size_t(kM8Warps) * ns * kSlot);  // [warp][slot]
    float* red = reinterpret_cast<float*>(bars + kM8Warps * kM8MaxSlots);       // [16 warps][4 pairs][16 rows]
    uint8_t* spare = reinterpret_cast<uint8_t*>(red + kM8Warps * 64);           // kM8WhereSBytes
    uint32_t* need = reinterpret_cast<uint32_t*>(spare + kM8WhereSBytes - kM8SMaskRows / 8);  // kM8SMaskRows bits
    uint32_t* lut = reinterpret_cast<uint32_t*>(spare + kM8WhereSBytes);        // 512 x 16 words
    const int xblocks = static_cast<int>(a.cols / kM8XBlock);
    // the activation rows xr_lo .. xr_lo + xwin - 1 (row xr at xr - xr_lo)
    float* xscale = reinterpret_cast<float*>(lut + (D::kLut ? 8192 : 0));        // [xwin][xblocks]
    int8_t* xhi = reinterpret_cast<int8_t*>(xscale + ((a.xwin * xblocks + 3) & ~3));  // [xwin][cols]
    int8_t* xlo = xhi + size_t(a.xwin) * a.cols;
    float* xsum = reinterpret_cast<float*>(xlo + size_t(a.xwin) * a.cols);  // [xwin][cols / 16] (the K-types)

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gid = lane >> 2, tig = lane & 3;
    const bool withhold = g_mv8_withhold == 1;
    if (smem_addr(sm) & 127u) return;  // a tiled copy's destination is 128-byte aligned (the launch gives that)
    const int team = a.team, teams = kM8Warps / team;
    const int tid_team = warp / team, kq = warp % team;
    const int S = static_cast<int>(a.cols / D::kStageCols);
    const int my_stages = S > kq ? (S - kq + team - 1) / team : 0;
    // CTA b takes the jobs [b J / G, (b + 1) J / G) (neighbouring tiles, so few activation rows); its team i
    // takes every teams-th of them from the i-th on (at most 32: one per lane of the warp's job table)
    const int cj0 = static_cast<int>(int64_t(blockIdx.x) * a.jobs / gridDim.x);
    const int cj1 = static_cast<int>(int64_t(blockIdx.x + 1) * a.jobs / gridDim.x);
    const int tok = a.tok;
    const int units = static_cast<int>((a.pairs + tok - 1) / tok);  // a job's pairs: [unit tok, unit tok + tok)
    const int per_prob = units * a.tiles;  // < 2^30 (the host checks)
    // a window of the activation rows (xwin < xrows, one problem): the CTA's jobs are consecutive, so their rows
    // run from its first job's to its last job's, which the host sized xwin for (checked here once: a CTA
    // whose rows would not fit records SMOE_ESHAPE and takes no job)
    int xr_lo = 0;
    bool window_ok = true;
    if (a.xwin < a.xrows && cj0 < cj1) {
        const int u0 = cj0 / a.tiles, u1 = (cj1 - 1) / a.tiles;
        const int share = static_cast<int>(a.share);
        xr_lo = tok == 1 ? u0 / share : u0 * tok;
        const int xr_hi = tok == 1 ? u1 / share : min(u1 * tok + tok - 1, a.xrows - 1);
        window_ok = a.jobs == per_prob && xr_hi - xr_lo < a.xwin;
        if (!window_ok && threadIdx.x == 0) atomicExch(&g_mv8_status, SMOE_ESHAPE);
    }
    const int q0 = cj0 + tid_team;
    const int my_jobs = q0 < cj1 && window_ok ? min((cj1 - q0 + teams - 1) / teams, 32) : 0;
    uint8_t* my_ring = ring + size_t(warp) * ns * kSlot;
    uint64_t* my_bars = bars + warp * kM8MaxSlots;

    if (lane == 0) {
        for (int i = 0; i < ns; ++i) tc::mbar_init(&my_bars[i], 1);
        tc::fence_barrier_init();
    }
    const bool masked = a.xrows <= kM8SMaskRows;
    for (int i = threadIdx.x; i < kM8SMaskRows / 32; i += kM8Threads) need[i] = 0u;
    // the codebook fills while the kernel before this one finishes; so do the first weight copies and the
    // activation split when their inputs are older than that kernel (a.early); the rest waits for it
    if constexpr (D::kLut) D::fill(lut);
    const bool early_idx = a.early & 1, early_x = (a.early >> 1) & 1;

    // lane l's job (the warp's l-th): problem, pair, tile (residue class and block); its expert and the first
    // row of its TMA box once the indices may be read. A job's activation row is its pair's / share.
    int j_prob = 0, j_pair = 0, j_cls = 0, j_blk = 0, j_y = 0, j_valid = 0;
    const bool has = lane < my_jobs;
    if (has) {
        const int j = q0 + lane * teams;
        j_prob = j / per_prob;
        const int rest = j - j_prob * per_prob;
        j_pair = rest / a.tiles;
        const int tile = rest - j_pair * a.tiles;
        j_cls = tile & (a.q - 1);
        j_blk = tile >> a.lq;
    }
    auto place = [&]() {
        if (has) {
            const uint32_t e = __ldg(a.idx + int64_t(j_pair) * tok);
            j_valid = e < a.experts ? 1 : 0;
            j_y = static_cast<int>((int64_t(j_valid ? e : 0) * a.rows) >> a.lq) + 16 * j_blk;
        }
    };
    __syncthreads();
    if (masked && has && my_stages > 0) {
        if (tok == 1) {
            const int xr = j_pair / static_cast<int>(a.share);
            atomicOr(&need[xr >> 5], 1u << (xr & 31));
        } else {
            for (int t = 0; t < tok && j_pair * tok + t < a.xrows; ++t) {
                const int xr = j_pair * tok + t;
                atomicOr(&need[xr >> 5], 1u << (xr & 31));
            }
        }
    }
    __syncthreads();

    // the copy cursor (warp-uniform): the next item's job, stage, slot, byte position in the row
    int i_job = 0, i_k = 0, i_slot = 0, i_pos = 0, i_y = 0, i_map = 0, i_valid = 0, issued = 0;
    auto seek = [&](int job) {
        i_job = job;
        i_k = 0;
        if (job >= my_jobs || my_stages == 0) {
            i_job = my_jobs;
            return;
        }
        i_map = __shfl_sync(0xffffffffu, j_prob, job);
        i_pos = __shfl_sync(0xffffffffu, j_cls, job) * static_cast<int>(a.row_bytes) + kq * D::kStageBytes;
        i_y = __shfl_sync(0xffffffffu, j_y, job);
        i_valid = __shfl_sync(0xffffffffu, j_valid, job);
    };
    // issue the cursor's item (a pair naming no expert copies nothing and completes the slot's phase with a
    // plain arrive, so every item takes one phase) and move on; the weights are read once: evict-first in L2
    const uint64_t stream_policy = tc::policy_evict_first();
    auto issue = [&]() {
        if (lane == 0 && !(withhold && issued == 0)) {
            if (i_valid) {
                tc::mbar_arrive_expect_tx(&my_bars[i_slot], static_cast<uint32_t>(kSlot));
                tc::tma_load_2d_hint(smem_addr(my_ring + i_slot * kSlot), &maps.w[i_map], (i_pos & ~15) >> 2, i_y,
                                     &my_bars[i_slot], stream_policy);
            } else {
                tc::mbar_arrive(&my_bars[i_slot]);
            }
        }
        ++issued;
        if (++i_slot == ns) i_slot = 0;
        i_pos += team * D::kStageBytes;
        if (++i_k == my_stages) seek(i_job + 1);
    };
    // the activations, split per 256-column block into int8 hi and lo: a warp per block, 8 values a lane
    auto split = [&]() {
        for (int blk = warp; blk < a.xwin * xblocks; blk += kM8Warps) {
            const int xw = blk / xblocks, b = blk % xblocks, xr = xr_lo + xw;
            if (xr >= a.xrows) break;
            if (masked && !((need[xr >> 5] >> (xr & 31)) & 1u)) continue;
            const int64_t at = int64_t(xw) * a.cols + int64_t(b) * kM8XBlock + 8 * lane;
            m8_split(a.x, a.gate, a.up, at + int64_t(xr_lo) * a.cols, xhi + at, xlo + at, xscale + blk, lane,
                     D::kXsum ? xsum + (int64_t(xw) * a.cols + int64_t(b) * kM8XBlock) / 16 : nullptr);
        }
    };
    if (early_idx) {
        place();
        seek(0);
        while (i_job < my_jobs && issued < ns - 1) issue();
    }
    if (early_x) split();
    pdl_wait();  // (from here on every input may be read and outputs written)
    if (!early_idx) {
        place();
        seek(0);
        while (i_job < my_jobs && issued < ns - 1) issue();
    }
    if (!early_x) split();
    __syncthreads();

    // a team of one warp needs no named barrier (there are 16, barrier 0 is __syncthreads')
    auto team_sync = [&]() {
        if (team == 1) __syncwarp();
        else asm volatile("bar.sync %0, %1;\n" ::"r"(1 + tid_team), "r"(32 * team) : "memory");
    };
    // a wait that gives up (it should not) leaves the warp's remaining stages undone but keeps it in step
    // with its team's barriers
    bool ok = true;
    const uint32_t polls = g_mv8_polls;
    float total[2] = {0.f, 0.f};
    int slot = 0, waited = 0;
    uint32_t phase = 0;
    for (int job = 0; job < my_jobs; ++job) {
        const int prob = __shfl_sync(0xffffffffu, j_prob, job);
        const int pair = __shfl_sync(0xffffffffu, j_pair, job);
        const int cls = __shfl_sync(0xffffffffu, j_cls, job);
        const int blk = __shfl_sync(0xffffffffu, j_blk, job);
        const int valid = __shfl_sync(0xffffffffu, j_valid, job);
        const int xr = (tok == 1 ? pair / static_cast<int>(a.share) : pair * tok) - xr_lo;  // (in the window)
        const int nt = tok == 1 ? 1 : min(tok, static_cast<int>(a.pairs) - pair * tok);
        const uint8_t* xh = reinterpret_cast<const uint8_t*>(xhi) + int64_t(xr) * a.cols;
        const uint8_t* xl = reinterpret_cast<const uint8_t*>(xlo) + int64_t(xr) * a.cols;
        const float* xsc = xscale + xr * xblocks;
        int pos = cls * static_cast<int>(a.row_bytes) + kq * D::kStageBytes;
        int xc = kq * D::kStageCols;
        for (int k = 0; k < my_stages; ++k, pos += team * D::kStageBytes, xc += team * D::kStageCols) {
            // keep ns - 1 copies ahead; the slot refilled is the one this warp finished last
            __syncwarp();
            if (ok && i_job < my_jobs) issue();  // (after a wait gave up, nothing more is copied)
            const int cur = slot;
            if (ok) {
                ok = __all_sync(0xffffffffu, tc::mbar_wait(&my_bars[cur], phase, polls));
                if (ok) ++waited;
                else mv8_gave_up(lane);
            }
            if (++slot == ns) {
                slot = 0;
                phase ^= 1;
            }
            if (!ok || !valid) continue;
            const uint8_t* st = my_ring + cur * kSlot + (pos & 15);
            if constexpr (D::kTokens) {
                if (tok > 1) {
                    D::stage_tokens(st + gid * D::kRS, st + (gid + 8) * D::kRS, tig, gid, xh + xc, xl + xc, a.cols,
                                    xsc + xc / kM8XBlock, xblocks, nt, total);
                    continue;
                }
            }
            if constexpr (D::kXsum)
                D::stage(st + gid * D::kRS, st + (gid + 8) * D::kRS, tig, gid, xh + xc, xl + xc, xsc + xc / kM8XBlock,
                         xsum + (int64_t(xr) * a.cols + xc) / 16, total);
            else
                D::stage(st + gid * D::kRS, st + (gid + 8) * D::kRS, tig, gid, lut, xh + xc, xl + xc,
                         xsc + xc / kM8XBlock, total);
        }
        // the two sub-blocks' lanes of a run (the K-types with sub-blocks of 16) into one
        if constexpr (D::kHalves) {
            total[0] += __shfl_xor_sync(0xffffffffu, total[0], 1);
            total[1] += __shfl_xor_sync(0xffffffffu, total[1], 1);
        }
        // the team's partial sums of this job's 16 rows (for each of its pairs: lane tig holds pair tig's),
        // added in warp order
        float* rq = red + (tid_team * team) * 64;
        if (tig < nt) {
            rq[(kq * 4 + tig) * 16 + gid] = total[0];
            rq[(kq * 4 + tig) * 16 + gid + 8] = total[1];
        }
        total[0] = total[1] = 0.f;
        team_sync();
        if (kq == 0 && lane < 16) {
            const int64_t row = int64_t(blk) * 16 * a.q + cls + int64_t(a.q) * lane;
            if (valid && row < a.rows) {
                for (int t = 0; t < nt; ++t) {
                    float v = rq[t * 16 + lane];
                    for (int i = 1; i < team; ++i) v += rq[(i * 4 + t) * 16 + lane];
                    const __half prod = __float2half_rn(v);
                    const int64_t pp = tok == 1 ? pair : int64_t(pair) * tok + t;
                    __half* o = (prob ? a.out[1] : a.out[0]) + pp * a.rows + row;
                    if (a.cy == nullptr) *o = prod;
                    else *o = combine_one(a.cy + pp * a.ck * a.rows + row, a.rows, a.cw + pp * a.ck, a.ck, a.cg[pp],
                                          prod);
                }
            }
        }
        team_sync();
    }
    // the next kernel may start placing its CTAs (releasing right after the wait instead measured slower: the
    // waiting CTAs of the next kernel crowd the running ones)
    pdl_release();
    // no copy may still be writing this CTA's shared memory when it exits: every item was waited for, unless a
    // wait gave up; then the items from the one it gave up on are waited for here with the full bound (no item
    // was issued after it)
    if (!ok && lane == 0)
        for (int i = withhold ? max(waited, 1) : waited; i < issued; ++i)
            tc::mbar_wait(&my_bars[i % ns], (i / ns) & 1, kM8WaitLimit);
    __syncwarp();
}

// ---------------------------------------------------------------- several stacks in one launch
// The same work for up to four problems of either type (the decode step's routed and shared gate / up
// products): a job's problem, its type and geometry are read per job.

// One stack's products in a launch: its pairs (expert idx[p], activation row p / share of source xs) times
// its row tiles. Two stacks that share pairs and activations (gate and up) are two problems.
struct M8Prob {
    const uint32_t* idx;
    __half* out;
    int64_t rows, row_bytes;
    uint32_t experts;
    int kind;                     // 21 IQ3_S (two-block stages), 8 Q8_0
    int stage_cols, stage_bytes;  // a stage of one row
    int rs;                       // its rows' stride in a ring slot (an odd number of 16-byte chunks)
    int q, lq;                    // rows per 16-byte aligned group of rows (a power of two) and its log2
    int tiles, stages;            // tiles of 16 rows (of one residue class) per pair, stages per row
    int job0, jobs;               // its jobs in the launch: [job0, job0 + jobs)
    int pairs, share, xs;         // pairs, pairs per activation row, activation source
    int early;                    // idx may be read before pdl_wait (the launch ahead does not write it)
    int wait;                     // idx is written by this launch's route: read it once the route is in
};
// An activation source: rows of `cols` float16, or the SwiGLU of two such (down's input).
struct M8X {
    const __half *x, *gate, *up;
    int rows, cols;
    int row0;    // its first row among all sources' rows
    int scale0;  // its first block scale
    int64_t byte0;  // its hi values' offset in the split area (its lo values follow rows x cols later)
    int early;      // may be read before pdl_wait
};
constexpr int kM8MaxProbs = 4, kM8MaxX = 4;
constexpr int kM8MaxRows = 1024;   // activation rows of all sources
constexpr int kM8MaxWarpJobs = 32;  // jobs of one warp (one per lane of its job table)
constexpr int kM8MaxPref = 2;
struct M8Launch {
    M8Prob p[kM8MaxProbs];
    M8X x[kM8MaxX];
    M8Pref pf[kM8MaxPref];  // later launches' weights fetched into L2 while this one streams its own
    M8Route r;              // the route of the tokens (has_route): CTAs [0, route_ctas) hold two router rows each
    int npf, has_route, route_ctas;
    int nprob, nx, jobs, team, nslots, slot_bytes, lut, scales;
    int64_t xbytes;
};
constexpr int kM8RouteBytes = 2 * 4 * kRtTokens * 4 + 16;  // the route's partial sums and its last-CTA flag

__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
// warps 0..7 of a CTA (the route's rows) meet at named barrier 15 (team barriers use 1..8)
__device__ __forceinline__ void route_sync() { asm volatile("bar.sync 15, 256;" ::: "memory"); }
struct alignas(64) M8Maps {
    CUtensorMap w[kM8MaxProbs];
};

// Layout: jobs go round-robin over all the launch's teams, CTA-fastest (every SM gets a share of every
// problem, the costliest problems first). A warp's jobs (at most 32) are worked out once, lane l holding its
// l-th job's place in registers; the copy cursor and the consumer read them with a shuffle per job, and every
// per-stage step is warp-uniform arithmetic (lane 0 alone issues the copy).
__global__ void __launch_bounds__(kM8Threads, 1) mv8_kernel(const __grid_constant__ M8Launch L,
                                                            const __grid_constant__ M8Maps maps) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int ns = L.nslots, slot_bytes = L.slot_bytes;
    uint8_t* ring = sm;                                                                   // [warp][slot]
    uint64_t* bars = reinterpret_cast<uint64_t*>(ring + size_t(kM8Warps) * ns * slot_bytes);  // [warp][slot]
    float* red = reinterpret_cast<float*>(bars + kM8Warps * kM8MaxSlots);                 // [16 warps][16 rows]
    uint32_t* need = reinterpret_cast<uint32_t*>(red + kM8Warps * 16);                    // kM8MaxRows bits
    uint32_t* lut = need + kM8MaxRows / 32;                                               // 512 x 16 words (IQ3_S)
    float* xscale = reinterpret_cast<float*>(lut + (L.lut ? 8192 : 0));
    int8_t* xsplit = reinterpret_cast<int8_t*>(xscale + ((L.scales + 3) & ~3));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gid = lane >> 2, tig = lane & 3;
    const bool withhold = g_mv8_withhold == 1;
    if (smem_addr(sm) & 127u) return;  // a tiled copy's destination is 128-byte aligned (the launch gives that)
    const int team = L.team, teams = kM8Warps / team;
    const int tid_team = warp / team, kq = warp % team;
    const int nteams = gridDim.x * teams;
    const int q0 = tid_team * gridDim.x + blockIdx.x;
    const int my_jobs = q0 < L.jobs ? min((L.jobs - q0 + nteams - 1) / nteams, kM8MaxWarpJobs) : 0;
    uint8_t* my_ring = ring + size_t(warp) * ns * slot_bytes;
    uint64_t* my_bars = bars + warp * kM8MaxSlots;
    // the route's scratch (has_route): partial sums [2 rows][4 quarters][tokens], the launch number as read at
    // the start, whether this CTA arrived last
    float* rpart = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xsplit) + L.xbytes);
    uint32_t* rseq = reinterpret_cast<uint32_t*>(rpart + 2 * 4 * kRtTokens);
    uint32_t* rlast = rseq + 1;

    // barriers and the codebook are set up while the kernel before this one finishes; the route CTAs' warps
    // 0..7 load their router rows' first chunks (weights: no kernel writes them)
    if (lane == 0) {
        for (int i = 0; i < ns; ++i) tc::mbar_init(&my_bars[i], 1);
        tc::fence_barrier_init();
    }
    for (int i = threadIdx.x; i < kM8MaxRows / 32; i += kM8Threads) need[i] = 0u;
    const M8Route& R = L.r;
    const int64_t rrows = L.has_route ? R.experts + (R.gw != nullptr ? 1 : 0) : 0;
    const int64_t rrow = int64_t(blockIdx.x) * 2 + (warp >> 2);
    const bool rt_warp = L.has_route && warp < 8;
    const bool rt_live = rt_warp && rrow < rrows;
    const __half* rrow_ptr = rrow < R.experts ? R.w + rrow * R.hidden : R.gw;
    float rwv[4][8];
    if (rt_live) router_first(rrow_ptr, true, R.hidden, rwv);
    // (read before this CTA arrives below, so before the launch's last CTA moves it on)
    if (L.has_route && threadIdx.x == 0) *rseq = ld_relaxed_u32(R.counters + 1);
    if (L.lut) m8_fill_grid(lut);

    // lane l's job: problem, pair, tile (residue class and block), activation row; then its expert and the
    // first row of its TMA box, once the indices may be read
    int j_prob = 0, j_pair = 0, j_cls = 0, j_blk = 0, j_xr = 0, j_y = 0, j_valid = 0;
    const bool has = lane < my_jobs;
    if (has) {
        const int j = q0 + lane * nteams;
#pragma unroll
        for (int pr = 1; pr < kM8MaxProbs; ++pr)
            if (pr < L.nprob && j >= L.p[pr].job0) j_prob = pr;
        const M8Prob& P = L.p[j_prob];
        const int rest = j - P.job0;
        j_pair = rest / P.tiles;
        const int tile = rest - j_pair * P.tiles;
        j_cls = tile & (P.q - 1);
        j_blk = tile >> P.lq;
        j_xr = L.x[P.xs].row0 + j_pair / P.share;
    }
    auto place = [&](bool now) {  // the expert of lane l's job, for the jobs whose indices may be read now
        if (has && now) {
            const M8Prob& P = L.p[j_prob];
            const uint32_t e = P.wait ? __ldcg(P.idx + j_pair) : __ldg(P.idx + j_pair);
            j_valid = e < P.experts ? 1 : 0;
            j_y = static_cast<int>((int64_t(j_valid ? e : 0) * P.rows) >> P.lq) + 16 * j_blk;
        }
    };
    place(has && L.p[j_prob].early);
    // the activation rows this CTA's jobs read (not those of pairs already known to name no expert)
    if (has && (!L.p[j_prob].early || j_valid)) atomicOr(&need[j_xr >> 5], 1u << (j_xr & 31));
    __syncthreads();

    // the copy cursor (warp-uniform): the next item's job, its stage index k of n, slot, byte position in the
    // row, box row; lane 0 issues
    int i_job = 0, i_k = 0, i_n = 0, i_slot = 0, i_pos = 0, i_step = 0, i_y = 0, i_map = 0, i_valid = 0, i_bytes = 0;
    int issued = 0;
    auto stages_of = [&](int prob) {
        const int S = L.p[prob].stages;
        return S > kq ? (S - kq + team - 1) / team : 0;
    };
    // move the cursor to job `job` or the first after it with a stage for this warp
    auto seek = [&](int job) {
        for (i_job = job; i_job < my_jobs; ++i_job) {
            const int pr = __shfl_sync(0xffffffffu, j_prob, i_job);
            i_n = stages_of(pr);
            if (i_n == 0) continue;
            const M8Prob& P = L.p[pr];
            i_map = pr;
            i_k = 0;
            i_pos = __shfl_sync(0xffffffffu, j_cls, i_job) * static_cast<int>(P.row_bytes) + kq * P.stage_bytes;
            i_step = team * P.stage_bytes;
            i_y = __shfl_sync(0xffffffffu, j_y, i_job);
            i_valid = __shfl_sync(0xffffffffu, j_valid, i_job);
            i_bytes = 16 * P.rs;
            return;
        }
    };
    // issue the cursor's item (a pair naming no expert copies nothing and completes the slot's phase with a
    // plain arrive, so every item takes one phase) and move on; the weights are read once: evict-first in L2
    const uint64_t stream_policy = tc::policy_evict_first();
    auto issue = [&]() {
        if (lane == 0 && !(withhold && issued == 0)) {
            if (i_valid) {
                tc::mbar_arrive_expect_tx(&my_bars[i_slot], static_cast<uint32_t>(i_bytes));
                tc::tma_load_2d_hint(smem_addr(my_ring + i_slot * slot_bytes), &maps.w[i_map], (i_pos & ~15) >> 2,
                                     i_y, &my_bars[i_slot], stream_policy);
            } else {
                tc::mbar_arrive(&my_bars[i_slot]);
            }
        }
        ++issued;
        if (++i_slot == ns) i_slot = 0;
        i_pos += i_step;
        if (++i_k == i_n) seek(i_job + 1);
    };
    // the early problems' first copies go out before the wait; the cursor stops at a job whose indices wait
    seek(0);
    while (i_job < my_jobs && issued < ns - 1 && L.p[i_map].early) issue();

    // the activation blocks of the rows this CTA's jobs read, early sources first
    auto split = [&](bool early_pass) {
        for (int src = 0; src < L.nx; ++src) {
            const M8X& X = L.x[src];
            if ((X.early != 0) != early_pass) continue;
            const int xblocks = X.cols / kM8XBlock;
            for (int blk = warp; blk < X.rows * xblocks; blk += kM8Warps) {
                const int xr = blk / xblocks, b = blk - xr * xblocks;
                const int grow = X.row0 + xr;
                if (!((need[grow >> 5] >> (grow & 31)) & 1u)) continue;
                const int64_t at = int64_t(xr) * X.cols + int64_t(b) * kM8XBlock + 8 * lane;
                int8_t* hi = xsplit + X.byte0 + at;
                m8_split(X.x, X.gate, X.up, at, hi, hi + int64_t(X.rows) * X.cols, xscale + X.scale0 + blk, lane);
            }
        }
    };
    split(true);
    pdl_wait();
    // the route: a route CTA's two router rows (four warps to a row, as smoe_route computes them) into the
    // logits; then every CTA arrives (thread 0), and the last one in takes the top-k below
    if (rt_warp) {
        if (blockIdx.x < L.route_ctas) {
            float acc[kRtTokens];
            router_rows(rrow_ptr, rt_live, R.x, R.hidden, 0, R.tokens, acc, rwv);
#pragma unroll
            for (int t = 0; t < kRtTokens; ++t) acc[t] = warp_sum(acc[t]);
            if (lane == 0) {
#pragma unroll
                for (int t = 0; t < kRtTokens; ++t) rpart[((warp >> 2) * 4 + (warp & 3)) * kRtTokens + t] = acc[t];
            }
            route_sync();
            if (threadIdx.x < 2 * kRtTokens) {
                const int r = threadIdx.x / kRtTokens, t = threadIdx.x % kRtTokens;
                const int64_t er = int64_t(blockIdx.x) * 2 + r;
                if (er < rrows && t < R.tokens) {
                    float sum = rpart[(r * 4 + 0) * kRtTokens + t];
                    sum += rpart[(r * 4 + 1) * kRtTokens + t];
                    sum += rpart[(r * 4 + 2) * kRtTokens + t];
                    sum += rpart[(r * 4 + 3) * kRtTokens + t];
                    if (er < R.experts) R.logits[int64_t(t) * R.experts + er] = sum;
                    else R.gate_out[t] = __float2half_rn(sum);
                }
            }
        }
        __threadfence();
        route_sync();
        if (threadIdx.x == 0) *rlast = atomicAdd(R.counters, 1u) == gridDim.x - 1 ? 1u : 0u;
        route_sync();
    }
    place(has && !L.p[j_prob].early && !L.p[j_prob].wait);
    if (i_job < my_jobs && !L.p[i_map].early && !L.p[i_map].wait) seek(i_job);  // (its expert is known now)
    split(false);
    __syncthreads();
    while (i_job < my_jobs && issued < ns - 1 && (!L.has_route || !L.p[i_map].wait)) issue();
    // the last CTA in: one warp a token takes its top-k and softmax over the logits all CTAs wrote, then the
    // launch number moves on (release: idx, weights, lidx and gate_out are written)
    const uint32_t seq0 = L.has_route ? *rseq : 0u;
    if (rt_warp && *rlast && warp < R.tokens) {
        __threadfence();
        const float* in = R.logits + int64_t(warp) * R.experts;
        topk_row<8>([&](int j) { return __ldcg(in + j); }, R.experts, R.k, R.idx + int64_t(warp) * R.k,
                    R.weights + int64_t(warp) * R.k);
        if (R.lidx != nullptr) {
            __syncwarp();
            for (int j = lane; j < R.k; j += 32) {
                const uint32_t e = R.idx[int64_t(warp) * R.k + j] - R.lo;
                R.lidx[int64_t(warp) * R.k + j] = e < R.count ? e : R.count;
            }
        }
        __threadfence();
        asm volatile("bar.sync 14, %0;" ::"r"(32 * R.tokens) : "memory");
        if (threadIdx.x == 0) {
            R.counters[0] = 0u;
            __threadfence();
            if (g_mv8_withhold != 2) st_release_u32(R.counters + 1, seq0 + 1u);  // (2: a test withholds it)
        }
    }

    // a team of one warp needs no named barrier (there are 16, barrier 0 is __syncthreads')
    auto team_sync = [&]() {
        if (team == 1) __syncwarp();
        else asm volatile("bar.sync %0, %1;\n" ::"r"(1 + tid_team), "r"(32 * team) : "memory");
    };
    // a wait that gives up (it should not) leaves the warp's remaining stages undone but keeps it in step
    // with its team's barriers
    bool ok = true;
    const uint32_t polls = g_mv8_polls;
    float total[2] = {0.f, 0.f};
    int slot = 0, waited = 0;
    uint32_t phase = 0;
    // the route's indices: the copy cursor stops at the first job of a problem that reads them until the
    // launch number has moved on (lane 0 reads it a stage ahead of looking at it, and waits for it, bounded,
    // only when the item the warp is to decode next has not been issued)
    bool rdy = !L.has_route;
    uint32_t fpoll = seq0;
    int consumed = 0;
    auto route_in = [&]() {  // the number has moved: the routed jobs' places, the cursor's (at a job's start)
        fence_acq_rel_gpu();
        place(has && L.p[j_prob].wait);
        if (i_job < my_jobs) seek(i_job);
        rdy = true;
    };
    auto route_wait = [&]() -> bool {
        bool got = true;
        if (lane == 0) {
            uint32_t v = fpoll;
            if (v == seq0) {
                const uint64_t t0 = tc::globaltimer_ns();
                for (uint32_t i = 0;; ++i) {
                    v = ld_relaxed_u32(R.counters + 1);
                    if (v != seq0) break;
                    if (i >= polls || tc::globaltimer_ns() - t0 > tc::kWaitNs) {
                        got = false;
                        break;
                    }
                }
            }
            fpoll = v;
        }
        got = __shfl_sync(0xffffffffu, got ? 1 : 0, 0) != 0;
        if (got) route_in();
        else mv8_gave_up(lane);
        return got;
    };
    for (int job = 0; job < my_jobs; ++job) {
        const int pr = __shfl_sync(0xffffffffu, j_prob, job);
        const int pair = __shfl_sync(0xffffffffu, j_pair, job);
        const int cls = __shfl_sync(0xffffffffu, j_cls, job);
        const int blk = __shfl_sync(0xffffffffu, j_blk, job);
        const int xr = __shfl_sync(0xffffffffu, j_xr, job);
        int valid = __shfl_sync(0xffffffffu, j_valid, job);
        const M8Prob& P = L.p[pr];
        const M8X& X = L.x[P.xs];
        const int lx = xr - X.row0;
        const uint8_t* xh = reinterpret_cast<const uint8_t*>(xsplit) + X.byte0 + int64_t(lx) * X.cols;
        const uint8_t* xl = xh + int64_t(X.rows) * X.cols;
        const float* xsc = xscale + X.scale0 + lx * (X.cols / kM8XBlock);
        const int n = stages_of(pr);
        const bool iq3 = P.kind == M8IQ3S<2>::kKind;
        int pos = cls * static_cast<int>(P.row_bytes) + kq * P.stage_bytes;
        const int step = team * P.stage_bytes;
        int xc = kq * P.stage_cols;
        const int xstep = team * P.stage_cols;
        for (int k = 0; k < n; ++k, pos += step, xc += xstep) {
            // keep ns - 1 copies ahead; the slot refilled is the one this warp finished last
            __syncwarp();
            if (!rdy && ok && i_job < my_jobs && L.p[i_map].wait) {
                if (__shfl_sync(0xffffffffu, fpoll != seq0 ? 1 : 0, 0)) route_in();
                else if (lane == 0) fpoll = ld_relaxed_u32(R.counters + 1);
            }
            if (ok && i_job < my_jobs && (rdy || !L.p[i_map].wait)) issue();  // (after a wait gave up, nothing)
            if (ok && issued == consumed) {  // this item waits for the route
                ok = route_wait();
                if (ok) issue();
            }
            if (!rdy || k == 0) valid = __shfl_sync(0xffffffffu, j_valid, job);  // (placed once the route is in)
            ++consumed;
            const int cur = slot;
            if (ok) {
                ok = __all_sync(0xffffffffu, tc::mbar_wait(&my_bars[cur], phase, polls));
                if (ok) ++waited;
                else mv8_gave_up(lane);
            }
            if (++slot == ns) {
                slot = 0;
                phase ^= 1;
            }
            if (!ok || !valid) continue;
            const uint8_t* st = my_ring + cur * slot_bytes + (pos & 15);
            if (iq3)
                M8IQ3S<2>::stage(st + gid * M8IQ3S<2>::kRS, st + (gid + 8) * M8IQ3S<2>::kRS, tig, gid, lut, xh + xc,
                                 xl + xc, xsc + xc / kM8XBlock, total);
            else
                M8Q8_0::stage(st + gid * M8Q8_0::kRS, st + (gid + 8) * M8Q8_0::kRS, tig, gid, lut, xh + xc, xl + xc,
                              xsc + xc / kM8XBlock, total);
        }
        // the team's partial sums of this job's 16 rows, added in warp order
        float* rq = red + (tid_team * team) * 16;
        if (tig == 0) {
            rq[kq * 16 + gid] = total[0];
            rq[kq * 16 + gid + 8] = total[1];
        }
        total[0] = total[1] = 0.f;
        team_sync();
        if (kq == 0 && lane < 16) {
            const int64_t row = int64_t(blk) * 16 * P.q + cls + int64_t(P.q) * lane;
            if (valid && row < P.rows) {
                float v = rq[lane];
                for (int i = 1; i < team; ++i) v += rq[16 * i + lane];
                P.out[int64_t(pair) * P.rows + row] = __float2half_rn(v);
            }
        }
        team_sync();
    }
    // this CTA's slice of every expert the later launches read, into L2 (evict-last), once its own weights
    // are in (the launch's tail leaves HBM idle)
    if (warp == 0) {
        const uint64_t keep = tc::policy_evict_last();
        for (int f = 0; f < L.npf; ++f) {
            const M8Pref& Pf = L.pf[f];
            const int64_t eb = Pf.expert_bytes;
            const int64_t s0 = (int64_t(blockIdx.x) * eb / gridDim.x) & ~int64_t(15);
            const int64_t s1 = (int64_t(blockIdx.x + 1) * eb / gridDim.x) & ~int64_t(15);
            for (int i = lane; i < Pf.pairs; i += 32) {
                const uint32_t e = __ldcg(Pf.idx + i);  // (the launch's own route may have written it)
                if (e >= Pf.experts) continue;
                const uint8_t* base = Pf.blocks + int64_t(e) * eb;
                for (int64_t o = s0; o < s1; o += 65536)
                    tc::prefetch_l2_bulk(base + o, static_cast<uint32_t>(min(int64_t(65536), s1 - o)), keep);
            }
        }
    }
    // the next kernel may start placing its CTAs (releasing right after the wait instead measured slower: the
    // waiting CTAs of the next kernel crowd the running ones)
    pdl_release();
    // no copy may still be writing this CTA's shared memory when it exits: every item was waited for, unless a
    // wait gave up; then the items from the one it gave up on are waited for here with the full bound (no item
    // was issued after it)
    if (!ok && lane == 0)
        for (int i = withhold ? max(waited, 1) : waited; i < issued; ++i)
            tc::mbar_wait(&my_bars[i % ns], (i / ns) & 1, kM8WaitLimit);
    __syncwarp();
}

typedef CUresult (*M8EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                               const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                               CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static M8EncodeFn m8_encoder() {
    static std::once_flag once;
    static M8EncodeFn fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<M8EncodeFn>(p);
    });
    return fn;
}

static int g_m8_sms = 0;

// Launch the int8 tensor-core decode matvec when it takes the problem: 0 launched, 1 not taken, else an error.
// x, or (gate, up) whose SwiGLU is the activations.
int mv8s_try(int kind0, int kind1, const uint8_t* b0, const uint8_t* b1, int64_t experts, int64_t rows, int64_t cols,
            int64_t row_bytes, const uint32_t* idx, int64_t pairs, int64_t share, const __half* x, const __half* gate,
            const __half* up, __half* o0, __half* o1, int nprob, cudaStream_t st, const __half* cy = nullptr,
            const float* cw = nullptr, const __half* cg = nullptr, int ck = 0) {
    if (kind0 != kind1) return 1;
    auto go = [&](auto dec) -> int {
        using D = decltype(dec);
        if (cols % kM8XBlock || cols % D::kStageCols) return 1;
        if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(gate) & 15) ||
            (reinterpret_cast<uintptr_t>(up) & 15) || (reinterpret_cast<uintptr_t>(b0) & 15) ||
            (reinterpret_cast<uintptr_t>(b1) & 15) || (gate != nullptr) != (up != nullptr) ||
            (gate == nullptr) == (x == nullptr))
            return 1;
        int gcd = 16;
        while (row_bytes % gcd) gcd >>= 1;
        const int q = 16 / gcd;
        if (rows % q) return 1;
        const int64_t xrows = (pairs + share - 1) / share;
        const int xblocks = static_cast<int>(cols / kM8XBlock);
        // tokens a job takes: a one-expert stack's tokens (an activation row each) up to four a pass
        const int tok = D::kTokens && experts == 1 && share == 1 && pairs > 1 ? 4 : 1;
        // the activation rows a CTA holds: all of them when they fit beside two ring slots (one launch);
        // else, with one problem, only the CTA's own: CTA b's jobs [b J / G, (b + 1) J / G) are consecutive, so
        // their rows are those from its first job's to its last job's (two problems hold all: the callers then
        // split the pairs over launches). (Holding the window where all rows fit measured slower at decode.)
        const size_t slot = size_t(kM8Warps) * 16 * D::kRS;
        const size_t base = size_t(kM8Warps) * kM8MaxSlots * 8 + kM8Warps * 64 * 4 + kM8WhereSBytes +
                            (D::kLut ? 8192 * 4 : 0);
        const auto xbytes_of = [&](int64_t r) {
            return size_t(((r * xblocks + 3) & ~int64_t(3)) * 4) + size_t(r * cols * 2) +
                   (D::kXsum ? size_t(r * (cols / 16) * 4) : 0);
        };
        if (g_m8_sms == 0) {
            int dev = 0;
            cudaGetDevice(&dev);
            cudaDeviceGetAttribute(&g_m8_sms, cudaDevAttrMultiProcessorCount, dev);
            if (g_m8_sms <= 0) g_m8_sms = 148;
        }
        const int64_t ntiles = (rows + 16 * q - 1) / (16 * q) * q;
        const int64_t njobs = int64_t(nprob) * ((pairs + tok - 1) / tok) * ntiles;
        int64_t xwin = xrows;
        if (nprob == 1 && njobs > 0 && base + xbytes_of(xrows) + 2 * slot > size_t(227 * 1024)) {
            const int64_t G = std::min<int64_t>(g_m8_sms, njobs);
            xwin = 0;
            for (int64_t b = 0; b < G; ++b) {
                const int64_t c0 = b * njobs / G, c1 = (b + 1) * njobs / G;
                if (c0 >= c1) continue;
                const int64_t u0 = c0 / ntiles, u1 = (c1 - 1) / ntiles;
                const int64_t lo = tok == 1 ? u0 / share : u0 * tok;
                const int64_t hi = tok == 1 ? u1 / share : std::min(u1 * tok + tok - 1, xrows - 1);
                xwin = std::max(xwin, hi - lo + 1);
            }
            xwin = std::min(std::max<int64_t>(xwin, 1), xrows);
        }
        const size_t fixed = base + xbytes_of(xwin);
        int ns = kM8MaxSlots;
        while (ns > 2 && fixed + ns * slot > size_t(227 * 1024)) --ns;
        if (fixed + ns * slot > size_t(227 * 1024)) return 1;
        M8EncodeFn encode = m8_encoder();
        if (!encode) return 1;
        M8Maps2 maps;
        const uint8_t* bl[2] = {b0, b1};
        for (int p = 0; p < 2; ++p) {
            const cuuint64_t dims[2] = {static_cast<cuuint64_t>(q * row_bytes / 4),
                                        static_cast<cuuint64_t>(experts * rows / q)};
            const cuuint64_t strides[1] = {static_cast<cuuint64_t>(q * row_bytes)};
            const cuuint32_t box[2] = {static_cast<cuuint32_t>(D::kRS / 4), 16};
            const cuuint32_t estr[2] = {1, 1};
            if (encode(&maps.w[p], CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint8_t*>(bl[p]), dims, strides, box,
                       estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
                return 1;
        }
        M8Args a{};
        a.idx = idx;
        a.x = x;
        a.gate = gate;
        a.up = up;
        a.out[0] = o0;
        a.out[1] = o1;
        a.experts = experts;
        a.rows = rows;
        a.cols = cols;
        a.row_bytes = row_bytes;
        a.pairs = pairs;
        a.share = share;
        a.q = q;
        a.lq = q == 1 ? 0 : q == 2 ? 1 : q == 4 ? 2 : q == 8 ? 3 : 4;
        a.tiles = static_cast<int>((rows + 16 * q - 1) / (16 * q)) * q;
        a.tok = tok;
        const int64_t jobs = int64_t(nprob) * ((pairs + a.tok - 1) / a.tok) * a.tiles;
        if (jobs > (int64_t(1) << 30) || xrows > (int64_t(1) << 20) || experts * rows / q >= (int64_t(1) << 31) ||
            q * row_bytes >= (int64_t(1) << 27))
            return 1;
        a.jobs = static_cast<int>(jobs);
        a.xrows = static_cast<int>(xrows);
        a.xwin = static_cast<int>(xwin);
        a.nslots = ns;
        a.cy = cy;
        a.cw = cw;
        a.cg = cg;
        a.ck = ck;
        if (g_m8_sms == 0) {
            int dev = 0;
            cudaGetDevice(&dev);
            cudaDeviceGetAttribute(&g_m8_sms, cudaDevAttrMultiProcessorCount, dev);
            if (g_m8_sms <= 0) g_m8_sms = 148;
        }
        // the team size with the least work on the busiest warp, in quarters of a stage: CTA b takes the jobs
        // [b J / G, (b + 1) J / G), its teams share them round-robin; a warp does its share of each job's
        // stages plus about 3/4 of a stage for the team's reduction when the team has more than one warp
        // A one-expert stack (a dense layer: a verify window's product) takes the team its shape gives one token,
        // whatever the window: a token's float32 sums are then grouped alike alone and in a window, so it gets
        // the same bits (the integer sums are exact either way).
        const int64_t S = cols / D::kStageCols;
        const int64_t G = std::min<int64_t>(g_m8_sms, jobs);
        const int64_t tjobs = experts == 1 ? int64_t(nprob) * a.tiles : jobs;
        const int64_t tG = std::min<int64_t>(g_m8_sms, tjobs);
        int team = 1;
        int64_t best = -1;
        for (int t = 1; t <= kM8Warps; t *= 2) {
            const int64_t teams = kM8Warps / t;
            const int64_t most = ((tjobs + tG - 1) / tG + teams - 1) / teams;  // jobs of the busiest team
            if (most > 32) continue;  // (a warp's job table holds 32)
            const int64_t span = most * (4 * ((S + t - 1) / t) + (t > 1 ? 3 : 0));
            if (best < 0 || span < best) {
                best = span;
                team = t;
            }
        }
        if (best < 0) return 1;
        if (((jobs + G - 1) / G + kM8Warps / team - 1) / (kM8Warps / team) > 32) return 1;  // (split by mv8_try)
        a.team = team;
        const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, G));
        const size_t smem = fixed + ns * slot;
        if (int s = max_smem(mv8s_kernel<D>, static_cast<int>(smem))) return fail(s, "matvec: shared memory limit");
        const size_t xb = size_t(xrows) * cols * sizeof(__half);
        a.early = (pdl_early(st, idx, size_t(pairs) * 4) ? 1 : 0) |
                  ((x ? pdl_early(st, x, xb) : pdl_early(st, gate, xb) && pdl_early(st, up, xb)) ? 2 : 0);
        Writes wr;
        wr.add(o0, size_t(pairs) * rows * sizeof(__half));
        if (nprob == 2 && o1 != o0) wr.add(o1, size_t(pairs) * rows * sizeof(__half));
        launch_pdl(wr, mv8s_kernel<D>, dim3(grid), dim3(kM8Threads), smem, st, a, maps);
        return launch_status("matvec (int8 tensor cores)");
    };
    if (kind0 == M8IQ3S<2>::kKind) return cols % M8IQ3S<2>::kStageCols ? go(M8IQ3S<1>{}) : go(M8IQ3S<2>{});
    if (kind0 == M8Q8_0::kKind) return go(M8Q8_0{});
    if (kind0 == M8Q2_0::kKind) return go(M8Q2_0{});
    if (kind0 == M8IQ4XS<2>::kKind) return cols % M8IQ4XS<2>::kStageCols ? go(M8IQ4XS<1>{}) : go(M8IQ4XS<2>{});
    if (kind0 == M8IQ3XXS<2>::kKind) return cols % M8IQ3XXS<2>::kStageCols ? go(M8IQ3XXS<1>{}) : go(M8IQ3XXS<2>{});
    // the K-types (Q2_K and Q3_K in stages of two blocks: widths of an odd number of 256 columns stay on the
    // CUDA cores for those two)
    if (kind0 == M8Q2K::kKind) return cols % 512 ? 1 : go(M8Q2K{});
    if (kind0 == M8Q3K::kKind) return cols % 512 ? 1 : go(M8Q3K{});
    if (kind0 == M8Q45K<false>::kKind) return go(M8Q45K<false>{});
    if (kind0 == M8Q45K<true>::kKind) return go(M8Q45K<true>{});
    if (kind0 == M8Q6K::kKind) return go(M8Q6K{});
    return 1;
}


// Launch several matvec problems as one int8 tensor-core kernel: 0 launched, 1 not taken (the caller runs
// them another way), else an error status. Problems with the same activation pointers share one source.
int mv8_batch(int n, const M8Spec* specs_in, cudaStream_t st, int npf, const M8Pref* pf, const M8Route* route) {
    if (n < 1 || n > kM8MaxProbs || npf < 0 || npf > kM8MaxPref) return 1;
    // with the route in this launch, a problem whose indices lie in its idx or lidx reads them once the route
    // is in: such problems go after the others (their jobs come last in every warp's list)
    auto overlaps = [](const uint32_t* a, int64_t na, const uint32_t* b, int64_t nb) {
        return b != nullptr && a < b + nb && b < a + na;
    };
    auto waits = [&](const M8Spec& sp) {
        if (route == nullptr) return false;
        const int64_t nk = int64_t(route->tokens) * route->k;
        return overlaps(sp.idx, sp.pairs, route->idx, nk) || overlaps(sp.idx, sp.pairs, route->lidx, nk);
    };
    // then in order of falling cost per job (bytes of a 16-row tile), so that the round-robin of jobs over
    // teams hands the big jobs out first
    M8Spec specs[kM8MaxProbs];
    for (int i = 0; i < n; ++i) specs[i] = specs_in[i];
    auto job_bytes = [](const M8Spec& sp) { return sp.row_bytes * 16; };
    auto before = [&](const M8Spec& a, const M8Spec& b) {
        return waits(a) != waits(b) ? !waits(a) : job_bytes(a) > job_bytes(b);
    };
    for (int i = 1; i < n; ++i)
        for (int j = i; j > 0 && before(specs[j], specs[j - 1]); --j) std::swap(specs[j], specs[j - 1]);
    if (route != nullptr) {
        const int64_t rows = int64_t(route->experts) + (route->gw != nullptr ? 1 : 0);
        if (route->tokens < 1 || route->tokens > kRtTokens || route->experts < 1 || route->experts > 256 ||
            route->k < 1 || route->k > std::min(route->experts, 32) || route->hidden < 8 || route->hidden % 8 ||
            !route->w || !route->x || !route->logits || !route->idx || !route->weights || !route->counters ||
            (reinterpret_cast<uintptr_t>(route->w) & 15) || (reinterpret_cast<uintptr_t>(route->gw) & 15) ||
            (reinterpret_cast<uintptr_t>(route->x) & 15) || (route->gw != nullptr) != (route->gate_out != nullptr) ||
            rows > 2 * 148)
            return 1;
    }
    M8EncodeFn encode = m8_encoder();
    if (!encode) return 1;
    M8Launch L{};
    M8Maps maps;
    int jobs = 0, rows = 0, scales = 0;
    int64_t xbytes = 0;
    bool lut = false;
    int max_rs = 0;
    for (int i = 0; i < n; ++i) {
        const M8Spec& sp = specs[i];
        int stage_cols, stage_bytes, rs;
        if (sp.kind == M8IQ3S<2>::kKind) {  // (widths of an odd number of 256 columns go problem by problem)
            stage_cols = M8IQ3S<2>::kStageCols, stage_bytes = M8IQ3S<2>::kStageBytes, rs = M8IQ3S<2>::kRS;
            lut = true;
        } else if (sp.kind == M8Q8_0::kKind) {
            stage_cols = M8Q8_0::kStageCols, stage_bytes = M8Q8_0::kStageBytes, rs = M8Q8_0::kRS;
        } else {
            return 1;
        }
        if (sp.cols % kM8XBlock || sp.cols % stage_cols || sp.pairs <= 0 || sp.share < 1) return 1;
        if ((reinterpret_cast<uintptr_t>(sp.x) & 15) || (reinterpret_cast<uintptr_t>(sp.gate) & 15) ||
            (reinterpret_cast<uintptr_t>(sp.up) & 15) || (reinterpret_cast<uintptr_t>(sp.blocks) & 15) ||
            (sp.gate != nullptr) != (sp.up != nullptr) || (sp.gate == nullptr) == (sp.x == nullptr))
            return 1;
        int gcd = 16;
        while (sp.row_bytes % gcd) gcd >>= 1;
        const int q = 16 / gcd;
        if (sp.rows % q || sp.experts * sp.rows / q >= (int64_t(1) << 31) || q * sp.row_bytes >= (int64_t(1) << 27))
            return 1;
        // the activation source: an earlier problem's if it names the same activations
        int xs = -1;
        for (int j = 0; j < L.nx; ++j)
            if (L.x[j].x == sp.x && L.x[j].gate == sp.gate && L.x[j].up == sp.up && L.x[j].cols == sp.cols)
                xs = j;
        const int64_t xrows = (sp.pairs + sp.share - 1) / sp.share;
        if (xs < 0) {
            if (L.nx == kM8MaxX) return 1;
            xs = L.nx++;
            M8X& X = L.x[xs];
            X.x = sp.x;
            X.gate = sp.gate;
            X.up = sp.up;
            X.rows = static_cast<int>(xrows);
            X.cols = static_cast<int>(sp.cols);
            X.row0 = rows;
            X.scale0 = scales;
            X.byte0 = xbytes;
            const size_t xb = size_t(xrows) * sp.cols * sizeof(__half);
            X.early = (sp.x ? pdl_early(st, sp.x, xb) : pdl_early(st, sp.gate, xb) && pdl_early(st, sp.up, xb)) ? 1 : 0;
            rows += X.rows;
            scales += X.rows * static_cast<int>(sp.cols / kM8XBlock);
            xbytes += 2 * xrows * sp.cols;
        } else if (L.x[xs].rows < xrows) {
            return 1;
        }
        M8Prob& P = L.p[i];
        P.idx = sp.idx;
        P.out = sp.out;
        P.rows = sp.rows;
        P.row_bytes = sp.row_bytes;
        P.experts = static_cast<uint32_t>(sp.experts);
        P.kind = sp.kind;
        P.stage_cols = stage_cols;
        P.stage_bytes = stage_bytes;
        P.rs = rs;
        P.q = q;
        P.lq = q == 1 ? 0 : q == 2 ? 1 : q == 4 ? 2 : q == 8 ? 3 : 4;
        P.tiles = static_cast<int>((sp.rows + 16 * q - 1) / (16 * q)) * q;
        P.stages = static_cast<int>(sp.cols / stage_cols);
        P.pairs = static_cast<int>(sp.pairs);
        P.share = static_cast<int>(sp.share);
        P.xs = xs;
        P.wait = waits(sp) ? 1 : 0;
        P.early = !P.wait && pdl_early(st, sp.idx, size_t(sp.pairs) * 4) ? 1 : 0;
        P.job0 = jobs;
        const int64_t pj = int64_t(P.pairs) * P.tiles;
        if (pj + jobs > (int64_t(1) << 30)) return 1;
        P.jobs = static_cast<int>(pj);
        jobs += P.jobs;
        max_rs = std::max(max_rs, rs);
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(q * sp.row_bytes / 4),
                                    static_cast<cuuint64_t>(sp.experts * sp.rows / q)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(q * sp.row_bytes)};
        const cuuint32_t box[2] = {static_cast<cuuint32_t>(rs / 4), 16};
        const cuuint32_t estr[2] = {1, 1};
        if (encode(&maps.w[i], CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint8_t*>(sp.blocks), dims, strides, box,
                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return 1;
    }
    if (rows > kM8MaxRows) return 1;
    L.nprob = n;
    L.npf = 0;
    for (int i = 0; i < npf; ++i)
        if (pf[i].blocks && pf[i].idx && pf[i].pairs > 0 && pf[i].expert_bytes % 16 == 0 &&
            (reinterpret_cast<uintptr_t>(pf[i].blocks) & 15) == 0)
            L.pf[L.npf++] = pf[i];
    L.jobs = jobs;
    L.scales = scales;
    L.xbytes = xbytes;
    L.lut = lut ? 1 : 0;
    L.slot_bytes = 16 * max_rs;
    const size_t fixed = size_t(kM8Warps) * kM8MaxSlots * 8 + kM8Warps * 16 * 4 + kM8MaxRows / 8 +
                         (lut ? 8192 * 4 : 0) + size_t((scales + 3) & ~3) * 4 + size_t(xbytes) +
                         (route ? kM8RouteBytes : 0);
    const size_t slot = size_t(kM8Warps) * L.slot_bytes;
    int ns = kM8MaxSlots;
    while (ns > 2 && fixed + ns * slot > size_t(227 * 1024)) --ns;
    if (fixed + ns * slot > size_t(227 * 1024)) return 1;
    L.nslots = ns;
    if (g_m8_sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_m8_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_m8_sms <= 0) g_m8_sms = 148;
    }
    // the team size with the least work on the busiest warp: jobs go round-robin over all teams (CTA-fastest)
    // in problem order; a warp's share of a job is its stages' bytes, plus about 3/4 of a stage for the team's
    // reduction when the team has more than one warp
    const int64_t G = std::min<int64_t>(g_m8_sms, jobs);
    int team = 1;
    int64_t best = -1;
    std::vector<int64_t> load;
    for (int t = 1; t <= kM8Warps; t *= 2) {
        const int64_t nteams = G * (kM8Warps / t);
        load.assign(static_cast<size_t>(std::min<int64_t>(nteams, jobs)), 0);
        int64_t j = 0;
        for (int i = 0; i < n; ++i) {
            const M8Prob& P = L.p[i];
            const int64_t sb = int64_t(16) * P.stage_bytes;
            const int64_t w = (P.stages + t - 1) / t * sb * 4 + (t > 1 ? 3 * sb : 0);
            for (int64_t k = 0; k < P.jobs; ++k, ++j) load[static_cast<size_t>(j % nteams)] += w;
        }
        const int64_t span = *std::max_element(load.begin(), load.end());
        if (best < 0 || span < best) {
            best = span;
            team = t;
        }
    }
    L.team = team;
    // a warp keeps at most 32 jobs (one per lane of its job table)
    if (jobs > int64_t(kM8MaxWarpJobs) * G * (kM8Warps / team)) return 1;
    const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, G));
    const size_t smem = fixed + ns * slot;
    if (int s = max_smem(mv8_kernel, static_cast<int>(smem))) return fail(s, "matvec: shared memory limit");
    if (route != nullptr) {
        // a CTA for every two router rows, all in the grid (one CTA an SM: all are running at once)
        L.has_route = 1;
        L.r = *route;
        L.route_ctas = (route->experts + (route->gw != nullptr ? 1 : 0) + 1) / 2;
        if (L.route_ctas > static_cast<int>(grid)) return 1;
    }
    Writes wr;
    for (int i = 0; i < n; ++i) wr.add(L.p[i].out, size_t(L.p[i].pairs) * L.p[i].rows * sizeof(__half));
    if (route != nullptr) {
        const size_t tk = size_t(route->tokens) * route->k * 4;
        wr.add(route->logits, size_t(route->tokens) * route->experts * 4).add(route->idx, tk).add(route->weights, tk);
        wr.add(route->gate_out, size_t(route->tokens) * sizeof(__half)).add(route->counters, 8).add(route->lidx, tk);
    }
    launch_pdl(wr, mv8_kernel, dim3(grid), dim3(kM8Threads), smem, st, L, maps);
    return launch_status("matvec (int8 tensor cores)");
}

// The shared expert's down product (one expert, pair t = token t) with the block's combine as its epilogue.
int mv8_glu_combine(int kind, const uint8_t* blocks, int64_t rows, int64_t cols, int64_t row_bytes,
                    const uint32_t* idx, int64_t tokens, const __half* gate, const __half* up, const __half* y,
                    const float* w, const __half* g, int k, __half* out, cudaStream_t st) {
    return mv8s_try(kind, kind, blocks, blocks, 1, rows, cols, row_bytes, idx, tokens, 1, nullptr, gate, up, out, out, 1,
                    st, y, w, g, k);
}

// One or two problems (gate and up) of the existing entry points: the single-stack kernel. Pairs whose
// activations do not fit one launch's shared memory (or its warps' job tables) go in equal launches of a
// multiple of `share` pairs each; every pair's result is the one a single launch would give.
int mv8_try(int kind0, int kind1, const uint8_t* b0, const uint8_t* b1, int64_t experts, int64_t rows, int64_t cols,
            int64_t row_bytes, const uint32_t* idx, int64_t pairs, int64_t share, const __half* x, const __half* gate,
            const __half* up, __half* o0, __half* o1, int nprob, cudaStream_t st) {
    const auto part = [&](int64_t p0, int64_t n) {
        const int64_t x0 = p0 / share * cols;
        return mv8s_try(kind0, kind1, b0, b1, experts, rows, cols, row_bytes, idx + p0, n, share, x ? x + x0 : nullptr,
                        gate ? gate + p0 * cols : nullptr, up ? up + p0 * cols : nullptr, o0 + p0 * rows,
                        o1 + p0 * rows, nprob, st);
    };
    int r = part(0, pairs);
    if (r != 1 || share < 1 || pairs <= share || pairs % share) return r;
    for (int64_t parts = 2; parts <= 64; parts *= 2) {
        const int64_t n = ((pairs / share + parts - 1) / parts) * share;  // pairs a launch
        if (n >= pairs) continue;
        r = part(0, n);
        if (r == 1) continue;
        if (r != 0) return r;
        for (int64_t p0 = n; p0 < pairs; p0 += n) {
            r = part(p0, std::min(n, pairs - p0));
            if (r == 1) return fail(SMOE_ESHAPE, "matvec: a part of the pairs was not taken");
            if (r != 0) return r;
        }
        return 0;
    }
    return 1;
}

}  // namespace smoe

using namespace smoe;

extern "C" int smoe_matvec_status(int* status, int clear) {
    SMOE_REQUIRE(status, SMOE_EARG, "matvec_status: null pointer");
    int v = 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, g_mv8_status, sizeof(int));
    if (e == cudaSuccess && clear) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_mv8_status, &zero, sizeof(int));
    }
    if (e != cudaSuccess) return fail(-static_cast<int>(e), std::string("matvec_status: ") + cudaGetErrorString(e));
    *status = v;
    return SMOE_OK;
}

extern "C" int smoe_matvec_wait_test(int64_t polls, int withhold) {
    const uint32_t v = polls < 0 ? kM8WaitLimit : static_cast<uint32_t>(std::min<int64_t>(polls, kM8WaitLimit));
    const int w = withhold == 2 ? 2 : withhold ? 1 : 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_mv8_polls, &v, sizeof(v));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_mv8_withhold, &w, sizeof(w));
    if (e != cudaSuccess) return fail(-static_cast<int>(e), std::string("matvec_wait_test: ") + cudaGetErrorString(e));
    return SMOE_OK;
}
