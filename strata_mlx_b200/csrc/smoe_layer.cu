// The MoE block's decode step for one token in one persistent launch: the router with its top-k and the
// softmax over the chosen and the shared expert's gate, the routed experts' and the shared expert's gate / up
// products, their down products, and the block's combine -- the work of smoe_route, smoe_matvec_batch,
// smoe_matvec_glu and smoe_matvec_glu_combine, without the four launches' prologues and pipeline drains.
//
// B200 layout: one CTA of 16 warps per SM, all co-resident (a cooperative launch). The phases whose inputs are
// other CTAs' outputs are separated by grid barriers (an atomic counter in global memory, every wait bounded):
//   A  every CTA: its router rows' weights in flight, codebook, the token's int8 split, the shared expert's
//      first weight copies (they need no routing);
//   B  router rows -> logits (global), the shared gate row -> gate value;            barrier 1
//   C  every CTA takes the top-k of the logits itself (the same choice everywhere), so the routed experts'
//      copies start at once; CTA 0 writes idx and weights;
//   D  gate / up tiles of the four stacks (jobs round-robin over all teams, CTA-fastest, costliest first),
//      products to global;                                                          barrier 2
//   E  down tiles: the routed down on the first CTAs, the shared down on the rest (contiguous job ranges, so
//      a CTA splits one or two SwiGLU rows), products to global;                     barrier 3
//   F  the combine of every output row, by row ranges.
// Each warp's copy cursor runs through its phase-D items and on into its phase-E items: the down weights
// stream in while the gate / up products finish and while the CTAs wait at barrier 2. Stage decoders, the
// activation split and the combine are the matvec kernels' own (mv8_dev.cuh, common.cuh), so every product is
// the same integer arithmetic.
#include <algorithm>

#include "mv8_dev.cuh"
#include "router_dev.cuh"

namespace smoe {

constexpr int kLyRep = 8;        // copies of the IQ3_S grid (16 KB; the ring needs the rest)
constexpr int kLyMaxK = 32;      // routed experts a token takes
constexpr int kLyMaxExperts = 256;
constexpr int kLyTopkNV = kLyMaxExperts / 32;

// One stack of a phase: a job is a tile of 16 weight rows (one residue class mod q) of one pair.
struct LyStack {
    __half* out;             // [pairs][rows]
    int64_t rows, row_bytes;
    int kind;                // 21 IQ3_S (two-block stages) or 8 Q8_0
    int stage_cols, stage_bytes, rs, q, lq, tiles, stages;
    int routed;              // expert idx[pair] (pairs = k), or the one expert (pairs = 1)
    int pairs;
    int job0, jobs;          // its jobs within the phase
    int map;                 // its tensor map
    int src;                 // its activation source within the phase
};
// Activation rows of a phase, split into int8 hi / lo: the token (phase D) or swiglu(gate, up) rows (E).
struct LySource {
    const __half *x, *gate, *up;
    int rows, cols;          // rows: the token's 1, or the k routed pairs' (a CTA splits the ones it needs)
};
struct LyArgs {
    const __half* router;    // [experts][hidden]
    const __half* sgate;     // [hidden]
    const __half* x;         // [hidden]
    int experts, hidden, k;
    float* logits;
    uint32_t* idx;
    float* weights;
    __half* gate_out;
    __half* out;             // [hidden]
    __half *y, *s;           // routed down products [k][hidden], the shared down product [hidden]
    unsigned long long* bar; // grid barrier arrivals (never reset: launches count on from a multiple of 3 G)
    int* err;                // set when a wait gave up
    LyStack d[4];            // gate / up stacks, costliest first
    LyStack e[2];            // routed down, shared down
    LySource src_d, src_e[2];
    int nd, jobs_d;
    int nslots, slot_bytes, split_bytes;
};
struct alignas(64) LyMaps {
    CUtensorMap w[6];
};

__device__ __forceinline__ unsigned long long ld_acquire(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Every CTA arrives, then waits (thread 0, bounded) until all G have: `target` arrivals in all. Returns false
// when the wait gave up (the error flag is then set).
// A test hook (smoe_decode_layer_wait_test): CTA 0 does not arrive at the first barrier, so every wait there runs
// out (bounded) and the launch reports it.
static __device__ int g_ly_withhold = 0;

__device__ __forceinline__ bool grid_sync(unsigned long long* bar, unsigned long long target, int* err, int* flag,
                                          bool arrive = true) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (arrive) atomicAdd(bar, 1ull);
        bool ok = true;
        if (ld_acquire(bar) < target) {
            const uint64_t t0 = tc::globaltimer_ns();
            while (ld_acquire(bar) < target) {
                if (tc::globaltimer_ns() - t0 > tc::kWaitNs) {
                    ok = false;
                    atomicExch(err, 1);
                    break;
                }
            }
        }
        __threadfence();
        *flag = ok ? 1 : 0;
    }
    __syncthreads();
    return *flag != 0;
}

__device__ __forceinline__ uint4 ldcg16(const __half* p) { return __ldcg(reinterpret_cast<const uint4*>(p)); }

// m8_split for a SwiGLU row written by other CTAs before a barrier (read from L2)
__device__ __forceinline__ void ly_split_glu(const __half* gate, const __half* up, int64_t at, int8_t* hi, int8_t* lo,
                                             float* scale, int lane) {
    float v[8];
    const uint4 gr = ldcg16(gate + at), ur = ldcg16(up + at);
    const __half* gh = reinterpret_cast<const __half*>(&gr);
    const __half* uh = reinterpret_cast<const __half*>(&ur);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __half2float(swiglu_one(gh[i], uh[i]));
    m8_split_values(v, hi, lo, scale, lane);
}

// A CTA's jobs of a phase, each with a slot for its warps' partial sums (the host keeps every CTA within it)
constexpr int kLySlots = 17;

__global__ void __launch_bounds__(kM8Threads, 1) decode_layer_kernel(const __grid_constant__ LyArgs A,
                                                                     const __grid_constant__ LyMaps M) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int ns = A.nslots, slot_bytes = A.slot_bytes;
    uint8_t* ring = sm;                                                                    // [warp][slot]
    uint64_t* bars = reinterpret_cast<uint64_t*>(ring + size_t(kM8Warps) * ns * slot_bytes);  // [warp][slot]
    float* partial = reinterpret_cast<float*>(bars + kM8Warps * kM8MaxSlots);              // [job slot][warp][16]
    int* cnt = reinterpret_cast<int*>(partial + kLySlots * kM8Warps * 16);                 // [job slot] units in
    float* part = reinterpret_cast<float*>(cnt + 32);                                      // [4 rows][4 quarters]
    uint32_t* sidx = reinterpret_cast<uint32_t*>(part + 16);                               // [k]
    float* sw = reinterpret_cast<float*>(sidx + kLyMaxK);                                  // [k]
    int* flag = reinterpret_cast<int*>(sw + kLyMaxK);                                      // barrier result
    uint32_t* lut = reinterpret_cast<uint32_t*>(flag + 32);                                // 512 x kLyRep words
    float* xscale = reinterpret_cast<float*>(lut + 512 * kLyRep);                          // [64]
    int8_t* xsplit = reinterpret_cast<int8_t*>(xscale + 64);                               // split_bytes

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gid = lane >> 2, tig = lane & 3;
    if (smem_addr(sm) & 127u) return;  // a tiled copy's destination is 128-byte aligned (the launch gives that)
    const int G = gridDim.x, b = blockIdx.x;
    const int H = A.hidden, E = A.experts, K = A.k;

    // ---- A: the global loads first (router weights, the token's split block, the codebook), their uses later
    const int router_rows_n = E + (A.sgate != nullptr ? 1 : 0);
    const int my_row = b + G * (warp >> 2);
    const bool row_live = my_row < router_rows_n;
    const __half* row_ptr = my_row < E ? A.router + int64_t(my_row) * H : A.sgate;
    float wv[4][8], acc[kRtTokens];
    router_first(row_ptr, row_live, H, wv);
    const int xblocks_d = H / kM8XBlock;
    uint4 xr0 = make_uint4(0u, 0u, 0u, 0u);
    if (warp < xblocks_d) xr0 = *reinterpret_cast<const uint4*>(A.x + int64_t(warp) * kM8XBlock + 8 * lane);
    uint32_t g0 = 0u, g1 = 0u;
    const int li0 = threadIdx.x, li1 = threadIdx.x + kM8Threads;  // 1024 groups of 4 words: 512 x kLyRep / 4
    g0 = __ldg(kIq3sSigned + (4 * li0) / kLyRep);
    g1 = __ldg(kIq3sSigned + (4 * li1) / kLyRep);

    // the arrival count this launch starts from: a multiple of 3 G (early arrivals at barrier 1 are fewer
    // than G)
    __shared__ unsigned long long base_s;
    if (threadIdx.x == 0) {
        const unsigned long long v0 = ld_acquire(A.bar);
        base_s = v0 - v0 % (3ull * G);
    }
    if (lane == 0) {
        for (int i = 0; i < ns; ++i) tc::mbar_init(&bars[warp * kM8MaxSlots + i], 1);
        tc::fence_barrier_init();
    }
    if (threadIdx.x < kLySlots) cnt[threadIdx.x] = 0;
    for (int i = threadIdx.x; i < kLySlots * kM8Warps * 16; i += kM8Threads) partial[i] = 0.f;

    // ---- this CTA's jobs. A phase's jobs are of two stacks: the compute-heavy one (kind A: IQ3_S, SA stages a
    // job) and the bandwidth-heavy one (kind B: Q8_0, SB stages); lane i of every warp holds the CTA's job i
    // (its A jobs first, then its B jobs): meta = stack | cls << 2 | valid << 6 | pair << 7 | blk << 13, and y,
    // the first row of its TMA box. The CTA's units (stages) of both kinds are merged in proportion (unit p is
    // of kind A when floor((p + 1) NA / N) > floor(p NA / N)), so every SM decodes and streams at once, and
    // dealt round-robin to the 16 warps.
    auto job_meta = [&](const LyStack& S, int stack, int rest) {
        const int pair = rest / S.tiles, tile = rest - pair * S.tiles;
        return stack | ((tile & (S.q - 1)) << 2) | (pair << 7) | ((tile >> S.lq) << 13);
    };
    auto place = [&](const LyStack& S, int meta, uint32_t e, int& valid_meta) {
        const int ok = e < uint32_t(S.routed ? E : 1) ? 1 : 0;
        valid_meta = meta | (ok << 6);
        return static_cast<int>((int64_t(ok ? e : 0) * S.rows) >> S.lq) + 16 * (meta >> 13);
    };
    // phase D: the jobs of all four stacks round-robin over the CTAs; stacks 0, 1 (the shared expert, B) take
    // the first jobs, so a CTA's B jobs come first in its round-robin list: reorder to A first
    const int nj_d = b < A.jobs_d ? min((A.jobs_d - b + G - 1) / G, kLySlots) : 0;
    const int jb_d = b < A.d[2].job0 ? min((A.d[2].job0 - b + G - 1) / G, nj_d) : 0;  // B jobs of this CTA
    const int ja_d = nj_d - jb_d;
    int md = 0, yd = 0;
    if (lane < nj_d) {
        const int li = lane < ja_d ? jb_d + lane : lane - ja_d;  // round-robin index of lane's job
        const int j = b + li * G;
        int st = 0;
#pragma unroll
        for (int i = 1; i < 4; ++i)
            if (i < A.nd && j >= A.d[i].job0) st = i;
        md = job_meta(A.d[st], st, j - A.d[st].job0);
        if (!A.d[st].routed) yd = place(A.d[st], md, 0u, md);
    }
    const int sa_d = A.d[2].stages, sb_d = A.d[0].stages;
    // phase E: this CTA's tiles of one routed pair (the CTAs split the pairs evenly, then a pair's tiles), and
    // its share of the shared down's jobs
    const LyStack& ER = A.e[0];
    const LyStack& ES = A.e[1];
    const int npair = ER.pairs;
    const int epair = static_cast<int>(int64_t(b) * npair / G);
    const int pc0 = static_cast<int>((int64_t(epair) * G + npair - 1) / npair);
    const int pc1 = static_cast<int>((int64_t(epair + 1) * G + npair - 1) / npair);
    const int rt0 = static_cast<int>(int64_t(b - pc0) * ER.tiles / (pc1 - pc0));
    const int rt1 = static_cast<int>(int64_t(b - pc0 + 1) * ER.tiles / (pc1 - pc0));
    const int ja_e = min(rt1 - rt0, kLySlots);
    const int sj0 = static_cast<int>(int64_t(b) * ES.jobs / G), sj1 = static_cast<int>(int64_t(b + 1) * ES.jobs / G);
    const int jb_e = min(sj1 - sj0, kLySlots - ja_e);
    int me = 0, ye = 0;
    if (lane < ja_e) me = job_meta(ER, 0, epair * ER.tiles + rt0 + lane);
    else if (lane < ja_e + jb_e) me = job_meta(ES, 1, sj0 + lane - ja_e);
    const int sa_e = ER.stages, sb_e = ES.stages;

    // ---- the token's split and the codebook, now that their loads are in
    if (warp < xblocks_d) {
        const __half2* h2 = reinterpret_cast<const __half2*>(&xr0);
        float v[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(h2[i]);
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
        const int at = warp * kM8XBlock + 8 * lane;
        m8_split_values(v, xsplit + at, xsplit + A.split_bytes / 2 + at, xscale + warp, lane);
    }
    for (int blk = warp + kM8Warps; blk < xblocks_d; blk += kM8Warps) {  // (hidden above 4096)
        const int64_t at = int64_t(blk) * kM8XBlock + 8 * lane;
        m8_split(A.x, nullptr, nullptr, at, xsplit + at, xsplit + A.split_bytes / 2 + at, xscale + blk, lane);
    }
    reinterpret_cast<uint4*>(lut)[li0] = make_uint4(g0, g0, g0, g0);
    reinterpret_cast<uint4*>(lut)[li1] = make_uint4(g1, g1, g1, g1);
    __syncthreads();

    // ---- units: phase P's merged sequence of NA A units and NB B units; position p -> (job, stage)
    const int na_d = ja_d * sa_d, nb_d = jb_d * sb_d, n_d = na_d + nb_d;
    const int na_e = ja_e * sa_e, nb_e = jb_e * sb_e, n_e = na_e + nb_e;
    // A warp walks positions p = warp, warp + 16, ...: a = floor(p NA / N) A units lie before p, r the
    // remainder; p is an A unit when r + NA >= N. Jobs from unit indices by multiplying with 2^16 / stages
    // rounded up (exact below 2048 units).
    struct Unit {
        int job, stage, kind;  // job: the CTA's job index (its lane); kind 0 = A, 1 = B
    };
    struct UnitWalk {
        int p, a, r;
    };
    auto walk_start = [&](int P, int p0) {
        const int na = P == 0 ? na_d : na_e, n = P == 0 ? n_d : n_e;
        UnitWalk w;
        w.p = p0;
        w.a = n > 0 ? p0 * na / n : 0;
        w.r = n > 0 ? p0 * na - w.a * n : 0;
        return w;
    };
    const int q16_d = n_d > 0 ? kM8Warps * na_d / n_d : 0, r16_d = n_d > 0 ? kM8Warps * na_d - q16_d * n_d : 0;
    const int q16_e = n_e > 0 ? kM8Warps * na_e / n_e : 0, r16_e = n_e > 0 ? kM8Warps * na_e - q16_e * n_e : 0;
    const int ma_d = (65536 + sa_d - 1) / sa_d, mb_d = (65536 + sb_d - 1) / sb_d;
    const int ma_e = (65536 + sa_e - 1) / sa_e, mb_e = (65536 + sb_e - 1) / sb_e;
    auto walk_unit = [&](int P, const UnitWalk& w) {
        const int na = P == 0 ? na_d : na_e, n = P == 0 ? n_d : n_e;
        Unit u;
        if (w.r + na >= n) {
            const int sa = P == 0 ? sa_d : sa_e;
            u.kind = 0;
            u.job = (w.a * (P == 0 ? ma_d : ma_e)) >> 16;
            u.stage = w.a - u.job * sa;
        } else {
            const int sb = P == 0 ? sb_d : sb_e, ja = P == 0 ? ja_d : ja_e, q = w.p - w.a;
            const int jb = (q * (P == 0 ? mb_d : mb_e)) >> 16;
            u.kind = 1;
            u.job = ja + jb;
            u.stage = q - jb * sb;
        }
        return u;
    };
    auto walk_next = [&](int P, UnitWalk& w) {
        const int n = P == 0 ? n_d : n_e;
        w.p += kM8Warps;
        w.a += P == 0 ? q16_d : q16_e;
        w.r += P == 0 ? r16_d : r16_e;
        if (w.r >= n) {
            w.r -= n;
            ++w.a;
        }
    };

    // ---- the copy cursor over this warp's units: phase D's, then phase E's
    uint8_t* my_ring = ring + size_t(warp) * ns * slot_bytes;
    uint64_t* my_bars = bars + warp * kM8MaxSlots;
    int c_phase = 0, c_slot = 0, issued = 0;
    UnitWalk cw = walk_start(0, warp);
    auto c_norm = [&]() {  // to the next phase when this one is done
        if (c_phase == 0 && cw.p >= n_d) {
            c_phase = 1;
            cw = walk_start(1, warp);
        }
        if (c_phase == 1 && cw.p >= n_e) c_phase = 2;
    };
    c_norm();
    bool placed = false;
    auto cursor_ready = [&]() {  // the cursor's unit has its place (phase D's routed jobs wait for the choice)
        if (c_phase == 2) return false;
        if (placed) return true;
        if (c_phase == 1) return false;
        return walk_unit(0, cw).kind == 1;  // the shared expert's units need no routing
    };
    auto issue = [&]() {
        const Unit u = walk_unit(c_phase, cw);
        const int meta = __shfl_sync(0xffffffffu, c_phase == 0 ? md : me, u.job);
        const int y = __shfl_sync(0xffffffffu, c_phase == 0 ? yd : ye, u.job);
        const LyStack& S = c_phase == 0 ? A.d[meta & 3] : A.e[meta & 3];
        if (lane == 0) {
            if ((meta >> 6) & 1) {
                const int pos = ((meta >> 2) & 15) * static_cast<int>(S.row_bytes) + u.stage * S.stage_bytes;
                tc::mbar_arrive_expect_tx(&my_bars[c_slot], static_cast<uint32_t>(16 * S.rs));
                tc::tma_load_2d(smem_addr(my_ring + c_slot * slot_bytes), &M.w[S.map], (pos & ~15) >> 2, y,
                                &my_bars[c_slot]);
            } else {
                tc::mbar_arrive(&my_bars[c_slot]);
            }
        }
        ++issued;
        if (++c_slot == ns) c_slot = 0;
        walk_next(c_phase, cw);
        c_norm();
    };
    // the shared expert's first copies go out now (they need no routing)
    while (issued < ns - 1 && cursor_ready()) issue();

    // ---- B: router rows -> logits, the shared gate row -> the gate value
    if (row_live) {
        router_rows(row_ptr, true, A.x, H, 0, 1, acc, wv);
        acc[0] = warp_sum(acc[0]);
    } else {
        acc[0] = 0.f;
    }
    if (lane == 0) part[(warp >> 2) * 4 + (warp & 3)] = acc[0];
    __syncthreads();
    if (threadIdx.x < 4) {
        const int r = b + G * threadIdx.x;
        if (r < router_rows_n) {
            float s = part[threadIdx.x * 4 + 0];
            s += part[threadIdx.x * 4 + 1];
            s += part[threadIdx.x * 4 + 2];
            s += part[threadIdx.x * 4 + 3];
            if (r < E) A.logits[r] = s;
            else *A.gate_out = __float2half_rn(s);
        }
    }
    const unsigned long long base = base_s;
    bool ok = grid_sync(A.bar, base + G, A.err, flag, !(g_ly_withhold && b == 0));

    // ---- C: the top-k of the logits, in every CTA
    if (warp == 0) {
        topk_row<kLyTopkNV>([&](int j) { return __ldcg(A.logits + j); }, E, K, sidx, sw);
        __syncwarp();
        if (b == 0 && lane < K) {
            A.idx[lane] = sidx[lane];
            A.weights[lane] = sw[lane];
        }
    }
    __syncthreads();
    if (lane < nj_d && A.d[md & 3].routed) yd = place(A.d[md & 3], md, sidx[(md >> 7) & 63], md);
    if (lane < ja_e) ye = place(ER, me, sidx[(me >> 7) & 63], me);
    else if (lane < ja_e + jb_e) ye = place(ES, me, 0u, me);
    placed = true;
    while (ok && issued < ns - 1 && cursor_ready()) issue();  // (nothing more after a wait gave up)

    // ---- D and E: this warp's units. A warp adds up each job's units it has (two jobs open at a time: one
    // of each kind); its partial sums then go to the job's slot, and the warp whose units complete the job adds
    // the 16 warps' slots in warp order (zero where a warp had none) and writes the 16 rows.
    float tot[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
    int open_job[2] = {-1, -1}, open_units[2] = {0, 0};
    int slot = 0, waited = 0;
    uint32_t phase = 0;
    auto flush = [&](int P, int kind) {
        const int job = open_job[kind];
        if (job < 0) return;
        const int js = job;
        const int meta = __shfl_sync(0xffffffffu, P == 0 ? md : me, job);
        const LyStack& S = P == 0 ? A.d[meta & 3] : A.e[meta & 3];
        float* pw = partial + (js * kM8Warps + warp) * 16;
        if (tig == 0) {
            pw[gid] = tot[kind][0];
            pw[gid + 8] = tot[kind][1];
        }
        tot[kind][0] = tot[kind][1] = 0.f;
        __syncwarp();
        int last = 0;
        if (lane == 0) {
            __threadfence_block();
            last = atomicAdd(cnt + js, open_units[kind]) + open_units[kind] == S.stages;
            __threadfence_block();
        }
        open_job[kind] = -1;
        open_units[kind] = 0;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) return;
        const int cls = (meta >> 2) & 15, valid = (meta >> 6) & 1, pair = (meta >> 7) & 63, blk = meta >> 13;
        float* pj = partial + js * kM8Warps * 16;
        if (lane < 16) {
            float v = pj[lane];
            for (int w = 1; w < kM8Warps; ++w) v += pj[w * 16 + lane];
            const int64_t row = int64_t(blk) * 16 * S.q + cls + int64_t(S.q) * lane;
            if (valid && row < S.rows) S.out[int64_t(pair) * S.rows + row] = __float2half_rn(v);
        }
        __syncwarp();
        // the slot back to zero for the next phase
#pragma unroll
        for (int i = 0; i < 8; ++i) pj[i * 32 + lane] = 0.f;
        if (lane == 0) cnt[js] = 0;
    };
    auto run_units = [&](int P) {
        const int n = P == 0 ? n_d : n_e;
        for (UnitWalk w = walk_start(P, warp); w.p < n; walk_next(P, w)) {
            const Unit u = walk_unit(P, w);
            if (u.job != open_job[u.kind]) {
                flush(P, u.kind);
                open_job[u.kind] = u.job;
            }
            ++open_units[u.kind];
            // keep ns - 1 copies ahead; the slot refilled is the one this warp finished last
            __syncwarp();
            if (ok && cursor_ready()) issue();  // (after a wait gave up, nothing more is copied)
            const int cs = slot;
            if (ok) {
                ok = __all_sync(0xffffffffu, tc::mbar_wait(&my_bars[cs], phase, kM8WaitLimit));
                if (ok) ++waited;
            }
            if (++slot == ns) {
                slot = 0;
                phase ^= 1;
            }
            const int meta = __shfl_sync(0xffffffffu, P == 0 ? md : me, u.job);
            if (!ok || !((meta >> 6) & 1)) continue;
            const LyStack& S = P == 0 ? A.d[meta & 3] : A.e[meta & 3];
            // the unit's activation row in the split area: the token (D); in E the CTA's routed pair's row, or
            // the shared row after it
            const int xoff = P == 0 ? 0 : (u.kind == 0 ? 0 : ER.stages * ER.stage_cols);
            const int soff = P == 0 ? 0 : (u.kind == 0 ? 0 : ER.stages * ER.stage_cols / kM8XBlock);
            const uint8_t* xh = reinterpret_cast<const uint8_t*>(xsplit) + xoff;
            const uint8_t* xl = xh + A.split_bytes / 2;
            const float* xsc = xscale + soff;
            const int pos = ((meta >> 2) & 15) * static_cast<int>(S.row_bytes) + u.stage * S.stage_bytes;
            const int xc = u.stage * S.stage_cols;
            const uint8_t* st = my_ring + cs * slot_bytes + (pos & 15);
            if (S.kind == M8IQ3S<2>::kKind)
                M8IQ3S<2, kLyRep>::stage(st + gid * M8IQ3S<2>::kRS, st + (gid + 8) * M8IQ3S<2>::kRS, tig, gid, lut,
                                         xh + xc, xl + xc, xsc + xc / kM8XBlock, tot[u.kind]);
            else
                M8Q8_0::stage(st + gid * M8Q8_0::kRS, st + (gid + 8) * M8Q8_0::kRS, tig, gid, lut, xh + xc, xl + xc,
                              xsc + xc / kM8XBlock, tot[u.kind]);
        }
        flush(P, 0);
        flush(P, 1);
    };
    run_units(0);
    ok = grid_sync(A.bar, base + 2ull * G, A.err, flag) && ok;

    // ---- E: the split of this CTA's SwiGLU rows (its routed pair's, then the shared one), then its units
    {
        const int xb_r = ER.stages * ER.stage_cols / kM8XBlock;  // blocks of a routed row
        const int xb_s = ES.stages * ES.stage_cols / kM8XBlock;
        const int nr = ja_e > 0 ? xb_r : 0, nsb = jb_e > 0 ? xb_s : 0;
        for (int blk = warp; blk < nr + nsb; blk += kM8Warps) {
            const bool routed = blk < nr;
            const LySource& X = A.src_e[routed ? 0 : 1];
            const int c = routed ? blk : blk - nr;
            const int64_t at = int64_t(routed ? epair : 0) * X.cols + int64_t(c) * kM8XBlock + 8 * lane;
            const int lat = (routed ? 0 : xb_r * kM8XBlock) + c * kM8XBlock + 8 * lane;
            ly_split_glu(X.gate, X.up, at, xsplit + lat, xsplit + A.split_bytes / 2 + lat,
                         xscale + (routed ? c : xb_r + c), lane);
        }
        __syncthreads();
    }
    run_units(1);
    ok = grid_sync(A.bar, base + 3ull * G, A.err, flag) && ok;

    // ---- F: the combine, rows [b H / G, (b + 1) H / G)
    if (ok) {
        const __half g = __ldcg(A.gate_out);
        const int r0 = static_cast<int>(int64_t(b) * H / G), r1 = static_cast<int>(int64_t(b + 1) * H / G);
        for (int r = r0 + threadIdx.x; r < r1; r += kM8Threads) {
            const __half sv = __ldcg(A.s + r);
            // combine_one reads the k experts' values at y + j * stride; they were written by other CTAs
            __half yv[kLyMaxK];
            for (int j = 0; j < K; ++j) yv[j] = __ldcg(A.y + int64_t(j) * H + r);
            A.out[r] = combine_one(yv, 1, sw, K, g, sv);
        }
    }
    // no copy may still be writing this CTA's shared memory when it exits: every item was waited for, unless a
    // wait gave up; then the items issued after the last one waited for are waited for here (no item was issued
    // after the wait gave up)
    if (!ok && lane == 0)
        for (int i = waited; i < issued; ++i) tc::mbar_wait(&my_bars[i % ns], (i / ns) & 1, kM8WaitLimit);
    __syncwarp();
}

}  // namespace smoe

using namespace smoe;

extern "C" size_t smoe_decode_layer_scratch(int64_t hidden, int64_t k, int64_t ffn, int64_t sffn) {
    // g_r, u_r [k][ffn]; gs, us [sffn]; y [k][hidden]; s [hidden] (float16), then the barrier counter and flag
    const size_t halves = size_t(2 * k * ffn + 2 * sffn + k * hidden + hidden);
    return ((halves * 2 + 255) & ~size_t(255)) + 256;
}

namespace {
typedef CUresult (*LyEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                               const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                               CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
LyEncodeFn ly_encoder() {
    static LyEncodeFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return reinterpret_cast<LyEncodeFn>(p);
        return static_cast<LyEncodeFn>(nullptr);
    }();
    return fn;
}
}  // namespace

extern "C" int smoe_decode_layer(const SmoeDecodeLayer* L, const void* x, void* stream) {
    SMOE_REQUIRE(L && x, SMOE_EARG, "decode_layer: null argument");
    const int64_t H = L->hidden, E = L->experts, K = L->k, F = L->ffn, FS = L->sffn;
    SMOE_REQUIRE(L->router && L->shared_gate && L->gate && L->up && L->down && L->sgate && L->sup && L->sdown && L->logits && L->idx &&
                     L->weights && L->gate_out && L->out && L->scratch,
                 SMOE_EARG, "decode_layer: null pointer");
    SMOE_REQUIRE(L->kind == 21 && L->shared_kind == 8, SMOE_EKIND,
                 "decode_layer takes IQ3_S routed experts and a Q8_0 shared expert");
    SMOE_REQUIRE(E >= 1 && E <= kLyMaxExperts && K >= 1 && K <= std::min<int64_t>(E, kLyMaxK), SMOE_ESHAPE,
                 "decode_layer: 1 <= k <= experts <= 256, k <= 32");
    SMOE_REQUIRE(H % 512 == 0 && F % 512 == 0 && FS % 256 == 0 && H <= 16384 && F <= 16384 && FS <= 16384,
                 SMOE_ESHAPE, "decode_layer: hidden and ffn multiples of 512, shared ffn of 256");
    const void* ptrs[] = {L->router, L->shared_gate, x, L->gate, L->up, L->down, L->sgate, L->sup, L->sdown,
                          L->scratch};
    for (const void* p : ptrs)
        SMOE_REQUIRE((reinterpret_cast<uintptr_t>(p) & 15) == 0, SMOE_EARG, "decode_layer: 16-byte aligned inputs");
    LyEncodeFn encode = ly_encoder();
    SMOE_REQUIRE(encode != nullptr, SMOE_EARG, "decode_layer: no tensor-map encoder");
    cudaStream_t st = as_stream(stream);
    int dev = 0, sms = 0, coop = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
    SMOE_REQUIRE(sms > 1 && coop, SMOE_EARG, "decode_layer: needs cooperative launches");
    const int G = sms;

    LyArgs A{};
    A.router = reinterpret_cast<const __half*>(L->router);
    A.sgate = reinterpret_cast<const __half*>(L->shared_gate);
    A.x = static_cast<const __half*>(x);
    A.experts = static_cast<int>(E);
    A.hidden = static_cast<int>(H);
    A.k = static_cast<int>(K);
    A.logits = L->logits;
    A.idx = L->idx;
    A.weights = L->weights;
    A.gate_out = static_cast<__half*>(L->gate_out);
    A.out = static_cast<__half*>(L->out);
    __half* scr = static_cast<__half*>(L->scratch);
    __half* g_r = scr;
    __half* u_r = g_r + K * F;
    __half* gs = u_r + K * F;
    __half* us = gs + FS;
    A.y = us + FS;
    A.s = A.y + K * H;
    const size_t halves = size_t(2 * K * F + 2 * FS + K * H + H);
    uint8_t* tail = reinterpret_cast<uint8_t*>(L->scratch) + ((halves * 2 + 255) & ~size_t(255));
    A.bar = reinterpret_cast<unsigned long long*>(tail);
    A.err = reinterpret_cast<int*>(tail + 64);

    // the six stacks: geometry, TMA maps (raw rows seen as [rows / q][q row_bytes / 4] words)
    LyMaps maps;
    auto stack = [&](LyStack& S, int map, int kind, const uint8_t* blocks, int64_t experts, int64_t rows, int64_t cols,
                     int routed, int pairs, __half* out) -> bool {
        const int64_t per = kind == 21 ? 256 : 32, bb = kind == 21 ? 110 : 34;
        S.row_bytes = cols / per * bb;
        S.kind = kind;
        S.stage_cols = kind == 21 ? M8IQ3S<2>::kStageCols : M8Q8_0::kStageCols;
        S.stage_bytes = kind == 21 ? M8IQ3S<2>::kStageBytes : M8Q8_0::kStageBytes;
        S.rs = kind == 21 ? M8IQ3S<2>::kRS : M8Q8_0::kRS;
        int gcd = 16;
        while (S.row_bytes % gcd) gcd >>= 1;
        S.q = 16 / gcd;
        S.lq = S.q == 1 ? 0 : S.q == 2 ? 1 : S.q == 4 ? 2 : S.q == 8 ? 3 : 4;
        if (rows % S.q || experts * rows / S.q >= (int64_t(1) << 31)) return false;
        S.rows = rows;
        S.tiles = static_cast<int>((rows + 16 * S.q - 1) / (16 * S.q)) * S.q;
        S.stages = static_cast<int>(cols / S.stage_cols);
        S.routed = routed;
        S.pairs = pairs;
        S.jobs = pairs * S.tiles;
        S.map = map;
        S.out = out;
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(S.q * S.row_bytes / 4),
                                    static_cast<cuuint64_t>(experts * rows / S.q)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(S.q * S.row_bytes)};
        const cuuint32_t box[2] = {static_cast<cuuint32_t>(S.rs / 4), 16};
        const cuuint32_t estr[2] = {1, 1};
        return encode(&maps.w[map], CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint8_t*>(blocks), dims, strides,
                      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    };
    // phase D, costliest jobs first: the shared expert's rows (Q8_0 of hidden columns) before the routed
    const int kk = static_cast<int>(K);
    bool good = stack(A.d[0], 0, 8, L->sgate, 1, FS, H, 0, 1, gs) && stack(A.d[1], 1, 8, L->sup, 1, FS, H, 0, 1, us) &&
                stack(A.d[2], 2, 21, L->gate, E, F, H, 1, kk, g_r) && stack(A.d[3], 3, 21, L->up, E, F, H, 1, kk, u_r) &&
                stack(A.e[0], 4, 21, L->down, E, H, F, 1, kk, A.y) && stack(A.e[1], 5, 8, L->sdown, 1, H, FS, 0, 1, A.s);
    SMOE_REQUIRE(good, SMOE_ESHAPE, "decode_layer: stack geometry");
    A.nd = 4;
    int jobs = 0;
    for (int i = 0; i < 4; ++i) {
        A.d[i].job0 = jobs;
        jobs += A.d[i].jobs;
    }
    A.jobs_d = jobs;
    A.e[0].job0 = A.e[1].job0 = 0;
    A.src_d = LySource{A.x, nullptr, nullptr, 1, static_cast<int>(H)};
    A.src_e[0] = LySource{nullptr, g_r, u_r, kk, static_cast<int>(F)};
    A.src_e[1] = LySource{nullptr, gs, us, 1, static_cast<int>(FS)};

    // every CTA's jobs of a phase within its kLySlots partial-sum slots: phase D round-robin; phase E its tiles
    // of one routed pair (the CTAs split the pairs evenly) and its share of the shared down's jobs
    SMOE_REQUIRE(jobs <= int64_t(kLySlots) * G, SMOE_ESHAPE, "decode_layer: too many gate / up jobs");
    SMOE_REQUIRE(G >= K, SMOE_ESHAPE, "decode_layer: fewer SMs than routed experts");
    for (int b = 0; b < G; ++b) {
        const int p = static_cast<int>(int64_t(b) * K / G);
        const int c0 = static_cast<int>((int64_t(p) * G + K - 1) / K), c1 = static_cast<int>((int64_t(p + 1) * G + K - 1) / K);
        const int64_t rt = int64_t(b - c0 + 1) * A.e[0].tiles / (c1 - c0) - int64_t(b - c0) * A.e[0].tiles / (c1 - c0);
        const int64_t st_ = int64_t(b + 1) * A.e[1].jobs / G - int64_t(b) * A.e[1].jobs / G;
        SMOE_REQUIRE(rt + st_ <= kLySlots, SMOE_ESHAPE, "decode_layer: too many down jobs for a CTA");
    }
    SMOE_REQUIRE((F + FS) / 256 <= 64 && H / 256 <= 64, SMOE_ESHAPE, "decode_layer: activation scales");
    // shared memory: the split area holds the token (D) or a CTA's SwiGLU rows (E: its routed pair's and the
    // shared one)
    A.split_bytes = static_cast<int>((2 * std::max<int64_t>(H, F + FS) + 127) & ~int64_t(127));
    A.slot_bytes = 16 * std::max(M8IQ3S<2>::kRS, M8Q8_0::kRS);
    const size_t fixed = size_t(kM8Warps) * kM8MaxSlots * 8 + size_t(kLySlots) * kM8Warps * 16 * 4 + 32 * 4 + 16 * 4 +
                         kLyMaxK * 8 + 32 * 4 + 512 * kLyRep * 4 + 64 * 4 + size_t(A.split_bytes);
    const size_t slot = size_t(kM8Warps) * A.slot_bytes;
    int ns = kM8MaxSlots;
    while (ns > 2 && fixed + ns * slot > size_t(227 * 1024 - 256)) --ns;
    SMOE_REQUIRE(fixed + ns * slot <= size_t(227 * 1024 - 256), SMOE_ESHAPE, "decode_layer: shared memory");
    A.nslots = ns;
    const size_t smem = fixed + ns * slot;
    if (int s = max_smem(decode_layer_kernel, static_cast<int>(smem)))
        return fail(s, "decode_layer: shared memory limit");

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(kM8Threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, decode_layer_kernel, A, maps);
    return launch_status("decode_layer");
}

extern "C" int smoe_decode_layer_wait_test(int withhold) {
    const int w = withhold ? 1 : 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_ly_withhold, &w, sizeof(w));
    if (e != cudaSuccess) return fail(-static_cast<int>(e), std::string("decode_layer_wait_test: ") + cudaGetErrorString(e));
    return SMOE_OK;
}

extern "C" int smoe_decode_layer_status(const void* scratch, int64_t hidden, int64_t k, int64_t ffn, int64_t sffn,
                                        int* failed) {
    SMOE_REQUIRE(scratch && failed, SMOE_EARG, "decode_layer_status: null argument");
    const size_t halves = size_t(2 * k * ffn + 2 * sffn + k * hidden + hidden);
    const uint8_t* tail = static_cast<const uint8_t*>(scratch) + ((halves * 2 + 255) & ~size_t(255));
    int v = 0;
    cudaError_t e = cudaMemcpy(&v, tail + 64, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return fail(-static_cast<int>(e), "decode_layer_status: copy");
    *failed = v;
    return SMOE_OK;
}
