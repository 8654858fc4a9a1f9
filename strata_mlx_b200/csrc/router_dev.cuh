// Device pieces of the router and its top-k shared by the route kernels (smoe_router.cu) and the fused
// decode layer (smoe_layer.cu).
#pragma once

#include <cfloat>

#include "common.cuh"

namespace smoe {

// ---------------------------------------------------------------- router logits
//
// A CTA of 8 warps takes two expert rows and up to 8 tokens: four warps to a row, each reading every fourth
// 16-byte chunk of the row (coalesced across the four), float32 fused multiply-adds, a shuffle tree, then
// the four partials added in warp order. A token's sum is taken in the same order for any window size.

constexpr int kRtTokens = 8;

template <typename XT>
__device__ __forceinline__ void load8(const XT* p, float* v);
template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float* v) {
    const uint4 q = *reinterpret_cast<const uint4*>(p);
    const __half2* h = reinterpret_cast<const __half2*>(&q);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
    }
}
template <>
__device__ __forceinline__ void load8<float>(const float* p, float* v) {
    const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// The lane's first chunks of its row (router_rows' first round), loaded ahead: weights no kernel writes, so a
// launch may load them before it waits for the kernel before it.
__device__ __forceinline__ void router_first(const __half* __restrict__ row, bool live, int64_t hidden,
                                             float (&wv)[4][8]) {
    const int quarter = (threadIdx.x >> 5) & 3, lane = threadIdx.x & 31;
    const int64_t chunks = hidden >> 3, c0 = quarter * 32 + lane;
    if (!live) return;
#pragma unroll
    for (int u = 0; u < 4; ++u)
        if (c0 + 128 * u < chunks) load8<__half>(row + 8 * (c0 + 128 * u), wv[u]);
}

// acc[t] += this lane's share of row . x[t0 + t] for the CTA's layout (four warps to a row, every fourth
// 16-byte chunk); four chunks of the row in flight at once (hidden 4096: all of this lane's), then their
// products in chunk order. wv holds the first round's chunks (router_first).
template <typename XT>
__device__ __forceinline__ void router_rows(const __half* __restrict__ row, bool live, const XT* __restrict__ x,
                                            int64_t hidden, int64_t t0, int nt, float (&acc)[kRtTokens],
                                            float (&wv)[4][8]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int quarter = warp & 3;
#pragma unroll
    for (int t = 0; t < kRtTokens; ++t) acc[t] = 0.0f;
    if (!live) return;
    const int64_t chunks = hidden >> 3;
    for (int64_t c0 = quarter * 32 + lane; c0 < chunks; c0 += 4 * 128) {
        if (c0 >= 4 * 128) {
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (c0 + 128 * u < chunks) load8<__half>(row + 8 * (c0 + 128 * u), wv[u]);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t c = c0 + 128 * u;
            if (c >= chunks) break;
#pragma unroll
            for (int t = 0; t < kRtTokens; ++t) {
                if (t < nt) {
                    float xv[8];
                    load8<XT>(x + (t0 + t) * hidden + 8 * c, xv);
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[t] = fmaf(wv[u][j], xv[j], acc[t]);
                }
            }
        }
    }
}

// ---------------------------------------------------------------- top-k and softmax over the chosen
//
// A warp per row: its values in registers (NV per lane, -inf past n), k rounds of a (value, index)
// arg-max over the warp, ties to the lower index, the winner struck out. Then the softmax of the chosen.

__device__ __forceinline__ bool better(float v, uint32_t i, float bv, uint32_t bi) {
    return v > bv || (v == bv && i < bi);
}

// One row's top-k and softmax by one warp; `load` reads logit j of the row.
// Order-preserving 32-bit key of a logit: larger keys for larger values, equal keys for equal values (-0 as +0),
// 0 for NaN (never chosen: `better` takes no NaN) -- every other key is above 0 (-inf's is 0x007FFFFF).
__device__ __forceinline__ uint32_t topk_key(float v) {
    if (v != v) return 0u;
    const uint32_t u = v == 0.0f ? 0u : __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// One row's top-k and softmax by one warp; `load` reads logit j of the row. Lane l holds logits l, l + 32, ...;
// each round the warp takes the largest key among the lanes' own best (a max reduction), the lowest index
// among the lanes holding it (a min reduction: ties to the lower index), and the winning lane alone looks for
// its next best. The same choice as rounds of `better` over all live values: the largest value, the lowest
// index among equal ones, never a NaN; 0xffffffff (and -inf) once nothing is left.
template <int NV, class Load>
__device__ __forceinline__ void topk_row(Load load, int n, int k, uint32_t* __restrict__ idx, float* __restrict__ weights) {
    const int lane = threadIdx.x & 31;
    float v[NV];
    uint32_t key[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int j = 32 * i + lane;
        v[i] = j < n ? load(j) : -INFINITY;
        key[i] = j < n ? topk_key(v[i]) : 0u;
    }
    // this lane's best: its largest key, the first such (the lowest index)
    uint32_t hk = 0u;
    int hi = 0;
    auto rescan = [&]() {
        hk = 0u;
        hi = 0;
#pragma unroll
        for (int i = 0; i < NV; ++i)
            if (key[i] > hk) {
                hk = key[i];
                hi = i;
            }
    };
    rescan();
    float top0 = 0.0f, sum = 0.0f, chosen = 0.0f;
    for (int r = 0; r < k; ++r) {
        const uint32_t m = __reduce_max_sync(0xffffffffu, hk);
        float bv = -INFINITY;
        uint32_t bi = 0xffffffffu;
        if (m != 0u) {
            bi = __reduce_min_sync(0xffffffffu, hk == m ? uint32_t(32 * hi + lane) : 0xffffffffu);
            float mine = 0.0f;
#pragma unroll
            for (int i = 0; i < NV; ++i)
                if (i == hi) mine = v[i];
            bv = __shfl_sync(0xffffffffu, mine, bi & 31u);
            if ((bi & 31u) == uint32_t(lane)) {
#pragma unroll
                for (int i = 0; i < NV; ++i)
                    if (uint32_t(i) == (bi >> 5)) key[i] = 0u;
                rescan();
            }
        }
        if (lane == 0) idx[r] = bi;
        // softmax over the chosen, largest first: lane r keeps its own chosen logit
        if (r == 0) top0 = bv;
        if (lane == (r & 31) && r < 32) chosen = bv;
    }
    if (weights != nullptr) {
        // exp(v - max) / sum in float32; k <= 32 here (checked on the host), one value a lane
        const float ex = lane < k ? expf(chosen - top0) : 0.0f;
        sum = warp_sum(lane < k ? ex : 0.0f);
        if (lane < k) weights[lane] = ex / sum;
    }
}

}  // namespace smoe
