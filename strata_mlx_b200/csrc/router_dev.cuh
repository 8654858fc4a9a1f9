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
template <int NV, class Load>
__device__ __forceinline__ void topk_row(Load load, int n, int k, uint32_t* __restrict__ idx, float* __restrict__ weights) {
    const int lane = threadIdx.x & 31;
    float v[NV];
    bool live[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int j = 32 * i + lane;
        live[i] = j < n;
        v[i] = live[i] ? load(j) : -INFINITY;
    }
    float top0 = 0.0f, sum = 0.0f, chosen = 0.0f;
    for (int r = 0; r < k; ++r) {
        float bv = -INFINITY;
        uint32_t bi = 0xffffffffu;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const uint32_t j = 32u * i + lane;
            if (live[i] && better(v[i], j, bv, bi)) {
                bv = v[i];
                bi = j;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (better(ov, oi, bv, bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) idx[r] = bi;
        if (bi != 0xffffffffu && (bi & 31u) == uint32_t(lane)) {
#pragma unroll
            for (int i = 0; i < NV; ++i)
                if (uint32_t(i) == (bi >> 5)) live[i] = false;
        }
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
