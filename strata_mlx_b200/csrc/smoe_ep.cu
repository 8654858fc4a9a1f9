// Expert parallelism for a prompt chunk: each rank holds its own tokens, the experts are spread over the ranks
// (rank r owns experts [r E/N, (r+1) E/N)), and the pairs travel to their experts' ranks and back by two
// all-to-all exchanges. The kernels here are the two ends of those exchanges:
//
//   ep_plan_kernel     every pair's destination rank, the counts per destination, the pair's place in the
//                      send order (destinations in rank order, pairs of one destination in pair order), and the
//                      expert each place names in its owner's numbering;
//   ep_gather_kernel   the send buffer: the token row of every pair at its place;
//   combine_rows_kernel  the block's combine (strata_mlx/fused.py:448-462) reading each pair's expert output at
//                      its place in the returned buffer, so the outputs need no scatter of their own.
//
// The order within a destination is the pair order, so what a rank receives from one peer is that peer's pairs
// in order: the result does not depend on timing.

#include <algorithm>
#include <cstdint>

#include "common.cuh"

namespace smoe {
namespace {

constexpr int kEpThreads = 1024;
constexpr int kEpMaxRanks = 64;

// One CTA. Pass 1 counts the pairs per destination; pass 2 walks the pairs in chunks of 1024 and places each
// after the earlier pairs of its destination (lanes of one destination found by __match_any_sync, the warps
// before it by their per-destination totals). A pair whose expert is not below `experts` gets place -1 and
// is not sent.
__global__ void __launch_bounds__(kEpThreads) ep_plan_kernel(const uint32_t* __restrict__ idx, int64_t pairs,
                                                             uint32_t experts, int ranks, int32_t* __restrict__ counts,
                                                             int32_t* __restrict__ where,
                                                             uint32_t* __restrict__ send_expert) {
    __shared__ int base[kEpMaxRanks + 1];
    __shared__ int warp_count[kEpThreads / 32][kEpMaxRanks + 1];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t per = experts / static_cast<uint32_t>(ranks);
    for (int r = tid; r <= ranks; r += kEpThreads) base[r] = 0;
    __syncthreads();
    for (int64_t i = tid; i < pairs; i += kEpThreads) {
        const uint32_t e = idx[i];
        if (e < experts) atomicAdd(&base[e / per], 1);
    }
    __syncthreads();
    if (tid == 0) {
        int run = 0;
        for (int r = 0; r < ranks; ++r) {
            const int c = base[r];
            counts[r] = c;
            base[r] = run;
            run += c;
        }
    }
    __syncthreads();
    for (int64_t chunk = 0; chunk < pairs; chunk += kEpThreads) {
        const int64_t i = chunk + tid;
        uint32_t e = experts;
        int dest = ranks;  // not sent (past the end, or an expert out of range)
        if (i < pairs) {
            e = idx[i];
            if (e < experts) dest = static_cast<int>(e / per);
        }
        const unsigned same = __match_any_sync(0xffffffffu, dest);
        const int below = __popc(same & ((1u << lane) - 1u));
        for (int r = lane; r <= ranks; r += 32) warp_count[warp][r] = 0;
        __syncwarp();
        if (below == 0) warp_count[warp][dest] = __popc(same);
        __syncthreads();
        if (i < pairs) {
            if (dest < ranks) {
                int before = 0;
                for (int w = 0; w < warp; ++w) before += warp_count[w][dest];
                const int place = base[dest] + before + below;
                where[i] = place;
                send_expert[place] = e - static_cast<uint32_t>(dest) * per;
            } else {
                where[i] = -1;
            }
        }
        __syncthreads();
        for (int r = tid; r < ranks; r += kEpThreads) {
            int s = 0;
            for (int w = 0; w < kEpThreads / 32; ++w) s += warp_count[w][r];
            base[r] += s;
        }
        __syncthreads();
    }
}

// out[where[i]] = x[i / k] for every pair i with a place; rows of `vecs` words of type V.
template <typename V>
__global__ void ep_gather_kernel(const V* __restrict__ x, const int32_t* __restrict__ where, int64_t pairs, int k,
                                 int64_t vecs, V* __restrict__ out) {
    for (int64_t i = blockIdx.x; i < pairs; i += gridDim.x) {
        const int32_t place = where[i];
        if (place < 0) continue;
        const V* src = x + (i / k) * vecs;
        V* dst = out + int64_t(place) * vecs;
        for (int64_t j = threadIdx.x; j < vecs; j += blockDim.x) dst[j] = src[j];
    }
}

// out[t, i] = the combine of y[where[t k + j], i] (j < k), w[t], g[t], s[t, i]; a pair without a place adds 0.
template <typename T>
__global__ void combine_rows_kernel(const T* __restrict__ y, const int32_t* __restrict__ where,
                                    const float* __restrict__ w, const T* __restrict__ g, const T* __restrict__ s,
                                    int64_t tokens, int k, int64_t d, T* __restrict__ out) {
    __shared__ int32_t place[32];
    for (int64_t t = blockIdx.y; t < tokens; t += gridDim.y) {
        __syncthreads();
        if (threadIdx.x < k) place[threadIdx.x] = where[t * k + threadIdx.x];
        __syncthreads();
        for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < d; i += int64_t(gridDim.x) * blockDim.x) {
            T yv[32];
            for (int j = 0; j < k; ++j) yv[j] = place[j] >= 0 ? y[int64_t(place[j]) * d + i] : from_f32<T>(0.0f);
            out[t * d + i] = combine_one(yv, 1, w + t * k, k, g[t], s[t * d + i]);
        }
    }
}

}  // namespace
}  // namespace smoe

using namespace smoe;

extern "C" int smoe_ep_dispatch(const uint32_t* idx, int64_t pairs, int64_t k, int64_t experts, int64_t ranks,
                                const void* x, int64_t hidden, int dtype, int32_t* counts, int32_t* where,
                                uint32_t* send_expert, void* send_x, void* stream) {
    SMOE_REQUIRE(counts && ranks > 0 && ranks <= kEpMaxRanks, SMOE_EARG, "ep_dispatch: 1 to 64 ranks");
    SMOE_REQUIRE(experts > 0 && experts <= UINT32_MAX && experts % ranks == 0, SMOE_ESHAPE,
                 "ep_dispatch: the experts must split evenly over the ranks");
    SMOE_REQUIRE(k > 0 && pairs >= 0 && pairs % k == 0 && pairs <= INT32_MAX, SMOE_ESHAPE,
                 "ep_dispatch: pairs must be tokens x k");
    SMOE_REQUIRE(hidden > 0, SMOE_ESHAPE, "ep_dispatch: empty rows");
    const int esize = dtype == SMOE_F16 ? 2 : dtype == SMOE_F32 ? 4 : 0;
    SMOE_REQUIRE(esize, SMOE_EDTYPE, "ep_dispatch: rows must be float16 or float32");
    cudaStream_t st = as_stream(stream);
    if (pairs == 0) {
        if (cudaMemsetAsync(counts, 0, sizeof(int32_t) * ranks, st) != cudaSuccess) return launch_status("ep_dispatch");
        return SMOE_OK;
    }
    SMOE_REQUIRE(idx && where && send_expert && x && send_x, SMOE_EARG, "ep_dispatch: null pointer");
    ep_plan_kernel<<<1, kEpThreads, 0, st>>>(idx, pairs, static_cast<uint32_t>(experts), static_cast<int>(ranks),
                                            counts, where, send_expert);
    const int64_t row_bytes = hidden * esize;
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(pairs, 148 * 16));
    const auto addr = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(send_x);
    if (row_bytes % 16 == 0 && addr % 16 == 0)
        ep_gather_kernel<uint4><<<grid, 128, 0, st>>>(static_cast<const uint4*>(x), where, pairs, static_cast<int>(k),
                                                       row_bytes / 16, static_cast<uint4*>(send_x));
    else if (row_bytes % 4 == 0 && addr % 4 == 0)
        ep_gather_kernel<uint32_t><<<grid, 128, 0, st>>>(static_cast<const uint32_t*>(x), where, pairs,
                                                          static_cast<int>(k), row_bytes / 4,
                                                          static_cast<uint32_t*>(send_x));
    else
        ep_gather_kernel<uint16_t><<<grid, 128, 0, st>>>(static_cast<const uint16_t*>(x), where, pairs,
                                                          static_cast<int>(k), row_bytes / 2,
                                                          static_cast<uint16_t*>(send_x));
    return launch_status("ep_dispatch");
}

extern "C" int smoe_combine_rows(const void* y, const int32_t* where, const float* w, const void* g, const void* s,
                                 int64_t tokens, int64_t k, int64_t d, void* out, int dtype, void* stream) {
    if (tokens == 0) return SMOE_OK;
    SMOE_REQUIRE(y && where && w && g && s && out && tokens > 0 && d > 0, SMOE_EARG, "combine_rows: bad arguments");
    SMOE_REQUIRE(k > 0 && k <= 32, SMOE_ESHAPE, "combine_rows: k must be 1..32");
    dim3 grid(static_cast<unsigned>(std::min<int64_t>((d + 255) / 256, 64)),
              static_cast<unsigned>(std::min<int64_t>(tokens, 65535)));
    cudaStream_t st = as_stream(stream);
    if (dtype == SMOE_F16)
        combine_rows_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(y), where, w,
                                                         static_cast<const __half*>(g), static_cast<const __half*>(s),
                                                         tokens, static_cast<int>(k), d, static_cast<__half*>(out));
    else if (dtype == SMOE_F32)
        combine_rows_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(y), where, w,
                                                        static_cast<const float*>(g), static_cast<const float*>(s),
                                                        tokens, static_cast<int>(k), d, static_cast<float*>(out));
    else
        return fail(SMOE_EDTYPE, "combine_rows takes float16 or float32 activations");
    return launch_status("combine_rows");
}
