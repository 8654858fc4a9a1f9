// The router's product, its top-k choice with the softmax over the chosen, and the combine at the end of the
// MoE block.
#include <type_traits>

#include "router_dev.cuh"

namespace smoe {

// ---------------------------------------------------------------- router logits

template <typename XT>
__global__ void __launch_bounds__(256) router_kernel(const __half* __restrict__ w, const XT* __restrict__ x,
                                                     int64_t tokens, int64_t experts, int64_t hidden,
                                                     float* __restrict__ logits) {
    __shared__ float part[2][4][kRtTokens];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int local_row = warp >> 2, quarter = warp & 3;
    const int64_t e = int64_t(blockIdx.x) * 2 + local_row;
    const int64_t t0 = int64_t(blockIdx.y) * kRtTokens;
    const int nt = static_cast<int>(min(int64_t(kRtTokens), tokens - t0));
    float acc[kRtTokens], wv[4][8];
    router_first(w + e * hidden, e < experts, hidden, wv);
    router_rows(w + e * hidden, e < experts, x, hidden, t0, nt, acc, wv);
#pragma unroll
    for (int t = 0; t < kRtTokens; ++t) acc[t] = warp_sum(acc[t]);
    if (lane == 0) {
#pragma unroll
        for (int t = 0; t < kRtTokens; ++t) part[local_row][quarter][t] = acc[t];
    }
    __syncthreads();
    if (threadIdx.x < 2 * kRtTokens) {
        const int r = threadIdx.x / kRtTokens, t = threadIdx.x % kRtTokens;
        const int64_t er = int64_t(blockIdx.x) * 2 + r;
        if (er < experts && t < nt) {
            float s = part[r][0][t];
            s += part[r][1][t];
            s += part[r][2][t];
            s += part[r][3][t];
            logits[(t0 + t) * experts + er] = s;
        }
    }
}

template <int NV>
__global__ void __launch_bounds__(128) topk_kernel(const float* __restrict__ logits, int64_t rows, int n, int k,
                                                   uint32_t* __restrict__ idx, float* __restrict__ weights) {
    const int warp = threadIdx.x >> 5;
    const int64_t row = int64_t(blockIdx.x) * 4 + warp;
    if (row >= rows) return;
    const float* in = logits + row * n;
    topk_row<NV>([&](int j) { return in[j]; }, n, k, idx + row * k, weights ? weights + row * k : nullptr);
}

// ---------------------------------------------------------------- router, top-k, softmax and shared gate in
// one launch
//
// The router kernel's CTAs over the expert rows (the same sums in the same order as router_kernel), plus one
// more row when the shared expert's gate row is given: its sum, rounded to the activations' type, is the
// block's gate value (`shared_expert_gate(x).to(x.dtype)`). Every CTA then counts itself done on its token
// group's counter; the last one (which sees all the group's logits after the fence) runs top_k_softmax for
// the group's tokens, a warp per token, and sets the counter back to zero for the next launch.

template <typename XT, int NV>
__global__ void __launch_bounds__(256) route_kernel(const __half* __restrict__ w, const __half* __restrict__ gw,
                                                    const XT* __restrict__ x, int64_t tokens, int64_t experts,
                                                    int64_t hidden, int k, float* __restrict__ logits,
                                                    uint32_t* __restrict__ idx, float* __restrict__ weights,
                                                    XT* __restrict__ gate_out, uint32_t* __restrict__ counters,
                                                    uint32_t lo, uint32_t count, uint32_t* __restrict__ lidx) {
    __shared__ float part[2][4][kRtTokens];
    __shared__ bool last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int local_row = warp >> 2, quarter = warp & 3;
    const int64_t e = int64_t(blockIdx.x) * 2 + local_row;
    const int64_t t0 = int64_t(blockIdx.y) * kRtTokens;
    const int nt = static_cast<int>(min(int64_t(kRtTokens), tokens - t0));
    const int64_t rows = experts + (gw != nullptr ? 1 : 0);
    const __half* row = e < experts ? w + e * hidden : gw;
    float acc[kRtTokens], wv[4][8];
    // the router's weights load while the kernel before this one finishes; x, the outputs and the counters wait
    router_first(row, e < rows, hidden, wv);
    pdl_wait();
    pdl_release();
    router_rows(row, e < rows, x, hidden, t0, nt, acc, wv);
#pragma unroll
    for (int t = 0; t < kRtTokens; ++t) acc[t] = warp_sum(acc[t]);
    if (lane == 0) {
#pragma unroll
        for (int t = 0; t < kRtTokens; ++t) part[local_row][quarter][t] = acc[t];
    }
    __syncthreads();
    if (threadIdx.x < 2 * kRtTokens) {
        const int r = threadIdx.x / kRtTokens, t = threadIdx.x % kRtTokens;
        const int64_t er = int64_t(blockIdx.x) * 2 + r;
        if (er < rows && t < nt) {
            float s = part[r][0][t];
            s += part[r][1][t];
            s += part[r][2][t];
            s += part[r][3][t];
            if (er < experts) logits[(t0 + t) * experts + er] = s;
            else gate_out[t0 + t] = from_f32<XT>(s);
        }
    }
    // the last CTA of this token group to finish takes the group's top-k
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(&counters[blockIdx.y], 1u) == gridDim.x - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (warp < nt) {
        const float* in = logits + (t0 + warp) * experts;
        topk_row<NV>([&](int j) { return __ldcg(in + j); }, static_cast<int>(experts), k, idx + (t0 + warp) * k,
                     weights + (t0 + warp) * k);
        if (lidx != nullptr) {  // this rank's view of the choice: expert - lo for its own, `count` for the others'
            __syncwarp();
            for (int j = lane; j < k; j += 32) {
                const uint32_t e = idx[(t0 + warp) * k + j] - lo;
                lidx[(t0 + warp) * k + j] = e < count ? e : count;
            }
        }
    }
    if (threadIdx.x == 0) counters[blockIdx.y] = 0u;
}

// ---------------------------------------------------------------- the route of a prompt chunk
//
// The same sums as router_rows, bit for bit: for each (row, token) lane l of quarter q adds the products of
// its chunks q 32 + l + 128 u in increasing u, a chunk's eight in order, from 0.0f by fused multiply-adds; the
// quarter's lanes are added by warp_sum's shuffle tree and the four quarters in order. Only the mapping differs:
// a warp takes one quarter of kPrRows rows x kPrTok tokens, so a lane's chunk of a weight row serves kPrTok
// tokens and its chunk of a token kPrRows rows from registers; a CTA's 8 warps are the four quarters of two
// token halves (kPrRows rows x 2 kPrTok tokens), small enough in registers for five CTAs an SM: the kernel is
// bound by the latency of its loads, not by L2 bandwidth. Float16 activations multiply as they are (no
// conversions). The last CTA of a group of 8 tokens takes the group's top-k (counters: one word per 8 tokens,
// smoe_route_counters' size); without counters the launch writes only the logits.

constexpr int kPrRows = 4, kPrTok = 4;
// a counter word covers 8 tokens (smoe_route_counters' size): the CTAs of those tokens count on it
constexpr int kPrGroup = kRtTokens, kPrCtasPerGroup = kPrGroup / (2 * kPrTok);
static_assert(kPrGroup % (2 * kPrTok) == 0, "a counter's tokens are whole CTAs' tokens");

// the eight float16 values of a 16-byte chunk, in order
__device__ __forceinline__ void split8(const uint4 q, unsigned short (&h)[8]) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        h[2 * i] = static_cast<unsigned short>(w[i] & 0xffffu);
        h[2 * i + 1] = static_cast<unsigned short>(w[i] >> 16);
    }
}

// acc + w x as one float32 fused multiply-add of two float16 values (mixed precision: fmaf of the values widened
// to float32, which is exact)
__device__ __forceinline__ float fma_h(unsigned short w, unsigned short x, float acc) {
    asm("fma.rn.f32.f16 %0, %1, %2, %0;" : "+f"(acc) : "h"(w), "h"(x));
    return acc;
}
constexpr int64_t kPrFrom = 32;  // windows of more tokens than this take route_chunk_kernel

template <typename XT, int NV>
__global__ void __launch_bounds__(256) route_chunk_kernel(const __half* __restrict__ w, const __half* __restrict__ gw,
                                                          const XT* __restrict__ x, int64_t tokens, int64_t experts,
                                                          int64_t hidden, int k, float* __restrict__ logits,
                                                          uint32_t* __restrict__ idx, float* __restrict__ weights,
                                                          XT* __restrict__ gate_out, uint32_t* __restrict__ counters,
                                                          uint32_t lo, uint32_t count, uint32_t* __restrict__ lidx) {
    __shared__ float part[4][2 * kPrTok][kPrRows];
    __shared__ bool last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int quarter = warp & 3, half = warp >> 2;
    const int64_t rows = experts + (gw != nullptr ? 1 : 0);
    const int64_t r0 = int64_t(blockIdx.x) * kPrRows;
    const int64_t tg0 = int64_t(blockIdx.y) * (2 * kPrTok);
    const int64_t t0 = tg0 + half * kPrTok;
    const int nt = static_cast<int>(max(int64_t(0), min(int64_t(kPrTok), tokens - t0)));
    const __half* rp[kPrRows];
    bool live[kPrRows];
#pragma unroll
    for (int r = 0; r < kPrRows; ++r) {
        const int64_t e = r0 + r;
        live[r] = e < rows;
        rp[r] = e < experts ? w + e * hidden : gw;
    }
    float acc[kPrRows][kPrTok];
#pragma unroll
    for (int r = 0; r < kPrRows; ++r)
#pragma unroll
        for (int t = 0; t < kPrTok; ++t) acc[r][t] = 0.0f;
    pdl_wait();
    pdl_release();
    const int64_t chunks = hidden >> 3;
    if constexpr (std::is_same<XT, __half>::value) {
        // float16 activations: fma.rn.f32.f16 takes both float16 operands as they are (their float32 values are
        // exact, so each step is fmaf(float(w), float(x), acc), router_rows' step) with no conversions
#pragma unroll 2
        for (int64_t c = quarter * 32 + lane; c < chunks; c += 128) {
            unsigned short wh[kPrRows][8];
#pragma unroll
            for (int r = 0; r < kPrRows; ++r) {
                const uint4 q = live[r] ? *reinterpret_cast<const uint4*>(rp[r] + 8 * c) : make_uint4(0u, 0u, 0u, 0u);
                split8(q, wh[r]);
            }
#pragma unroll
            for (int t = 0; t < kPrTok; ++t) {
                if (t < nt) {
                    unsigned short xh[8];
                    split8(*reinterpret_cast<const uint4*>(x + (t0 + t) * hidden + 8 * c), xh);
#pragma unroll
                    for (int r = 0; r < kPrRows; ++r)
#pragma unroll
                        for (int j = 0; j < 8; ++j) acc[r][t] = fma_h(wh[r][j], xh[j], acc[r][t]);
                }
            }
        }
    } else {
#pragma unroll 2
    for (int64_t c = quarter * 32 + lane; c < chunks; c += 128) {
        float wv[kPrRows][8];
#pragma unroll
        for (int r = 0; r < kPrRows; ++r) {
            if (live[r]) {
                load8<__half>(rp[r] + 8 * c, wv[r]);
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) wv[r][j] = 0.0f;
            }
        }
#pragma unroll
        for (int t = 0; t < kPrTok; ++t) {
            if (t < nt) {
                float xv[8];
                load8<XT>(x + (t0 + t) * hidden + 8 * c, xv);
#pragma unroll
                for (int r = 0; r < kPrRows; ++r)
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[r][t] = fmaf(wv[r][j], xv[j], acc[r][t]);
            }
        }
    }
    }
#pragma unroll
    for (int r = 0; r < kPrRows; ++r)
#pragma unroll
        for (int t = 0; t < kPrTok; ++t) acc[r][t] = warp_sum(acc[r][t]);
    if (lane == 0) {
#pragma unroll
        for (int r = 0; r < kPrRows; ++r)
#pragma unroll
            for (int t = 0; t < kPrTok; ++t) part[quarter][half * kPrTok + t][r] = acc[r][t];
    }
    __syncthreads();
    if (threadIdx.x < 2 * kPrTok * kPrRows) {
        const int tt = threadIdx.x / kPrRows, r = threadIdx.x % kPrRows;
        const int64_t e = r0 + r, t = tg0 + tt;
        if (e < rows && t < tokens) {
            float s = part[0][tt][r];
            s += part[1][tt][r];
            s += part[2][tt][r];
            s += part[3][tt][r];
            if (e < experts) logits[t * experts + e] = s;
            else gate_out[t] = from_f32<XT>(s);
        }
    }
    if (counters == nullptr) return;
    // the last CTA of this group of 8 tokens to finish takes the group's top-k, a warp to a token
    const unsigned grp = blockIdx.y / kPrCtasPerGroup;
    const unsigned ys = min(unsigned(kPrCtasPerGroup), gridDim.y - grp * kPrCtasPerGroup);  // the group's rows of CTAs
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(&counters[grp], 1u) == gridDim.x * ys - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int tt = warp; tt < kPrGroup; tt += 8) {
        const int64_t t = int64_t(grp) * kPrGroup + tt;
        if (t >= tokens) break;
        const float* in = logits + t * experts;
        topk_row<NV>([&](int j) { return __ldcg(in + j); }, static_cast<int>(experts), k, idx + t * k, weights + t * k);
        if (lidx != nullptr) {  // this rank's view of the choice: expert - lo for its own, `count` for the others'
            __syncwarp();
            for (int j = lane; j < k; j += 32) {
                const uint32_t e = idx[t * k + j] - lo;
                lidx[t * k + j] = e < count ? e : count;
            }
        }
        __syncwarp();
    }
    if (threadIdx.x == 0) counters[grp] = 0u;
}

// ---------------------------------------------------------------- combine

template <typename T>
__global__ void combine_kernel(const T* __restrict__ y, const float* __restrict__ w, const T* __restrict__ g,
                               const T* __restrict__ s, int64_t tokens, int k, int64_t d, T* __restrict__ out) {
    const int64_t t = blockIdx.y;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < d; i += int64_t(gridDim.x) * blockDim.x)
        out[t * d + i] = combine_one(y + (t * k) * d + i, d, w + t * k, k, g[t], s[t * d + i]);
}

// combine_kernel for float16 with d a multiple of 8 and 16-byte aligned rows: eight values a thread in 16-byte
// loads and stores, each value combine_one's arithmetic (the token's gate is the same value for all of them)
__global__ void combine8_kernel(const __half* __restrict__ y, const float* __restrict__ w, const __half* __restrict__ g,
                                const __half* __restrict__ s, int64_t tokens, int k, int64_t d, __half* __restrict__ out) {
    const int64_t t = blockIdx.y;
    const __half gate = __float2half_rn(1.0f / (1.0f + expf(-__half2float(g[t]))));
    const float* wt = w + t * k;
    for (int64_t i = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) * 8; i < d;
         i += int64_t(gridDim.x) * blockDim.x * 8) {
        float acc[8];
        for (int j0 = 0; j0 < 8 && j0 < k; ++j0) {
            float part[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) part[e] = 0.0f;
            for (int kk = j0; kk < k; kk += 8) {
                const uint4 q = *reinterpret_cast<const uint4*>(y + (t * k + kk) * d + i);
                const __half* h = reinterpret_cast<const __half*>(&q);
                const float wk = wt[kk];
#pragma unroll
                for (int e = 0; e < 8; ++e) part[e] = __fadd_rn(__fmul_rn(__half2float(h[e]), wk), part[e]);
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] = j0 == 0 ? part[e] : __fadd_rn(part[e], acc[e]);
        }
        const uint4 sq = *reinterpret_cast<const uint4*>(s + t * d + i);
        const __half* sh = reinterpret_cast<const __half*>(&sq);
        uint4 o;
        __half* oh = reinterpret_cast<__half*>(&o);
#pragma unroll
        for (int e = 0; e < 8; ++e) oh[e] = __hadd_rn(__float2half_rn(acc[e]), __hmul_rn(gate, sh[e]));
        *reinterpret_cast<uint4*>(out + t * d + i) = o;
    }
}

// ---------------------------------------------------------------- expert parallelism

// lidx = idx - lo for experts of this rank's range [lo, lo + count), else count (a pair the kernels leave out)
__global__ void localize_kernel(const uint32_t* __restrict__ idx, int64_t n, uint32_t lo, uint32_t count,
                                uint32_t* __restrict__ out) {
    pdl_wait();
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const uint32_t e = idx[i];
        out[i] = (e >= lo && e - lo < count) ? e - lo : count;
    }
    pdl_release();
}

// sums[t, 0:d] = this rank's share of sum_k y_k w_k (pairs of its experts only, MLX's order among them);
// sums[t, d:2d] = its slice of the shared expert's output (float32), or 0.
template <typename T>
__global__ void partial_sum_kernel(const T* __restrict__ y, const float* __restrict__ w, const uint32_t* __restrict__ lidx,
                                   uint32_t experts, const T* __restrict__ s, int64_t tokens, int k, int64_t d,
                                   float* __restrict__ sums) {
    const int64_t t = blockIdx.y;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < d; i += int64_t(gridDim.x) * blockDim.x) {
        float acc = 0.0f;
        for (int j = 0; j < 8 && j < k; ++j) {
            float part = 0.0f;
            for (int kk = j; kk < k; kk += 8) {
                if (lidx[t * k + kk] < experts)
                    part = __fadd_rn(__fmul_rn(to_f32(y[(t * k + kk) * d + i]), w[t * k + kk]), part);
            }
            acc = j == 0 ? part : __fadd_rn(part, acc);
        }
        sums[t * 2 * d + i] = acc;
        sums[t * 2 * d + d + i] = s ? to_f32(s[t * d + i]) : 0.0f;
    }
}

// The combine from all ranks' summed partials: out = half(routed) + half(half(sigmoid(g)) half(shared)).
template <typename T>
__global__ void combine_sums_kernel(const float* __restrict__ sums, const T* __restrict__ g, int64_t tokens, int64_t d,
                                    T* __restrict__ out) {
    const int64_t t = blockIdx.y;
    const T gate = from_f32<T>(1.0f / (1.0f + expf(-to_f32(g[t]))));
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < d; i += int64_t(gridDim.x) * blockDim.x) {
        const T routed = from_f32<T>(sums[t * 2 * d + i]);
        const T shared = mul_t<T>(gate, from_f32<T>(sums[t * 2 * d + d + i]));
        out[t * d + i] = add_t<T>(routed, shared);
    }
}

}  // namespace smoe

using namespace smoe;

extern "C" int smoe_localize(const uint32_t* idx, int64_t n, int64_t lo, int64_t count, uint32_t* out, void* stream) {
    if (n == 0) return SMOE_OK;
    SMOE_REQUIRE(idx && out && n > 0 && lo >= 0 && count > 0 && lo + count <= 0xffffffffLL, SMOE_EARG,
                 "localize: bad arguments");
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 1024));
    const cudaError_t e = launch_pdl(Writes().add(out, size_t(n) * 4), localize_kernel, dim3(grid), dim3(256), 0,
                                     as_stream(stream), idx, n, static_cast<uint32_t>(lo), static_cast<uint32_t>(count),
                                     out);
    if (e != cudaSuccess) return fail(-static_cast<int>(e), std::string("localize: ") + cudaGetErrorString(e));
    return launch_status("localize");
}

extern "C" int smoe_partial_sums(const void* y, const float* w, const uint32_t* lidx, int64_t experts, const void* s,
                                 int64_t tokens, int64_t k, int64_t d, float* sums, int dtype, void* stream) {
    if (tokens == 0) return SMOE_OK;
    SMOE_REQUIRE(y && w && lidx && sums && tokens > 0 && k > 0 && d > 0 && experts > 0, SMOE_EARG,
                 "partial_sums: bad arguments");
    SMOE_REQUIRE(tokens <= 65535, SMOE_ESHAPE, "too many tokens for one call");
    dim3 grid(static_cast<unsigned>(std::min<int64_t>((d + 255) / 256, 64)), static_cast<unsigned>(tokens));
    cudaStream_t st = as_stream(stream);
    if (dtype == SMOE_F16)
        partial_sum_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(y), w, lidx, static_cast<uint32_t>(experts),
                                                        static_cast<const __half*>(s), tokens, static_cast<int>(k), d, sums);
    else if (dtype == SMOE_F32)
        partial_sum_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(y), w, lidx, static_cast<uint32_t>(experts),
                                                       static_cast<const float*>(s), tokens, static_cast<int>(k), d, sums);
    else
        return fail(SMOE_EDTYPE, "partial_sums takes float16 or float32 activations");
    return launch_status("partial_sums");
}

extern "C" int smoe_combine_sums(const float* sums, const void* g, int64_t tokens, int64_t d, void* out, int dtype,
                                 void* stream) {
    if (tokens == 0) return SMOE_OK;
    SMOE_REQUIRE(sums && g && out && tokens > 0 && d > 0, SMOE_EARG, "combine_sums: bad arguments");
    SMOE_REQUIRE(tokens <= 65535, SMOE_ESHAPE, "too many tokens for one call");
    dim3 grid(static_cast<unsigned>(std::min<int64_t>((d + 255) / 256, 64)), static_cast<unsigned>(tokens));
    cudaStream_t st = as_stream(stream);
    if (dtype == SMOE_F16)
        combine_sums_kernel<__half><<<grid, 256, 0, st>>>(sums, static_cast<const __half*>(g), tokens, d,
                                                         static_cast<__half*>(out));
    else if (dtype == SMOE_F32)
        combine_sums_kernel<float><<<grid, 256, 0, st>>>(sums, static_cast<const float*>(g), tokens, d,
                                                        static_cast<float*>(out));
    else
        return fail(SMOE_EDTYPE, "combine_sums takes float16 or float32 activations");
    return launch_status("combine_sums");
}

extern "C" int smoe_router_logits(const uint16_t* weight, const void* x, int x_dtype, int64_t tokens, int64_t experts,
                                  int64_t hidden, float* logits, void* stream) {
    if (tokens == 0) return SMOE_OK;
    SMOE_REQUIRE(weight && x && logits && tokens > 0 && experts > 0, SMOE_EARG, "null pointer or empty router");
    SMOE_REQUIRE(hidden > 0 && hidden % 8 == 0, SMOE_ESHAPE, "router rows must hold a multiple of 8 values");
    SMOE_REQUIRE((reinterpret_cast<uintptr_t>(weight) & 15) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0,
                 SMOE_EARG, "router weight and activations must be 16-byte aligned");
    SMOE_REQUIRE((tokens + kRtTokens - 1) / kRtTokens <= 65535, SMOE_ESHAPE, "too many tokens for one router call");
    dim3 grid(static_cast<unsigned>((experts + 1) / 2), static_cast<unsigned>((tokens + kRtTokens - 1) / kRtTokens));
    cudaStream_t st = as_stream(stream);
    const __half* w = reinterpret_cast<const __half*>(weight);
    // a prompt chunk: the same sums with the chunks reused from registers (route_chunk_kernel, logits only)
    const bool chunk = tokens > kPrFrom;
    const dim3 cgrid(static_cast<unsigned>((experts + kPrRows - 1) / kPrRows),
                     static_cast<unsigned>((tokens + 2 * kPrTok - 1) / (2 * kPrTok)));
    if (x_dtype == SMOE_F16) {
        const __half* xp = static_cast<const __half*>(x);
        if (chunk)
            route_chunk_kernel<__half, 8><<<cgrid, 256, 0, st>>>(w, nullptr, xp, tokens, experts, hidden, 1, logits,
                                                                 nullptr, nullptr, nullptr, nullptr, 0u, 0u, nullptr);
        else
            router_kernel<__half><<<grid, 256, 0, st>>>(w, xp, tokens, experts, hidden, logits);
    } else if (x_dtype == SMOE_F32) {
        const float* xp = static_cast<const float*>(x);
        if (chunk)
            route_chunk_kernel<float, 8><<<cgrid, 256, 0, st>>>(w, nullptr, xp, tokens, experts, hidden, 1, logits,
                                                                nullptr, nullptr, nullptr, nullptr, 0u, 0u, nullptr);
        else
            router_kernel<float><<<grid, 256, 0, st>>>(w, xp, tokens, experts, hidden, logits);
    } else {
        return fail(SMOE_EDTYPE, "router activations must be float16 or float32");
    }
    return launch_status("router_logits");
}

extern "C" int smoe_top_k(const float* logits, int64_t rows, int64_t n, int64_t k, uint32_t* idx, float* weights,
                          void* stream) {
    if (rows == 0) return SMOE_OK;
    SMOE_REQUIRE(logits && idx && rows > 0, SMOE_EARG, "null pointer");
    SMOE_REQUIRE(n > 0 && n <= 2048, SMOE_ESHAPE, "top_k takes rows of 1 to 2048 logits");
    SMOE_REQUIRE(k >= 1 && k <= n && k <= 32, SMOE_ESHAPE, "top_k takes 1 <= k <= min(n, 32)");
    const unsigned grid = static_cast<unsigned>((rows + 3) / 4);
    cudaStream_t st = as_stream(stream);
    const int nn = static_cast<int>(n), kk = static_cast<int>(k);
    if (n <= 256)
        topk_kernel<8><<<grid, 128, 0, st>>>(logits, rows, nn, kk, idx, weights);
    else if (n <= 512)
        topk_kernel<16><<<grid, 128, 0, st>>>(logits, rows, nn, kk, idx, weights);
    else if (n <= 1024)
        topk_kernel<32><<<grid, 128, 0, st>>>(logits, rows, nn, kk, idx, weights);
    else
        topk_kernel<64><<<grid, 128, 0, st>>>(logits, rows, nn, kk, idx, weights);
    return launch_status("top_k");
}

extern "C" size_t smoe_route_counters(int64_t tokens) {
    return static_cast<size_t>(tokens > 0 ? (tokens + kRtTokens - 1) / kRtTokens : 1) * sizeof(uint32_t);
}

static int route_launch(const uint16_t* weight, const uint16_t* gate_weight, const void* x, int x_dtype,
                        int64_t tokens, int64_t experts, int64_t hidden, int64_t k, float* logits, uint32_t* idx,
                        float* weights, void* gate_out, uint32_t* counters, int64_t lo, int64_t count, uint32_t* lidx,
                        void* stream) {
    if (tokens == 0) return SMOE_OK;
    SMOE_REQUIRE(weight && x && logits && idx && weights && counters && tokens > 0 && experts > 0, SMOE_EARG,
                 "null pointer or empty router");
    SMOE_REQUIRE((gate_weight == nullptr) == (gate_out == nullptr), SMOE_EARG,
                 "the shared gate's weight and output come together");
    SMOE_REQUIRE(hidden > 0 && hidden % 8 == 0, SMOE_ESHAPE, "router rows must hold a multiple of 8 values");
    SMOE_REQUIRE((reinterpret_cast<uintptr_t>(weight) & 15) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(gate_weight) & 15) == 0,
                 SMOE_EARG, "router weights and activations must be 16-byte aligned");
    SMOE_REQUIRE(experts <= 2048, SMOE_ESHAPE, "route takes rows of 1 to 2048 logits");
    SMOE_REQUIRE(k >= 1 && k <= experts && k <= 32, SMOE_ESHAPE, "route takes 1 <= k <= min(experts, 32)");
    SMOE_REQUIRE((tokens + kRtTokens - 1) / kRtTokens <= 65535, SMOE_ESHAPE, "too many tokens for one route call");
    const int64_t rows = experts + (gate_weight ? 1 : 0);
    dim3 grid(static_cast<unsigned>((rows + 1) / 2), static_cast<unsigned>((tokens + kRtTokens - 1) / kRtTokens));
    cudaStream_t st = as_stream(stream);
    const __half* w = reinterpret_cast<const __half*>(weight);
    const __half* gw = reinterpret_cast<const __half*>(gate_weight);
    const int kk = static_cast<int>(k);
    auto go = [&](auto xt) {
        using XT = decltype(xt);
        const XT* xp = static_cast<const XT*>(x);
        XT* go_ = static_cast<XT*>(gate_out);
        Writes wr;
        wr.add(logits, size_t(tokens) * experts * 4).add(idx, size_t(tokens) * k * 4).add(weights, size_t(tokens) * k * 4);
        wr.add(gate_out, size_t(tokens) * sizeof(XT)).add(counters, smoe_route_counters(tokens));
        wr.add(lidx, size_t(tokens) * k * 4);
        const uint32_t l0 = static_cast<uint32_t>(lo), cn = static_cast<uint32_t>(count);
        if (tokens > kPrFrom) {
            // a prompt chunk: the same sums with the chunks reused from registers, one counter per 16 tokens
            const dim3 cgrid(static_cast<unsigned>((rows + kPrRows - 1) / kPrRows),
                             static_cast<unsigned>((tokens + 2 * kPrTok - 1) / (2 * kPrTok)));
            if (experts <= 256)
                launch_pdl(wr, route_chunk_kernel<XT, 8>, cgrid, dim3(256), 0, st, w, gw, xp, tokens, experts, hidden, kk, logits, idx, weights, go_, counters, l0, cn, lidx);
            else if (experts <= 512)
                launch_pdl(wr, route_chunk_kernel<XT, 16>, cgrid, dim3(256), 0, st, w, gw, xp, tokens, experts, hidden, kk, logits, idx, weights, go_, counters, l0, cn, lidx);
            else if (experts <= 1024)
                launch_pdl(wr, route_chunk_kernel<XT, 32>, cgrid, dim3(256), 0, st, w, gw, xp, tokens, experts, hidden, kk, logits, idx, weights, go_, counters, l0, cn, lidx);
            else
                launch_pdl(wr, route_chunk_kernel<XT, 64>, cgrid, dim3(256), 0, st, w, gw, xp, tokens, experts, hidden, kk, logits, idx, weights, go_, counters, l0, cn, lidx);
            return;
        }
        if (experts <= 256)
            launch_pdl(wr, route_kernel<XT, 8>, grid, dim3(256), 0, st, w, gw, xp, tokens, experts, hidden, kk, logits, idx, weights, go_, counters, l0, cn, lidx);
        else if (experts <= 512)
            launch_pdl(wr, route_kernel<XT, 16>, grid, dim3(256), 0, st, w, gw, xp, tokens, experts, hidden, kk, logits, idx, weights, go_, counters, l0, cn, lidx);
        else if (experts <= 1024)
            launch_pdl(wr, route_kernel<XT, 32>, grid, dim3(256), 0, st, w, gw, xp, tokens, experts, hidden, kk, logits, idx, weights, go_, counters, l0, cn, lidx);
        else
            launch_pdl(wr, route_kernel<XT, 64>, grid, dim3(256), 0, st, w, gw, xp, tokens, experts, hidden, kk, logits, idx, weights, go_, counters, l0, cn, lidx);
    };
    if (x_dtype == SMOE_F16) go(__half{});
    else if (x_dtype == SMOE_F32) go(float{});
    else return fail(SMOE_EDTYPE, "router activations must be float16 or float32");
    return launch_status("route");
}

extern "C" int smoe_route(const uint16_t* weight, const uint16_t* gate_weight, const void* x, int x_dtype,
                          int64_t tokens, int64_t experts, int64_t hidden, int64_t k, float* logits, uint32_t* idx,
                          float* weights, void* gate_out, uint32_t* counters, void* stream) {
    return route_launch(weight, gate_weight, x, x_dtype, tokens, experts, hidden, k, logits, idx, weights, gate_out,
                        counters, 0, 0, nullptr, stream);
}

extern "C" int smoe_route_local(const uint16_t* weight, const uint16_t* gate_weight, const void* x, int x_dtype,
                                int64_t tokens, int64_t experts, int64_t hidden, int64_t k, float* logits,
                                uint32_t* idx, float* weights, void* gate_out, uint32_t* counters, int64_t lo,
                                int64_t count, uint32_t* lidx, void* stream) {
    SMOE_REQUIRE(lidx && lo >= 0 && count > 0 && lo + count <= experts, SMOE_EARG,
                 "route_local: this rank's experts [lo, lo + count) must lie within the router's");
    return route_launch(weight, gate_weight, x, x_dtype, tokens, experts, hidden, k, logits, idx, weights, gate_out,
                        counters, lo, count, lidx, stream);
}

extern "C" int smoe_combine(const void* y, const float* w, const void* g, const void* s, int64_t tokens, int64_t k,
                            int64_t d, void* out, int dtype, void* stream) {
    if (tokens == 0) return SMOE_OK;
    SMOE_REQUIRE(y && w && g && s && out && tokens > 0 && k > 0 && d > 0, SMOE_EARG, "null pointer or empty shape");
    SMOE_REQUIRE(tokens <= 65535, SMOE_ESHAPE, "too many tokens for one combine call");
    dim3 grid(static_cast<unsigned>(std::min<int64_t>((d + 255) / 256, 64)), static_cast<unsigned>(tokens));
    cudaStream_t st = as_stream(stream);
    const bool v8 = d % 8 == 0 && ((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(s) |
                                    reinterpret_cast<uintptr_t>(out)) & 15) == 0;
    if (dtype == SMOE_F16 && v8)
        combine8_kernel<<<dim3(static_cast<unsigned>(std::min<int64_t>((d / 8 + 255) / 256, 64)),
                               static_cast<unsigned>(tokens)), 256, 0, st>>>(
            static_cast<const __half*>(y), w, static_cast<const __half*>(g), static_cast<const __half*>(s), tokens,
            static_cast<int>(k), d, static_cast<__half*>(out));
    else if (dtype == SMOE_F16)
        combine_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(y), w, static_cast<const __half*>(g),
                                                    static_cast<const __half*>(s), tokens, static_cast<int>(k), d,
                                                    static_cast<__half*>(out));
    else if (dtype == SMOE_F32)
        combine_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(y), w, static_cast<const float*>(g),
                                                   static_cast<const float*>(s), tokens, static_cast<int>(k), d,
                                                   static_cast<float*>(out));
    else
        return fail(SMOE_EDTYPE, "combine takes float16 or float32 activations");
    return launch_status("combine");
}
