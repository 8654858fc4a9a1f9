// The router's product, its top-k choice with the softmax over the chosen, and the combine at the end of the
// MoE block.
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

// ---------------------------------------------------------------- combine

template <typename T>
__global__ void combine_kernel(const T* __restrict__ y, const float* __restrict__ w, const T* __restrict__ g,
                               const T* __restrict__ s, int64_t tokens, int k, int64_t d, T* __restrict__ out) {
    const int64_t t = blockIdx.y;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < d; i += int64_t(gridDim.x) * blockDim.x)
        out[t * d + i] = combine_one(y + (t * k) * d + i, d, w + t * k, k, g[t], s[t * d + i]);
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
    if (x_dtype == SMOE_F16)
        router_kernel<__half><<<grid, 256, 0, st>>>(w, static_cast<const __half*>(x), tokens, experts, hidden, logits);
    else if (x_dtype == SMOE_F32)
        router_kernel<float><<<grid, 256, 0, st>>>(w, static_cast<const float*>(x), tokens, experts, hidden, logits);
    else
        return fail(SMOE_EDTYPE, "router activations must be float16 or float32");
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
    if (dtype == SMOE_F16)
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
