// Products read straight from GGUF blocks: dequant, the pair matvec (gate/up/down of decoding), the down
// matvec with SwiGLU formed in shared memory, and a standalone SwiGLU.
//
// Matvec layout (B200): a CTA of 8 warps takes one pair and a run of rows of that pair's expert. The pair's
// activation row is staged once in shared memory as float32; each warp streams its rows' bytes into its own
// shared-memory slots with 16-byte cp.async copies (coalesced, all issued up front so every warp has several
// KB in flight), then its lanes decode runs of 32 weights in registers and reduce with warp shuffles.
#include "blocks.cuh"
#include "mv8.cuh"

namespace smoe {

// ---------------------------------------------------------------- dequant

template <class B, typename OT>
__global__ void dequant_kernel(const uint8_t* __restrict__ blocks, int64_t total_runs, int runs_per_row,
                               int64_t row_bytes, OT* __restrict__ out) {
    const int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= total_runs) return;
    const int64_t row = t / runs_per_row;
    const int n = static_cast<int>(t - row * runs_per_row);
    float w[32];
    B::run(blocks + row * row_bytes, n, w);
    OT* o = out + t * 32;  // row * cols + 32 n
    if constexpr (sizeof(OT) == 2) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            __align__(16) __half h[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) h[j] = __float2half_rn(w[8 * v + j]);
            reinterpret_cast<uint4*>(o)[v] = *reinterpret_cast<const uint4*>(h);
        }
    } else {
#pragma unroll
        for (int v = 0; v < 8; ++v)
            reinterpret_cast<float4*>(o)[v] = make_float4(w[4 * v], w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
    }
}

// ---------------------------------------------------------------- matvec

constexpr int kMvWarps = 8;
constexpr int kMvThreads = 32 * kMvWarps;

template <typename T>
struct MatvecArgs {
    const uint8_t* blocks[2];
    const uint8_t* end[2];  // one past each stack's last byte
    T* out[2];
    const uint32_t* idx;
    const T* x;      // (pairs / share, cols), or null when gate/up are given
    const T* gate;   // (pairs, cols): the activations are swiglu(gate, up)
    const T* up;
    int64_t experts, rows, cols, row_bytes, pairs, share;
    int rows_per_warp;  // rows a warp streams at once (<= 4)
    int stage;          // bytes of one row slot (row_bytes + 16, rounded to 16)
};

template <class B, typename T>
__global__ void __launch_bounds__(kMvThreads) matvec_kernel(const MatvecArgs<T> a) {
    extern __shared__ __align__(16) uint8_t smem[];
    float* xs = reinterpret_cast<float*>(smem);
    uint8_t* slots = smem + ((a.cols * 4 + 15) & ~int64_t(15));

    const int prob = blockIdx.z;
    const int64_t p = blockIdx.y;
    const uint32_t e = a.idx[p];
    if (e >= a.experts) return;  // a pair that names no expert is left out
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t rows_per_cta = int64_t(kMvWarps) * a.rows_per_warp;
    const int64_t r0 = blockIdx.x * rows_per_cta + int64_t(warp) * a.rows_per_warp;
    const int nr = static_cast<int>(max(int64_t(0), min(int64_t(a.rows_per_warp), a.rows - r0)));

    // 1. this warp's rows -> its slots (every lane commits one group per row, empty or not)
    const uint8_t* base = (prob ? a.blocks[1] : a.blocks[0]) + (int64_t(e) * a.rows) * a.row_bytes;
    uint8_t* my = slots + int64_t(warp) * a.rows_per_warp * a.stage;
    for (int i = 0; i < a.rows_per_warp; ++i) {
        if (i < nr) stage_bytes(my + i * a.stage, base + (r0 + i) * a.row_bytes, a.row_bytes, prob ? a.end[1] : a.end[0], lane, 32);
        cp_async_commit();
    }

    // 2. the pair's activations as float32
    if (a.gate != nullptr) {
        const T* g = a.gate + p * a.cols;
        const T* u = a.up + p * a.cols;
        for (int64_t c = threadIdx.x; c < a.cols; c += kMvThreads) xs[c] = to_f32(swiglu_one(g[c], u[c]));
    } else {
        const T* x = a.x + (p / a.share) * a.cols;
        for (int64_t c = threadIdx.x; c < a.cols; c += kMvThreads) xs[c] = to_f32(x[c]);
    }
    __syncthreads();

    // 3. decode and reduce, a row at a time as its bytes land
    const int runs = static_cast<int>(a.cols >> 5);
    T* out = (prob ? a.out[1] : a.out[0]) + p * a.rows;
    for (int i = 0; i < nr; ++i) {
        cp_async_wait_dyn(a.rows_per_warp - 1 - i);
        __syncwarp();
        const int off = static_cast<int>(reinterpret_cast<uintptr_t>(base + (r0 + i) * a.row_bytes) & 15);
        const uint8_t* row = my + i * a.stage + off;
        float acc = 0.0f;
        for (int n = lane; n < runs; n += 32) {
            float w[32];
            B::run(row, n, w);
            const float4* xv = reinterpret_cast<const float4*>(xs + 32 * n);
            float s = 0.0f;
#pragma unroll
            for (int v = 0; v < 8; ++v) {
                const float4 xq = xv[v];
                s = fmaf(w[4 * v], xq.x, s);
                s = fmaf(w[4 * v + 1], xq.y, s);
                s = fmaf(w[4 * v + 2], xq.z, s);
                s = fmaf(w[4 * v + 3], xq.w, s);
            }
            acc += s;
        }
        acc = warp_sum(acc);
        if (lane == 0) out[r0 + i] = from_f32<T>(acc);
    }
}

template <typename T>
__global__ void swiglu_kernel(const T* __restrict__ g, const T* __restrict__ u, int64_t n, T* __restrict__ out) {
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        out[i] = swiglu_one(g[i], u[i]);
}

// ---------------------------------------------------------------- host side

// the float16 tensor-core decode matvec (smoe_mv.cu), for what the int8 one does not take
int mv_mma_try(int kind0, int kind1, const uint8_t* b0, const uint8_t* b1, int64_t experts, int64_t rows, int64_t cols,
               int64_t row_bytes, const uint32_t* idx, int64_t pairs, int64_t share, const __half* x, __half* o0,
               __half* o1, int nprob, cudaStream_t st);

static int check_stack(int kind, int64_t experts, int64_t rows, int64_t cols, int& per, int& bytes) {
    if (!block_info(kind, per, bytes)) return fail(SMOE_EKIND, "block type " + std::to_string(kind) + " has no decoder");
    SMOE_REQUIRE(experts > 0 && rows > 0 && cols > 0, SMOE_ESHAPE, "empty stack");
    SMOE_REQUIRE(cols % per == 0, SMOE_ESHAPE,
                 "rows of " + std::to_string(cols) + " weights do not end on a block of " + std::to_string(per));
    return SMOE_OK;
}

template <typename T>
static int launch_matvec(int kind0, int kind1, MatvecArgs<T> a, int nprob, cudaStream_t st) {
    SMOE_REQUIRE(kind0 == kind1, SMOE_EKIND, "gate and up stacks of different types are not supported yet");
    const int64_t xs_bytes = (a.cols * 4 + 15) & ~int64_t(15);
    a.stage = static_cast<int>((a.row_bytes + 16 + 15) & ~int64_t(15));
    // about 64 KB of rows in flight per CTA, at most 4 rows a warp
    int rpw = static_cast<int>(std::min<int64_t>(4, std::max<int64_t>(1, (64 << 10) / (int64_t(kMvWarps) * a.stage))));
    int64_t smem = xs_bytes + int64_t(kMvWarps) * rpw * a.stage;
    SMOE_REQUIRE(smem <= 200 * 1024, SMOE_ESHAPE, "rows too long for the staged matvec");
    a.rows_per_warp = rpw;
    const int64_t rows_per_cta = int64_t(kMvWarps) * rpw;
    dim3 grid(static_cast<unsigned>((a.rows + rows_per_cta - 1) / rows_per_cta), static_cast<unsigned>(a.pairs), nprob);
    SMOE_REQUIRE(a.pairs <= 65535, SMOE_ESHAPE, "more than 65535 pairs in one matvec call");
    int status = dispatch_kind(kind0, [&](auto blk) {
        using B = decltype(blk);
        auto kern = matvec_kernel<B, T>;
        max_smem(kern, static_cast<int>(smem));
        kern<<<grid, kMvThreads, smem, st>>>(a);
    });
    if (status != SMOE_OK) return fail(status, "block type has no decoder");
    return launch_status("matvec");
}

template <typename T>
static int matvec_common(int kind0, const uint8_t* b0, int kind1, const uint8_t* b1, int64_t experts, int64_t rows,
                         int64_t cols, const uint32_t* idx, int64_t pairs, int64_t share, const void* x, const void* gate,
                         const void* up, void* out0, void* out1, int nprob, cudaStream_t st) {
    int per, bytes;
    if (int s = check_stack(kind0, experts, rows, cols, per, bytes)) return s;
    if (pairs == 0) return SMOE_OK;
    SMOE_REQUIRE(pairs > 0 && idx && b0 && out0, SMOE_EARG, "null pointer or negative pair count");
    SMOE_REQUIRE(share >= 1, SMOE_EARG, "share must be >= 1");
    SMOE_REQUIRE((reinterpret_cast<uintptr_t>(x ? x : gate) & 15) == 0, SMOE_EARG, "activations must be 16-byte aligned");
    MatvecArgs<T> a{};
    a.blocks[0] = b0;
    a.blocks[1] = b1 ? b1 : b0;
    a.row_bytes = cols / per * bytes;
    a.end[0] = b0 + experts * rows * a.row_bytes;
    a.end[1] = a.blocks[1] + experts * rows * a.row_bytes;
    a.out[0] = static_cast<T*>(out0);
    a.out[1] = static_cast<T*>(out1 ? out1 : out0);
    a.idx = idx;
    a.x = static_cast<const T*>(x);
    a.gate = static_cast<const T*>(gate);
    a.up = static_cast<const T*>(up);
    a.experts = experts;
    a.rows = rows;
    a.cols = cols;
    a.pairs = pairs;
    a.share = share;
    if constexpr (sizeof(T) == 2) {
        const int r8 = mv8_try(kind0, kind1, b0, a.blocks[1], experts, rows, cols, a.row_bytes, idx, pairs, share,
                               static_cast<const __half*>(x), static_cast<const __half*>(gate),
                               static_cast<const __half*>(up), a.out[0], a.out[1], nprob, st);
        if (r8 != 1) return r8;
        if (gate == nullptr) {
            const int r = mv_mma_try(kind0, kind1, b0, a.blocks[1], experts, rows, cols, a.row_bytes, idx, pairs, share,
                                     static_cast<const __half*>(x), a.out[0], a.out[1], nprob, st);
            if (r != 1) return r;
        }
    }
    return launch_matvec<T>(kind0, kind1, a, nprob, st);
}

}  // namespace smoe

using namespace smoe;

extern "C" int smoe_dequant(int kind, const uint8_t* blocks, int64_t n_rows, int64_t cols, void* out, int out_dtype,
                            void* stream) {
    int per, bytes;
    if (int s = check_stack(kind, 1, n_rows, cols, per, bytes)) return s;
    SMOE_REQUIRE(blocks && out, SMOE_EARG, "null pointer");
    SMOE_REQUIRE((reinterpret_cast<uintptr_t>(out) & 15) == 0, SMOE_EARG, "out must be 16-byte aligned");
    SMOE_REQUIRE(out_dtype == SMOE_F16 || out_dtype == SMOE_F32, SMOE_EDTYPE, "dequant writes float16 or float32");
    const int runs = static_cast<int>(cols / 32);
    const int64_t total = n_rows * runs;
    const int64_t row_bytes = cols / per * bytes;
    const unsigned grid = static_cast<unsigned>((total + 255) / 256);
    cudaStream_t st = as_stream(stream);
    int status = dispatch_kind(kind, [&](auto blk) {
        using B = decltype(blk);
        if (out_dtype == SMOE_F16)
            dequant_kernel<B, __half><<<grid, 256, 0, st>>>(blocks, total, runs, row_bytes, static_cast<__half*>(out));
        else
            dequant_kernel<B, float><<<grid, 256, 0, st>>>(blocks, total, runs, row_bytes, static_cast<float*>(out));
    });
    if (status) return fail(status, "block type has no decoder");
    return launch_status("dequant");
}

extern "C" int smoe_matvec(int kind, const uint8_t* blocks, int64_t experts, int64_t rows, int64_t cols,
                           const uint32_t* idx, int64_t pairs, int64_t share, const void* x, void* out, int dtype,
                           void* stream) {
    SMOE_REQUIRE(x != nullptr, SMOE_EARG, "null activations");
    if (dtype == SMOE_F16)
        return matvec_common<__half>(kind, blocks, kind, nullptr, experts, rows, cols, idx, pairs, share, x, nullptr,
                                     nullptr, out, nullptr, 1, as_stream(stream));
    if (dtype == SMOE_F32)
        return matvec_common<float>(kind, blocks, kind, nullptr, experts, rows, cols, idx, pairs, share, x, nullptr,
                                    nullptr, out, nullptr, 1, as_stream(stream));
    return fail(SMOE_EDTYPE, "activations must be float16 or float32");
}

extern "C" int smoe_matvec_batch(int n, const SmoeMatvec* pr, void* stream) {
    SMOE_REQUIRE(n >= 0 && n <= 64, SMOE_EARG, "a batch holds 0 to 64 problems");
    if (n == 0) return SMOE_OK;
    SMOE_REQUIRE(pr != nullptr, SMOE_EARG, "null problem list");
    // every problem checked as its own entry point checks it, before any launch
    M8Spec spec[4];
    M8Pref pref[2];
    int m = 0, npf = 0, ncomp = 0;
    for (int i = 0; i < n; ++i) ncomp += pr[i].out != nullptr ? 1 : 0;
    bool one_launch = ncomp <= 4;
    for (int i = 0; i < n; ++i) {
        const SmoeMatvec& p = pr[i];
        int per, bytes;
        if (int s = check_stack(p.kind, p.experts, p.rows, p.cols, per, bytes)) return s;
        if (p.out == nullptr) {
            // a prefetch: the experts' blocks named by idx, fetched into L2 for a later launch
            SMOE_REQUIRE(p.x == nullptr && p.gate == nullptr && p.up == nullptr, SMOE_EARG,
                         "a problem without out has no activations (it names weights to fetch ahead)");
            if (p.pairs > 0 && p.blocks && p.idx && npf < 2 && p.pairs < (int64_t(1) << 30))
                pref[npf++] = M8Pref{p.blocks, p.rows * (p.cols / per * bytes), p.idx, static_cast<int>(p.pairs),
                                     static_cast<uint32_t>(std::min<int64_t>(p.experts, 0xffffffffLL))};
            continue;
        }
        SMOE_REQUIRE(p.pairs >= 0, SMOE_EARG, "negative pair count");
        SMOE_REQUIRE((p.x != nullptr) != (p.gate != nullptr && p.up != nullptr), SMOE_EARG,
                     "a problem has x, or gate and up");
        SMOE_REQUIRE(p.dtype == SMOE_F16 || p.dtype == SMOE_F32, SMOE_EDTYPE, "activations must be float16 or float32");
        if (p.pairs == 0) continue;
        SMOE_REQUIRE(p.blocks && p.idx && p.out, SMOE_EARG, "null pointer");
        SMOE_REQUIRE(p.x == nullptr || p.share >= 1, SMOE_EARG, "share must be >= 1");
        if (p.dtype != SMOE_F16) one_launch = false;
        if (one_launch)
            spec[m++] = M8Spec{p.kind, p.blocks, p.experts, p.rows, p.cols, p.cols / per * bytes, p.idx, p.pairs,
                               p.x ? p.share : 1, static_cast<const __half*>(p.x), static_cast<const __half*>(p.gate),
                               static_cast<const __half*>(p.up), static_cast<__half*>(p.out)};
    }
    cudaStream_t st = as_stream(stream);
    if (one_launch && m > 0) {
        const M8Spec& a = spec[0];
        const int r = m == 1 && npf == 0
                          ? mv8_try(a.kind, a.kind, a.blocks, a.blocks, a.experts, a.rows, a.cols, a.row_bytes, a.idx,
                                    a.pairs, a.share, a.x, a.gate, a.up, a.out, a.out, 1, st)
                          : mv8_batch(m, spec, st, npf, pref);
        if (r != 1) return r;
    }
    for (int i = 0; i < n; ++i) {
        const SmoeMatvec& p = pr[i];
        if (p.pairs == 0 || p.out == nullptr) continue;
        const int r = p.x ? smoe_matvec(p.kind, p.blocks, p.experts, p.rows, p.cols, p.idx, p.pairs, p.share, p.x,
                                        p.out, p.dtype, stream)
                          : smoe_matvec_glu(p.kind, p.blocks, p.experts, p.rows, p.cols, p.idx, p.pairs, p.gate,
                                            p.up, p.out, p.dtype, stream);
        if (r) return r;
    }
    return SMOE_OK;
}

extern "C" int smoe_matvec_glu_combine(int kind, const uint8_t* blocks, int64_t rows, int64_t cols,
                                       const uint32_t* idx, int64_t tokens, const void* gate, const void* up,
                                       const void* y, const float* w, const void* g, int64_t k, void* out, int dtype,
                                       void* stream) {
    int per, bytes;
    if (int s = check_stack(kind, 1, rows, cols, per, bytes)) return s;
    if (tokens == 0) return SMOE_OK;
    SMOE_REQUIRE(tokens > 0 && blocks && idx && gate && up && y && w && g && out, SMOE_EARG, "null pointer");
    SMOE_REQUIRE(k >= 1 && k <= 64, SMOE_ESHAPE, "1 <= k <= 64");
    SMOE_REQUIRE(dtype == SMOE_F16, SMOE_EDTYPE, "the fused combine takes float16 activations");
    const int r = mv8_glu_combine(kind, blocks, rows, cols, cols / per * bytes, idx, tokens,
                                  static_cast<const __half*>(gate), static_cast<const __half*>(up),
                                  static_cast<const __half*>(y), w, static_cast<const __half*>(g), static_cast<int>(k),
                                  static_cast<__half*>(out), as_stream(stream));
    if (r == 1) return fail(SMOE_ESHAPE, "the fused combine does not take this stack (IQ3_S or Q8_0, columns a "
                                         "multiple of 256, activations within its shared memory)");
    return r;
}

extern "C" int smoe_matvec_gate_up(int gate_kind, const uint8_t* gate_blocks, int up_kind, const uint8_t* up_blocks,
                                   int64_t experts, int64_t rows, int64_t cols, const uint32_t* idx, int64_t pairs,
                                   int64_t share, const void* x, void* gate_out, void* up_out, int dtype, void* stream) {
    SMOE_REQUIRE(x && up_blocks && up_out, SMOE_EARG, "null pointer");
    if (dtype == SMOE_F16)
        return matvec_common<__half>(gate_kind, gate_blocks, up_kind, up_blocks, experts, rows, cols, idx, pairs, share, x,
                                     nullptr, nullptr, gate_out, up_out, 2, as_stream(stream));
    if (dtype == SMOE_F32)
        return matvec_common<float>(gate_kind, gate_blocks, up_kind, up_blocks, experts, rows, cols, idx, pairs, share, x,
                                    nullptr, nullptr, gate_out, up_out, 2, as_stream(stream));
    return fail(SMOE_EDTYPE, "activations must be float16 or float32");
}

extern "C" int smoe_matvec_glu(int kind, const uint8_t* blocks, int64_t experts, int64_t rows, int64_t cols,
                               const uint32_t* idx, int64_t pairs, const void* gate, const void* up, void* out, int dtype,
                               void* stream) {
    SMOE_REQUIRE(gate && up, SMOE_EARG, "null gate or up");
    if (dtype == SMOE_F16)
        return matvec_common<__half>(kind, blocks, kind, nullptr, experts, rows, cols, idx, pairs, 1, nullptr, gate, up,
                                     out, nullptr, 1, as_stream(stream));
    if (dtype == SMOE_F32)
        return matvec_common<float>(kind, blocks, kind, nullptr, experts, rows, cols, idx, pairs, 1, nullptr, gate, up,
                                    out, nullptr, 1, as_stream(stream));
    return fail(SMOE_EDTYPE, "activations must be float16 or float32");
}

extern "C" int smoe_swiglu(const void* gate, const void* up, int64_t n, void* out, int dtype, void* stream) {
    if (n == 0) return SMOE_OK;
    SMOE_REQUIRE(gate && up && out && n > 0, SMOE_EARG, "null pointer or negative size");
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 148 * 16));
    cudaStream_t st = as_stream(stream);
    if (dtype == SMOE_F16)
        swiglu_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(gate), static_cast<const __half*>(up), n,
                                                   static_cast<__half*>(out));
    else if (dtype == SMOE_F32)
        swiglu_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(gate), static_cast<const float*>(up), n,
                                                  static_cast<float*>(out));
    else
        return fail(SMOE_EDTYPE, "activations must be float16 or float32");
    return launch_status("swiglu");
}
