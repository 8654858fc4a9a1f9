// Products read straight from GGUF blocks: dequant, the pair matvec (gate/up/down of decoding), the down
// matvec with SwiGLU formed in shared memory, and a standalone SwiGLU.
//
// Matvec layout (B200): a CTA of 8 warps takes one pair and a run of rows of that pair's expert. The pair's
// activation row is staged once in shared memory as float32; each warp streams its rows' bytes into its own
// shared-memory slots with 16-byte cp.async copies (coalesced, all issued up front so every warp has several
// KB in flight), then its lanes decode runs of 32 weights in registers and reduce with warp shuffles.
#include <type_traits>

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

    // 2. the pair's activations as float32. Run n's eight float4 chunks are stored permuted (chunk v at
    // v ^ (n & 7)): the lanes of a warp each read their own run, 128 bytes apart, and without the permutation
    // every 16-byte read of eight lanes would fall on the same four banks.
    const auto at = [](int64_t c) {
        const int64_t n = c >> 5;
        return (n << 5) | ((((c >> 2) & 7) ^ (n & 7)) << 2) | (c & 3);
    };
    if (a.gate != nullptr) {
        const T* g = a.gate + p * a.cols;
        const T* u = a.up + p * a.cols;
        for (int64_t c = threadIdx.x; c < a.cols; c += kMvThreads) xs[at(c)] = to_f32(swiglu_one(g[c], u[c]));
    } else {
        const T* x = a.x + (p / a.share) * a.cols;
        for (int64_t c = threadIdx.x; c < a.cols; c += kMvThreads) xs[at(c)] = to_f32(x[c]);
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
            Staged<B>::run(row, n, w);
            const float4* xv = reinterpret_cast<const float4*>(xs + 32 * n);
            float s = 0.0f;
#pragma unroll
            for (int v = 0; v < 8; ++v) {
                const float4 xq = xv[v ^ (n & 7)];
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

// ---------------------------------------------------------------- matvec on int8 dot products
//
// The K-types with float16 activations. Every weight of a run is a small integer q times a float scale of its
// 32 (or 16) weights, less a float minimum of them (gguf-py quants.py:404-552): w = dl q - ml. The pair's
// activations are split once into two int8 vectors, x = s (hi + lo / 128) with s = max|x| / 127 (|x - that|
// <= s / 256), so a run's sum is dl s (sum q hi + sum q lo / 128) - ml sum x: the integer sums exact in int32,
// four products a dp4a, and the float work once per 16 or 32 weights. Results stay within 1e-3 of the largest
// value of the float64 product, the bar of the tensor-core kernels.

// the 32 activations of run n sit in two 16-byte chunks, the chunks of runs n and n + 4 in swapped order, so
// that the 8 lanes of a quarter warp (runs n .. n + 7, 32 bytes apart) read 8 different bank groups
__device__ __forceinline__ int x8_at(int c) {
    const int n = c >> 5;
    return (n << 5) | ((((c >> 4) & 1) ^ ((n >> 2) & 1)) << 4) | (c & 15);
}

// four bytes at byte position p of a row slot (any alignment; reads the aligned word after them too)
__device__ __forceinline__ uint32_t slot_word(const uint32_t* sw, int p) {
    return __funnelshift_r(sw[p >> 2], sw[(p >> 2) + 1], 8u * static_cast<uint32_t>(p & 3));
}
// eight consecutive words from byte position p
__device__ __forceinline__ void slot_words8(const uint32_t* sw, int p, uint32_t (&w)[8]) {
    const uint32_t sh = 8u * static_cast<uint32_t>(p & 3);
    const uint32_t* a = sw + (p >> 2);
    uint32_t r[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) r[i] = a[i];
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = __funnelshift_r(r[i], r[i + 1], sh);
}
__device__ __forceinline__ float slot_half(const uint32_t* sw, int p) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(slot_word(sw, p) & 0xffffu)));
}

// s (H + L / 128): a sum of q x from the integer sums against hi and lo
__device__ __forceinline__ float x8_sum(int hsum, int lsum, float s) {
    return s * fmaf(float(lsum), 0.0078125f, float(hsum));
}

// Dot8<B>::run: run n of a row in a slot (sw: the slot's words, p: the byte position of the row's block), the
// run's activations h / l (eight words of int8 each) and the sums of x over its two 16-column halves
template <class B>
struct Dot8 {
    static constexpr bool kTaken = false;
};

template <>
struct Dot8<Q4_K> {
    static constexpr bool kTaken = true, kMins = true;
    __device__ static float run(const uint32_t* sw, const uint8_t* b, int p, int n, const uint32_t (&h)[8],
                                const uint32_t (&l)[8], const float* sx, float s) {
        const int t = n & 7;
        float sc, mn;
        k4_scale_min(b + 4, t, sc, mn);
        const float dl = mul_rn(slot_half(sw, p), sc), ml = mul_rn(slot_half(sw, p + 2), mn);
        uint32_t q[8];
        slot_words8(sw, p + 16 + 32 * (t >> 1), q);
        const int shift = 4 * (t & 1);
        int hs = 0, ls = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int v = static_cast<int>((q[i] >> shift) & 0x0F0F0F0Fu);
            hs = __dp4a(v, static_cast<int>(h[i]), hs);
            ls = __dp4a(v, static_cast<int>(l[i]), ls);
        }
        return fmaf(dl, x8_sum(hs, ls, s), -ml * (sx[0] + sx[1]));
    }
};

template <>
struct Dot8<Q5_K> {
    static constexpr bool kTaken = true, kMins = true;
    __device__ static float run(const uint32_t* sw, const uint8_t* b, int p, int n, const uint32_t (&h)[8],
                                const uint32_t (&l)[8], const float* sx, float s) {
        const int t = n & 7;
        float sc, mn;
        k4_scale_min(b + 4, t, sc, mn);
        const float dl = mul_rn(slot_half(sw, p), sc), ml = mul_rn(slot_half(sw, p + 2), mn);
        uint32_t q[8], qh[8];
        slot_words8(sw, p + 48 + 32 * (t >> 1), q);
        slot_words8(sw, p + 16, qh);
        const int shift = 4 * (t & 1);
        int hs = 0, ls = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int v = static_cast<int>(((q[i] >> shift) & 0x0F0F0F0Fu) | (((qh[i] >> t) & 0x01010101u) << 4));
            hs = __dp4a(v, static_cast<int>(h[i]), hs);
            ls = __dp4a(v, static_cast<int>(l[i]), ls);
        }
        return fmaf(dl, x8_sum(hs, ls, s), -ml * (sx[0] + sx[1]));
    }
};

template <>
struct Dot8<Q6_K> {
    static constexpr bool kTaken = true, kMins = false;
    __device__ static float run(const uint32_t* sw, const uint8_t* b, int p, int n, const uint32_t (&h)[8],
                                const uint32_t (&l)[8], const float*, float s) {
        const int r = n & 7, hh = r >> 2, sub = r & 3;
        uint32_t ql[8], qh[8];
        slot_words8(sw, p + 64 * hh + 32 * (sub & 1), ql);
        slot_words8(sw, p + 128 + 32 * hh, qh);
        const int lshift = 4 * (sub >> 1), hshift = 2 * sub;
        const float d = slot_half(sw, p + 208);
        float acc = 0.0f;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const float dsc = mul_rn(d, float(int8_t(b[192 + 2 * r + half])));
            int hs = 0, ls = 0;
#pragma unroll
            for (int i = 4 * half; i < 4 * half + 4; ++i) {
                const uint32_t u = ((ql[i] >> lshift) & 0x0F0F0F0Fu) | (((qh[i] >> hshift) & 0x03030303u) << 4);
                const int v = static_cast<int>(__vsub4(u, 0x20202020u));  // q - 32 in each byte
                hs = __dp4a(v, static_cast<int>(h[i]), hs);
                ls = __dp4a(v, static_cast<int>(l[i]), ls);
            }
            acc = fmaf(dsc, x8_sum(hs, ls, s), acc);
        }
        return acc;
    }
};

template <>
struct Dot8<Q2_K> {
    static constexpr bool kTaken = true, kMins = true;
    __device__ static float run(const uint32_t* sw, const uint8_t* b, int p, int n, const uint32_t (&h)[8],
                                const uint32_t (&l)[8], const float* sx, float s) {
        const int r = n & 7;
        uint32_t q[8];
        slot_words8(sw, p + 16 + 32 * (r >> 2), q);
        const int shift = 2 * (r & 3);
        const float d = slot_half(sw, p + 80), dmin = slot_half(sw, p + 82);
        float acc = 0.0f;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const uint32_t sc = b[2 * r + half];
            const float dl = mul_rn(d, float(sc & 15)), ml = mul_rn(dmin, float(sc >> 4));
            int hs = 0, ls = 0;
#pragma unroll
            for (int i = 4 * half; i < 4 * half + 4; ++i) {
                const int v = static_cast<int>((q[i] >> shift) & 0x03030303u);
                hs = __dp4a(v, static_cast<int>(h[i]), hs);
                ls = __dp4a(v, static_cast<int>(l[i]), ls);
            }
            acc = fmaf(dl, x8_sum(hs, ls, s), fmaf(-ml, sx[half], acc));
        }
        return acc;
    }
};

template <>
struct Dot8<Q3_K> {
    static constexpr bool kTaken = true, kMins = false;
    __device__ static float run(const uint32_t* sw, const uint8_t* b, int p, int n, const uint32_t (&h)[8],
                                const uint32_t (&l)[8], const float*, float s) {
        const int r = n & 7;
        uint32_t q[8], hm[8];
        slot_words8(sw, p + 32 + 32 * (r >> 2), q);
        slot_words8(sw, p, hm);
        const int shift = 2 * (r & 3);
        const float d = slot_half(sw, p + 108);
        float acc = 0.0f;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const float dl = mul_rn(d, Q3_K::scale(b + 96, 2 * r + half));
            int hs = 0, ls = 0;
#pragma unroll
            for (int i = 4 * half; i < 4 * half + 4; ++i) {
                // q + 4 where bit r of hmask is set, q where it is clear; less 4
                const uint32_t u = ((q[i] >> shift) & 0x03030303u) | (((hm[i] >> r) & 0x01010101u) << 2);
                const int v = static_cast<int>(__vsub4(u, 0x04040404u));
                hs = __dp4a(v, static_cast<int>(h[i]), hs);
                ls = __dp4a(v, static_cast<int>(l[i]), ls);
            }
            acc = fmaf(dl, x8_sum(hs, ls, s), acc);
        }
        return acc;
    }
};

template <class B>
__global__ void __launch_bounds__(kMvThreads) matvec8_kernel(const MatvecArgs<__half> a) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int64_t cols = a.cols;
    int8_t* xh = reinterpret_cast<int8_t*>(smem);
    int8_t* xl = xh + cols;
    float* sx = reinterpret_cast<float*>(smem + 2 * cols);  // sum of x over each 16 columns
    float* red = sx + cols / 16;                             // 8 warps' maxima, then s
    uint8_t* slots = smem + ((2 * cols + (cols / 16) * 4 + 64 + 15) & ~int64_t(15));

    const int prob = blockIdx.z;
    const int64_t p = blockIdx.y;
    const uint32_t e = a.idx[p];
    if (e >= a.experts) return;  // a pair that names no expert is left out
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t rows_per_cta = int64_t(kMvWarps) * a.rows_per_warp;
    const int64_t r0 = blockIdx.x * rows_per_cta + int64_t(warp) * a.rows_per_warp;
    const int nr = static_cast<int>(max(int64_t(0), min(int64_t(a.rows_per_warp), a.rows - r0)));

    // 1. this warp's rows -> its slots
    const uint8_t* base = (prob ? a.blocks[1] : a.blocks[0]) + (int64_t(e) * a.rows) * a.row_bytes;
    uint8_t* my = slots + int64_t(warp) * a.rows_per_warp * a.stage;
    for (int i = 0; i < a.rows_per_warp; ++i) {
        if (i < nr) stage_bytes(my + i * a.stage, base + (r0 + i) * a.row_bytes, a.row_bytes, prob ? a.end[1] : a.end[0], lane, 32);
        cp_async_commit();
    }

    // 2. the pair's activations split into int8 hi / lo with one scale s = max|x| / 127
    const __half* g = a.gate ? a.gate + p * cols : nullptr;
    const __half* u = a.up ? a.up + p * cols : nullptr;
    const __half* x = a.gate ? nullptr : a.x + (p / a.share) * cols;
    const auto value = [&](int64_t c) { return __half2float(g ? swiglu_one(g[c], u[c]) : x[c]); };
    uint32_t m = 0;  // max |x| as bits (non-negative floats order as integers; a NaN orders above inf)
    for (int64_t c = threadIdx.x; c < cols; c += kMvThreads) m = max(m, __float_as_uint(fabsf(value(c))));
    m = __reduce_max_sync(0xffffffffu, m);
    if (lane == 0) reinterpret_cast<uint32_t*>(red)[warp] = m;
    __syncthreads();
    m = 0;
#pragma unroll
    for (int w = 0; w < kMvWarps; ++w) m = max(m, reinterpret_cast<uint32_t*>(red)[w]);
    const float xmax = __uint_as_float(m);
    const float s = xmax / 127.0f;  // (inf or NaN when x is: the products come out NaN)
    const float inv = xmax > 0.0f ? 127.0f / xmax : 0.0f;
    for (int64_t c = threadIdx.x; c < cols; c += kMvThreads) {
        const float v = value(c) * inv;
        const float hi = rintf(v);
        const int at = x8_at(static_cast<int>(c));
        xh[at] = static_cast<int8_t>(__float2int_rn(hi));
        xl[at] = static_cast<int8_t>(__float2int_rn((v - hi) * 128.0f));
    }
    __syncthreads();
    if constexpr (Dot8<B>::kMins) {
        for (int64_t gi = threadIdx.x; gi < cols / 16; gi += kMvThreads) {
            int hs = 0, ls = 0;
            for (int j = 0; j < 16; ++j) {
                const int at = x8_at(static_cast<int>(16 * gi + j));
                hs += xh[at];
                ls += xl[at];
            }
            sx[gi] = x8_sum(hs, ls, s);
        }
        __syncthreads();
    }

    // 3. decode and reduce, a row at a time as its bytes land
    const int runs = static_cast<int>(cols >> 5);
    __half* out = (prob ? a.out[1] : a.out[0]) + p * a.rows;
    const uint4* xh4 = reinterpret_cast<const uint4*>(xh);
    const uint4* xl4 = reinterpret_cast<const uint4*>(xl);
    for (int i = 0; i < nr; ++i) {
        cp_async_wait_dyn(a.rows_per_warp - 1 - i);
        __syncwarp();
        const int off = static_cast<int>(reinterpret_cast<uintptr_t>(base + (r0 + i) * a.row_bytes) & 15);
        const uint8_t* slot = my + i * a.stage;
        const uint32_t* sw = reinterpret_cast<const uint32_t*>(slot);
        float acc = 0.0f;
        for (int n = lane; n < runs; n += 32) {
            const int swz = (n >> 2) & 1;
            const uint4 h0 = xh4[2 * n + swz], h1 = xh4[2 * n + (swz ^ 1)];
            const uint4 l0 = xl4[2 * n + swz], l1 = xl4[2 * n + (swz ^ 1)];
            const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
            const uint32_t lw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
            const int pos = off + (n >> 3) * B::kBytes;
            acc += Dot8<B>::run(sw, slot + pos, pos, n, hw, lw, sx + 2 * n, s);
        }
        acc = warp_sum(acc);
        if (lane == 0) out[r0 + i] = __float2half_rn(acc);
    }
}

template <typename T>
__global__ void swiglu_kernel(const T* __restrict__ g, const T* __restrict__ u, int64_t n, T* __restrict__ out) {
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        out[i] = swiglu_one(g[i], u[i]);
}

// float32 gate and up, float16 out: the float32 SwiGLU rounded once to float16
__global__ void swiglu_to_half_kernel(const float* __restrict__ g, const float* __restrict__ u, int64_t n,
                                      __half* __restrict__ out) {
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        out[i] = __float2half_rn(swiglu_one(g[i], u[i]));
}

// the two above eight values a thread (n a multiple of 8, 16-byte aligned), in 16-byte loads and stores
template <typename T, typename O>
__global__ void swiglu8_kernel(const T* __restrict__ g, const T* __restrict__ u, int64_t n, O* __restrict__ out) {
    constexpr int kVec = 16 / sizeof(T);  // values a 16-byte load holds
    for (int64_t i = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) * 8; i < n;
         i += int64_t(gridDim.x) * blockDim.x * 8) {
        T gv[8], uv[8];
#pragma unroll
        for (int c = 0; c < 8 / kVec; ++c) {
            *reinterpret_cast<uint4*>(gv + c * kVec) = *reinterpret_cast<const uint4*>(g + i + c * kVec);
            *reinterpret_cast<uint4*>(uv + c * kVec) = *reinterpret_cast<const uint4*>(u + i + c * kVec);
        }
        O ov[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const T h = swiglu_one(gv[e], uv[e]);
            if constexpr (std::is_same<O, T>::value) ov[e] = h;
            else ov[e] = __float2half_rn(h);
        }
#pragma unroll
        for (int c = 0; c < int(8 * sizeof(O)) / 16; ++c)
            *reinterpret_cast<uint4*>(out + i + c * (16 / sizeof(O))) = *reinterpret_cast<const uint4*>(ov + c * (16 / sizeof(O)));
    }
}

static bool aligned8(int64_t n, const void* a, const void* b, const void* c) {
    return n % 8 == 0 && ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                           reinterpret_cast<uintptr_t>(c)) & 15) == 0;
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
    // (+16: the staged decoders read whole aligned words, up to 3 bytes past the end of a row's slot)
    int64_t smem = xs_bytes + int64_t(kMvWarps) * rpw * a.stage + 16;
    SMOE_REQUIRE(smem <= 200 * 1024, SMOE_ESHAPE, "rows too long for the staged matvec");
    a.rows_per_warp = rpw;
    const int64_t rows_per_cta = int64_t(kMvWarps) * rpw;
    dim3 grid(static_cast<unsigned>((a.rows + rows_per_cta - 1) / rows_per_cta), static_cast<unsigned>(a.pairs), nprob);
    SMOE_REQUIRE(a.pairs <= 65535, SMOE_ESHAPE, "more than 65535 pairs in one matvec call");
    int status = dispatch_kind(kind0, [&](auto blk) {
        using B = decltype(blk);
        if constexpr (sizeof(T) == 2 && Dot8<B>::kTaken) {
            // the int8 activations, the sums of x per 16 columns and 8 maxima take the float32 row's place
            const int64_t xs8 = (2 * a.cols + (a.cols / 16) * 4 + 64 + 15) & ~int64_t(15);
            const int64_t smem8 = smem - xs_bytes + xs8;
            auto kern = matvec8_kernel<B>;
            max_smem(kern, static_cast<int>(smem8));
            kern<<<grid, kMvThreads, smem8, st>>>(a);
            return;
        }
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

namespace {
// smoe_matvec_batch's checks, and the problems one int8 tensor-core launch takes: `one` when all are float16
// and at most four compute (spec[0 .. m)), with up to two L2 fetches for a later launch (pref[0 .. npf)).
int batch_specs(int n, const SmoeMatvec* pr, M8Spec* spec, int& m, M8Pref* pref, int& npf, bool& one) {
    SMOE_REQUIRE(n >= 0 && n <= 64, SMOE_EARG, "a batch holds 0 to 64 problems");
    m = npf = 0;
    one = false;
    if (n == 0) return SMOE_OK;
    SMOE_REQUIRE(pr != nullptr, SMOE_EARG, "null problem list");
    // every problem checked as its own entry point checks it, before any launch
    int ncomp = 0;
    for (int i = 0; i < n; ++i) ncomp += pr[i].out != nullptr ? 1 : 0;
    one = ncomp <= 4;
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
        if (p.dtype != SMOE_F16) one = false;
        if (one)
            spec[m++] = M8Spec{p.kind, p.blocks, p.experts, p.rows, p.cols, p.cols / per * bytes, p.idx, p.pairs,
                               p.x ? p.share : 1, static_cast<const __half*>(p.x), static_cast<const __half*>(p.gate),
                               static_cast<const __half*>(p.up), static_cast<__half*>(p.out)};
    }
    return SMOE_OK;
}

// the problems through their own entry points: a problem and the next one of the same kind and shape on the
// same pairs and activations (a gate / up pair) in one launch, the others one by one
int batch_each(int n, const SmoeMatvec* pr, void* stream) {
    for (int i = 0; i < n; ++i) {
        const SmoeMatvec& p = pr[i];
        if (p.pairs == 0 || p.out == nullptr) continue;
        if (p.x != nullptr && i + 1 < n) {
            const SmoeMatvec& q = pr[i + 1];
            if (q.out != nullptr && q.x == p.x && q.kind == p.kind && q.experts == p.experts && q.rows == p.rows &&
                q.cols == p.cols && q.idx == p.idx && q.pairs == p.pairs && q.share == p.share && q.dtype == p.dtype) {
                const int r = smoe_matvec_gate_up(p.kind, p.blocks, q.kind, q.blocks, p.experts, p.rows, p.cols, p.idx,
                                                  p.pairs, p.share, p.x, p.out, q.out, p.dtype, stream);
                if (r) return r;
                ++i;
                continue;
            }
        }
        const int r = p.x ? smoe_matvec(p.kind, p.blocks, p.experts, p.rows, p.cols, p.idx, p.pairs, p.share, p.x,
                                        p.out, p.dtype, stream)
                          : smoe_matvec_glu(p.kind, p.blocks, p.experts, p.rows, p.cols, p.idx, p.pairs, p.gate,
                                            p.up, p.out, p.dtype, stream);
        if (r) return r;
    }
    return SMOE_OK;
}
}  // namespace

extern "C" int smoe_matvec_batch(int n, const SmoeMatvec* pr, void* stream) {
    M8Spec spec[4];
    M8Pref pref[2];
    int m = 0, npf = 0;
    bool one_launch = false;
    if (int s = batch_specs(n, pr, spec, m, pref, npf, one_launch)) return s;
    cudaStream_t st = as_stream(stream);
    if (one_launch && m > 0) {
        const M8Spec& a = spec[0];
        const int r = m == 1 && npf == 0
                          ? mv8_try(a.kind, a.kind, a.blocks, a.blocks, a.experts, a.rows, a.cols, a.row_bytes, a.idx,
                                    a.pairs, a.share, a.x, a.gate, a.up, a.out, a.out, 1, st)
                          : mv8_batch(m, spec, st, npf, pref);
        if (r != 1) return r;
    }
    return batch_each(n, pr, stream);
}

// [0] the fused launch's arrivals, [1] its launch number, then smoe_route's counters (the two calls' form)
extern "C" size_t smoe_route_step_counters(int64_t tokens) {
    return (8 + smoe_route_counters(tokens) + 15) & ~size_t(15);
}

extern "C" int smoe_route_matvec_batch(const SmoeRouteStep* r, int n, const SmoeMatvec* pr, void* stream) {
    SMOE_REQUIRE(r != nullptr, SMOE_EARG, "null route");
    SMOE_REQUIRE(r->tokens >= 0, SMOE_EARG, "negative token count");
    if (r->tokens == 0) return SMOE_OK;  // (no tokens: no pairs)
    SMOE_REQUIRE(r->lidx == nullptr || (r->lo >= 0 && r->count >= 0 && r->lo + r->count <= r->experts &&
                                        r->count < (int64_t(1) << 31)),
                 SMOE_EARG, "route: this rank's experts [lo, lo + count) lie within the router's");
    M8Spec spec[4];
    M8Pref pref[2];
    int m = 0, npf = 0;
    bool one_launch = false;
    if (int s = batch_specs(n, pr, spec, m, pref, npf, one_launch)) return s;
    cudaStream_t st = as_stream(stream);
    if (one_launch && m > 0 && r->x_dtype == SMOE_F16 && r->weight && r->x && r->logits && r->idx && r->weights &&
        r->counters && r->experts > 0 && r->k > 0) {
        M8Route R{};
        R.w = reinterpret_cast<const __half*>(r->weight);
        R.gw = reinterpret_cast<const __half*>(r->gate_weight);
        R.x = static_cast<const __half*>(r->x);
        R.logits = r->logits;
        R.idx = r->idx;
        R.weights = r->weights;
        R.gate_out = static_cast<__half*>(r->gate_out);
        R.counters = r->counters;
        R.lidx = r->lidx;
        R.lo = static_cast<uint32_t>(r->lidx ? r->lo : 0);
        R.count = static_cast<uint32_t>(r->lidx ? r->count : 0);
        R.tokens = static_cast<int>(std::min<int64_t>(r->tokens, 1 << 20));
        R.experts = static_cast<int>(std::min<int64_t>(r->experts, 1 << 20));
        R.hidden = static_cast<int>(std::min<int64_t>(r->hidden, 1 << 30));
        R.k = static_cast<int>(std::min<int64_t>(r->k, 1 << 20));
        const int res = mv8_batch(m, spec, st, npf, pref, &R);
        if (res != 1) return res;
    }
    // the route alone, then the products
    uint32_t* rc = r->counters ? r->counters + 2 : nullptr;
    const int s = r->lidx ? smoe_route_local(r->weight, r->gate_weight, r->x, r->x_dtype, r->tokens, r->experts,
                                             r->hidden, r->k, r->logits, r->idx, r->weights, r->gate_out, rc, r->lo,
                                             r->count, r->lidx, stream)
                          : smoe_route(r->weight, r->gate_weight, r->x, r->x_dtype, r->tokens, r->experts, r->hidden,
                                       r->k, r->logits, r->idx, r->weights, r->gate_out, rc, stream);
    if (s) return s;
    return smoe_matvec_batch(n, pr, stream);
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

extern "C" int smoe_swiglu_to(const void* gate, const void* up, int64_t n, int dtype, void* out, int out_dtype,
                              void* stream) {
    if (dtype == out_dtype) return smoe_swiglu(gate, up, n, out, dtype, stream);
    if (n == 0) return SMOE_OK;
    SMOE_REQUIRE(gate && up && out && n > 0, SMOE_EARG, "null pointer or negative size");
    SMOE_REQUIRE(dtype == SMOE_F32 && out_dtype == SMOE_F16, SMOE_EDTYPE,
                 "swiglu_to takes float32 gate and up to float16, or one type throughout");
    if (aligned8(n, gate, up, out)) {
        const unsigned grid8 = static_cast<unsigned>(std::min<int64_t>((n / 8 + 255) / 256, 148 * 16));
        swiglu8_kernel<float, __half><<<grid8, 256, 0, as_stream(stream)>>>(
            static_cast<const float*>(gate), static_cast<const float*>(up), n, static_cast<__half*>(out));
        return launch_status("swiglu_to");
    }
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 148 * 16));
    swiglu_to_half_kernel<<<grid, 256, 0, as_stream(stream)>>>(static_cast<const float*>(gate),
                                                               static_cast<const float*>(up), n, static_cast<__half*>(out));
    return launch_status("swiglu_to");
}

extern "C" int smoe_swiglu(const void* gate, const void* up, int64_t n, void* out, int dtype, void* stream) {
    if (n == 0) return SMOE_OK;
    SMOE_REQUIRE(gate && up && out && n > 0, SMOE_EARG, "null pointer or negative size");
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 148 * 16));
    const unsigned grid8 = static_cast<unsigned>(std::min<int64_t>((n / 8 + 255) / 256, 148 * 16));
    cudaStream_t st = as_stream(stream);
    if (dtype == SMOE_F16 && aligned8(n, gate, up, out))
        swiglu8_kernel<__half, __half><<<grid8, 256, 0, st>>>(static_cast<const __half*>(gate),
                                                              static_cast<const __half*>(up), n, static_cast<__half*>(out));
    else if (dtype == SMOE_F32 && aligned8(n, gate, up, out))
        swiglu8_kernel<float, float><<<grid8, 256, 0, st>>>(static_cast<const float*>(gate),
                                                            static_cast<const float*>(up), n, static_cast<float*>(out));
    else if (dtype == SMOE_F16)
        swiglu_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(gate), static_cast<const __half*>(up), n,
                                                   static_cast<__half*>(out));
    else if (dtype == SMOE_F32)
        swiglu_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(gate), static_cast<const float*>(up), n,
                                                  static_cast<float*>(out));
    else
        return fail(SMOE_EDTYPE, "activations must be float16 or float32");
    return launch_status("swiglu");
}
