// The dense steps on either side of the MoE block in a decode pass:
//
//   hyper-connection  the read of the four residual streams before a block and the write of the block before it
//                     (strata_mlx/fused.py:46-131, 280-323): norm, projection down, projection up and mix;
//   Q3_K planes       a Q3_K tensor's blocks rearranged once into aligned planes, a window of tokens multiplied
//                     on them, their weights as floats (strata_mlx/blocks.py:399-512);
//   Q6_K parts        a Q6_K tensor as a signed byte a weight, a scale per 16 and d per 256 (ScaledLinear,
//                     strata_mlx/dense.py:109-167; parts as strata_mlx/gguf.py:150-165 makes them), a window of
//                     tokens multiplied on them, their weights as floats.
//
// Every product sums in float32 in an order fixed by the tensor's shape alone, so a token gets the same bits
// alone as in a window (the reference's rule for these kernels, strata_mlx/fused.py:40, blocks.py:487-488).
// All of them are small and bound by latency or by the bytes of the weights: one launch each, overlapped with
// the launch before by programmatic dependent launch.
#include <algorithm>

#include "blocks.cuh"

namespace smoe {
namespace {

constexpr int kDnThreads = 256;
constexpr int kDnTok = 8;  // tokens a pass of the window products keeps in registers

// ---- block reductions in a fixed order (xor tree in each warp, then the warps in order)

__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.0f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += red[w];
    return t;
}

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]);
template <>
__device__ __forceinline__ void load8<__half>(const __half* p, float (&v)[8]) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
    }
}
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&v)[8]) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p)), b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}

// ---------------------------------------------------------------- hyper-connection

// One (stream, token) a CTA: h = before + out * inject_in; the residual h in T, normed = h rsqrt(mean h^2 + eps)
// norm in float32 (strata_mlx/fused.py:63-90).
template <typename T>
__global__ void __launch_bounds__(kDnThreads) hc_norm_kernel(const T* __restrict__ before, const T* __restrict__ out,
                                                             const T* __restrict__ inject_in, const T* __restrict__ norm,
                                                             int hc, int d, float eps, T* __restrict__ residual,
                                                             float* __restrict__ normed) {
    __shared__ float red[kDnThreads / 32];
    const int s = blockIdx.x, t = blockIdx.y;
    const int64_t wide = int64_t(hc) * d;
    pdl_wait();
    const float back = to_f32(inject_in[int64_t(t) * hc + s]);
    const T* b = before + int64_t(t) * wide + int64_t(s) * d;
    const T* o = out + int64_t(t) * d;
    float sq = 0.0f;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float h = fmaf(to_f32(o[i]), back, to_f32(b[i]));
        sq = fmaf(h, h, sq);
    }
    const float total = block_sum(sq, red);
    const float scale = rsqrtf(total / static_cast<float>(d) + eps);
    T* res = residual + int64_t(t) * wide + int64_t(s) * d;
    float* nrm = normed + int64_t(t) * wide + int64_t(s) * d;
    const T* nw = norm + int64_t(s) * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float h = fmaf(to_f32(o[i]), back, to_f32(b[i]));
        res[i] = from_f32<T>(h);
        nrm[i] = h * scale * to_f32(nw[i]);
    }
    pdl_release();
}

// One row of `down` (or of the inject weight) a CTA, every token of the window: total = row . normed / hc; a
// down row gives low = total sigmoid(total), an inject row inject = 2 sigmoid(total) in T
// (strata_mlx/fused.py:92-119).
template <typename T>
__global__ void __launch_bounds__(kDnThreads) hc_down_kernel(const float* __restrict__ normed, const T* __restrict__ down,
                                                             const T* __restrict__ inject_w, int rank, int hc,
                                                             int64_t wide, int tokens, float* __restrict__ low,
                                                             T* __restrict__ inject) {
    __shared__ float red[kDnThreads / 32];
    const int j = blockIdx.x;
    const T* row = j < rank ? down + int64_t(j) * wide : inject_w + int64_t(j - rank) * wide;
    pdl_wait();
    for (int t0 = 0; t0 < tokens; t0 += kDnTok) {
        const int nt = min(kDnTok, tokens - t0);
        float acc[kDnTok];
#pragma unroll
        for (int tt = 0; tt < kDnTok; ++tt) acc[tt] = 0.0f;
        for (int64_t i = int64_t(threadIdx.x) * 8; i < wide; i += int64_t(blockDim.x) * 8) {
            float w[8];
            load8(row + i, w);
#pragma unroll
            for (int tt = 0; tt < kDnTok; ++tt) {
                if (tt < nt) {
                    const float4* x = reinterpret_cast<const float4*>(normed + int64_t(t0 + tt) * wide + i);
                    const float4 a = x[0], b = x[1];
                    float v = acc[tt];
                    v = fmaf(w[0], a.x, v), v = fmaf(w[1], a.y, v), v = fmaf(w[2], a.z, v), v = fmaf(w[3], a.w, v);
                    v = fmaf(w[4], b.x, v), v = fmaf(w[5], b.y, v), v = fmaf(w[6], b.z, v), v = fmaf(w[7], b.w, v);
                    acc[tt] = v;
                }
            }
        }
#pragma unroll
        for (int tt = 0; tt < kDnTok; ++tt) {
            if (tt < nt) {  // (uniform over the CTA)
                const float total = block_sum(acc[tt], red) / static_cast<float>(hc);
                if (threadIdx.x == 0) {
                    const float gate = 1.0f / (1.0f + expf(-total));
                    const int t = t0 + tt;
                    if (j < rank) low[int64_t(t) * rank + j] = total * gate;
                    else inject[int64_t(t) * hc + (j - rank)] = from_f32<T>(2.0f * gate);
                }
            }
        }
    }
    pdl_release();
}

// 32 columns a CTA, each with its hc rows of `up` (hc x 32 threads): gate = up[s d + c] . low; the streams'
// normed[s d + c] sigmoid(gate) mixed: mixed[c] = their sum / hc in T (strata_mlx/fused.py:121-146).
template <typename T>
__global__ void hc_up_kernel(const float* __restrict__ normed, const T* __restrict__ up, const float* __restrict__ low,
                             int rank, int hc, int d, int tokens, T* __restrict__ mixed) {
    extern __shared__ float sm[];
    float* lows = sm;                          // [kDnTok][rank]
    float* parts = sm + kDnTok * rank;         // [hc][32][kDnTok]
    const int cc = threadIdx.x & 31, s = threadIdx.x >> 5;
    const int c = blockIdx.x * 32 + cc;
    const int64_t wide = int64_t(hc) * d;
    const int64_t at = int64_t(s) * d + c;
    pdl_wait();
    for (int t0 = 0; t0 < tokens; t0 += kDnTok) {
        const int nt = min(kDnTok, tokens - t0);
        __syncthreads();
        for (int i = threadIdx.x; i < nt * rank; i += blockDim.x) lows[i] = low[int64_t(t0) * rank + i];
        __syncthreads();
        if (c < d) {
            float acc[kDnTok];
#pragma unroll
            for (int tt = 0; tt < kDnTok; ++tt) acc[tt] = 0.0f;
            const T* row = up + at * rank;
            for (int r = 0; r < rank; r += 8) {
                float w[8];
                load8(row + r, w);
#pragma unroll
                for (int tt = 0; tt < kDnTok; ++tt) {
                    if (tt < nt) {
                        const float* l = lows + tt * rank + r;
                        float v = acc[tt];
#pragma unroll
                        for (int q = 0; q < 8; ++q) v = fmaf(w[q], l[q], v);
                        acc[tt] = v;
                    }
                }
            }
#pragma unroll
            for (int tt = 0; tt < kDnTok; ++tt)
                if (tt < nt)
                    parts[(s * 32 + cc) * kDnTok + tt] = normed[int64_t(t0 + tt) * wide + at] / (1.0f + expf(-acc[tt]));
        }
        __syncthreads();
        if (s == 0 && c < d) {
            for (int tt = 0; tt < nt; ++tt) {
                float mix = 0.0f;
                for (int k = 0; k < hc; ++k) mix += parts[(k * 32 + cc) * kDnTok + tt];
                mixed[int64_t(t0 + tt) * d + c] = from_f32<T>(mix / static_cast<float>(hc));
            }
        }
    }
    pdl_release();
}

// ---------------------------------------------------------------- Q3_K planes

// One block a thread: hm (32 bytes as 8 words), qs (64 bytes as 16 words), the 16 six-bit scales less 32 as
// int8, d (strata_mlx/blocks.py:403-414).
__global__ void q3k_planes_kernel(const uint8_t* __restrict__ blocks, int64_t n, uint32_t* __restrict__ hm,
                                  uint32_t* __restrict__ qs, int8_t* __restrict__ sc, uint16_t* __restrict__ dd) {
    for (int64_t b = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; b < n; b += int64_t(gridDim.x) * blockDim.x) {
        const uint8_t* p = blocks + b * Q3_K::kBytes;
#pragma unroll
        for (int w = 0; w < 8; ++w) hm[b * 8 + w] = u32le(p + 4 * w);
#pragma unroll
        for (int w = 0; w < 16; ++w) qs[b * 16 + w] = u32le(p + 32 + 4 * w);
#pragma unroll
        for (int k = 0; k < 16; ++k) sc[b * 16 + k] = static_cast<int8_t>(Q3_K::scale(p + 96, k));
        dd[b] = static_cast<uint16_t>(u16le(p + 108));
    }
}

// Four weights of one run from one word of each plane, packed a byte each: byte k of the qs word holds the run's two
// bits at 2 (rr % 4), byte k of the hm word its high bit at rr; q + 4 h is then 0..7 and the weight (before its
// scale) q + 4 h - 4, as the block decoder has it (a clear high bit subtracts 4).
__device__ __forceinline__ uint32_t q3k_codes4(uint32_t qw, uint32_t hw, int rr) {
    return ((qw >> (2 * (rr & 3))) & 0x03030303u) | (((hw >> rr) & 0x01010101u) << 2);
}
// byte k of packed codes as the float (code - 4), exactly: the byte placed in the mantissa of 2^23
__device__ __forceinline__ float q3k_value(uint32_t codes, int k) {
    return __uint_as_float(__byte_perm(codes, 0x4B000000u, 0x7550u + k)) - 8388612.0f;
}

template <typename T>
__device__ __forceinline__ float4 load4(const T* p);
template <>
__device__ __forceinline__ float4 load4<__half>(const __half* p) {
    const uint2 raw = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
    return make_float4(a.x, a.y, b.x, b.y);
}
template <>
__device__ __forceinline__ float4 load4<float>(const float* p) {
    return *reinterpret_cast<const float4*>(p);
}

// A warp a row; lane l takes the half blocks (128 weights) l, l + 32, ... of the row. Per half: its 8 hm and 8
// qs words and its 8 scales; per run (a 2-bit field of every qs byte) the words give four weights each; every
// token of the window (kDnTok a pass) takes the run's two sub-blocks' sums, scaled once each. Lanes add by an xor
// tree. The split of the row depends on its length only (strata_mlx/blocks.py:426-459).
template <typename T>
__global__ void q3k_window_kernel(const uint32_t* __restrict__ hm, const uint32_t* __restrict__ qs,
                                  const int8_t* __restrict__ sc, const uint16_t* __restrict__ dd, int64_t rows, int cols,
                                  const T* __restrict__ x, int tokens, T* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t r = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    pdl_wait();
    if (r < rows) {
        const int halves = cols / 128;
        for (int t0 = 0; t0 < tokens; t0 += kDnTok) {
            const int nt = min(kDnTok, tokens - t0);
            float sum[kDnTok];
#pragma unroll
            for (int tt = 0; tt < kDnTok; ++tt) sum[tt] = 0.0f;
            for (int h = lane; h < halves; h += 32) {
                const int64_t blk = r * (cols / 256) + (h >> 1);
                const int n = h & 1;
                uint32_t hw[8], qw[8];
                const uint4* hp = reinterpret_cast<const uint4*>(hm + blk * 8);
                const uint4* qp = reinterpret_cast<const uint4*>(qs + blk * 16 + 8 * n);
                const uint4 h0 = __ldg(hp), h1 = __ldg(hp + 1), q0 = __ldg(qp), q1 = __ldg(qp + 1);
                hw[0] = h0.x, hw[1] = h0.y, hw[2] = h0.z, hw[3] = h0.w, hw[4] = h1.x, hw[5] = h1.y, hw[6] = h1.z, hw[7] = h1.w;
                qw[0] = q0.x, qw[1] = q0.y, qw[2] = q0.z, qw[3] = q0.w, qw[4] = q1.x, qw[5] = q1.y, qw[6] = q1.z, qw[7] = q1.w;
                const uint2 scw = __ldg(reinterpret_cast<const uint2*>(sc + blk * 16 + 8 * n));
                const float d = __half2float(__ushort_as_half(__ldg(dd + blk)));
                const T* xh = x + int64_t(t0) * cols + int64_t(h) * 128;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int rr = 4 * n + j;
                    float lo[kDnTok], hi[kDnTok];  // the run's first and second 16 weights
#pragma unroll
                    for (int tt = 0; tt < kDnTok; ++tt) lo[tt] = hi[tt] = 0.0f;
#pragma unroll
                    for (int w = 0; w < 8; ++w) {
                        const uint32_t c = q3k_codes4(qw[w], hw[w], rr);
                        const float v0 = q3k_value(c, 0), v1 = q3k_value(c, 1), v2 = q3k_value(c, 2), v3 = q3k_value(c, 3);
#pragma unroll
                        for (int tt = 0; tt < kDnTok; ++tt) {
                            if (tt < nt) {
                                const float4 xv = load4(xh + int64_t(tt) * cols + 32 * j + 4 * w);
                                float p = v0 * xv.x;
                                p = fmaf(v1, xv.y, p);
                                p = fmaf(v2, xv.z, p);
                                p = fmaf(v3, xv.w, p);
                                if (w < 4) lo[tt] += p;
                                else hi[tt] += p;
                            }
                        }
                    }
                    // scales 2 rr, 2 rr + 1 are bytes 2 j, 2 j + 1 of this half's eight
                    const uint32_t pair = (j < 2 ? scw.x : scw.y) >> (16 * (j & 1));
                    const float s0 = d * float(static_cast<int8_t>(pair & 0xffu));
                    const float s1 = d * float(static_cast<int8_t>((pair >> 8) & 0xffu));
#pragma unroll
                    for (int tt = 0; tt < kDnTok; ++tt) sum[tt] = fmaf(s1, hi[tt], fmaf(s0, lo[tt], sum[tt]));
                }
            }
#pragma unroll
            for (int tt = 0; tt < kDnTok; ++tt) {
                const float total = warp_sum(sum[tt]);
                if (lane == 0 && tt < nt) out[int64_t(t0 + tt) * rows + r] = from_f32<T>(total);
            }
        }
    }
    pdl_release();
}

template <typename T>
__device__ __forceinline__ void store4(T* p, float a, float b, float c, float e);
template <>
__device__ __forceinline__ void store4<float>(float* p, float a, float b, float c, float e) {
    *reinterpret_cast<float4*>(p) = make_float4(a, b, c, e);
}
template <>
__device__ __forceinline__ void store4<__half>(__half* p, float a, float b, float c, float e) {
    const __half2 lo = __floats2half2_rn(a, b), hi = __floats2half2_rn(c, e);
    uint2 v;
    v.x = *reinterpret_cast<const uint32_t*>(&lo);
    v.y = *reinterpret_cast<const uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(p) = v;
}

// A thread four weights: their codes from one qs and one hm word, (d scale) (code - 4) as the block decoder forms
// each weight, rounded once; a vector store (strata_mlx/blocks.py:462-479)
template <typename T>
__global__ void q3k_planes_dequant_kernel(const uint32_t* __restrict__ hm, const uint32_t* __restrict__ qs,
                                          const int8_t* __restrict__ sc, const uint16_t* __restrict__ dd, int64_t quads,
                                          T* __restrict__ out) {
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < quads; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t blk = i >> 6;
        const int at = 4 * static_cast<int>(i & 63);  // the first weight's place in the block
        const int n = at >> 7, j = (at >> 5) & 3, w = (at & 31) >> 2;
        const int rr = 4 * n + j;
        const uint32_t c = q3k_codes4(qs[blk * 16 + 8 * n + w], hm[blk * 8 + w], rr);
        const float s = mul_rn(__half2float(__ushort_as_half(dd[blk])), float(sc[blk * 16 + 2 * rr + (w >> 2)]));
        store4<T>(out + blk * 256 + at, mul_rn(s, q3k_value(c, 0)), mul_rn(s, q3k_value(c, 1)), mul_rn(s, q3k_value(c, 2)),
                  mul_rn(s, q3k_value(c, 3)));
    }
}

// ---------------------------------------------------------------- Q6_K parts (ScaledLinear)

// One block a thread: codes (256 int8, the six bits less 32, in the weights' order), the 16 scales, d
// (strata_mlx/gguf.py:150-165).
__global__ void q6k_parts_kernel(const uint8_t* __restrict__ blocks, int64_t n, int8_t* __restrict__ codes,
                                 int8_t* __restrict__ scales, uint16_t* __restrict__ d) {
    for (int64_t b = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; b < n; b += int64_t(gridDim.x) * blockDim.x) {
        const uint8_t* p = blocks + b * Q6_K::kBytes;
        int8_t* c = codes + b * 256;
        for (int h = 0; h < 2; ++h)
            for (int q = 0; q < 4; ++q)
                for (int l = 0; l < 32; ++l) {
                    const uint32_t lo = (uint32_t(p[64 * h + 32 * (q & 1) + l]) >> (4 * (q >> 1))) & 15u;
                    const uint32_t hi = (uint32_t(p[128 + 32 * h + l]) >> (2 * q)) & 3u;
                    c[128 * h + 32 * q + l] = static_cast<int8_t>(static_cast<int>(lo | (hi << 4)) - 32);
                }
        for (int k = 0; k < 16; ++k) scales[b * 16 + k] = static_cast<int8_t>(p[192 + k]);
        d[b] = static_cast<uint16_t>(u16le(p + 208));
    }
}

// A warp a row, lane l the groups of 16 weights l, l + 32, ...: per group s = d scale and s (codes . x); float32
// (strata_mlx/dense.py:30-72)
template <typename T>
__global__ void scaled_window_kernel(const int8_t* __restrict__ codes, const int8_t* __restrict__ scales,
                                     const uint16_t* __restrict__ dv, int64_t rows, int cols, int d_step,
                                     const T* __restrict__ x, int tokens, T* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t r = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    pdl_wait();
    if (r < rows) {
        const int groups = cols / 16, per_d = cols / d_step;
        for (int t0 = 0; t0 < tokens; t0 += kDnTok) {
            const int nt = min(kDnTok, tokens - t0);
            float sum[kDnTok];
#pragma unroll
            for (int tt = 0; tt < kDnTok; ++tt) sum[tt] = 0.0f;
            for (int g = lane; g < groups; g += 32) {
                const uint4 raw = __ldg(reinterpret_cast<const uint4*>(codes + r * cols) + g);
                const int8_t* cv = reinterpret_cast<const int8_t*>(&raw);
                const float s = __half2float(__ushort_as_half(__ldg(dv + r * per_d + (16 * g) / d_step))) *
                                float(__ldg(scales + r * groups + g));
#pragma unroll
                for (int tt = 0; tt < kDnTok; ++tt) {
                    if (tt < nt) {
                        const T* xr = x + int64_t(t0 + tt) * cols + 16 * g;
                        float a = 0.0f;
#pragma unroll
                        for (int v = 0; v < 16; ++v) a = fmaf(float(cv[v]), to_f32(xr[v]), a);
                        sum[tt] = fmaf(s, a, sum[tt]);
                    }
                }
            }
#pragma unroll
            for (int tt = 0; tt < kDnTok; ++tt) {
                const float total = warp_sum(sum[tt]);
                if (lane == 0 && tt < nt) out[int64_t(t0 + tt) * rows + r] = from_f32<T>(total);
            }
        }
    }
    pdl_release();
}

// every weight: (float(d) * float(scale)) * float(code) rounded once to T (strata_mlx/dense.py:75-84)
template <typename T>
__global__ void scaled_floats_kernel(const int8_t* __restrict__ codes, const int8_t* __restrict__ scales,
                                     const uint16_t* __restrict__ dv, int64_t rows, int cols, int d_step,
                                     T* __restrict__ out) {
    const int64_t groups = int64_t(rows) * (cols / 16);
    for (int64_t g = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; g < groups; g += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = g / (cols / 16), gc = g - r * (cols / 16);
        const float s = mul_rn(__half2float(__ushort_as_half(dv[r * (cols / d_step) + (16 * gc) / d_step])),
                               float(scales[g]));
        const int8_t* c = codes + r * cols + 16 * gc;
        T* o = out + r * cols + 16 * gc;
        for (int i = 0; i < 16; ++i) o[i] = from_f32<T>(mul_rn(s, float(c[i])));
    }
}

unsigned grid_of(int64_t items, int threads) {
    return static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((items + threads - 1) / threads, 148 * 16)));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace
}  // namespace smoe

using namespace smoe;

// ---------------------------------------------------------------- hyper-connection entry points

extern "C" size_t smoe_hyper_workspace_size(int64_t tokens, int64_t hc, int64_t d, int64_t rank) {
    if (tokens < 0 || hc < 1 || d < 1 || rank < 1) return 0;
    return size_t(((tokens * hc * d * 4 + 255) & ~int64_t(255)) + tokens * rank * 4);
}

extern "C" int smoe_hyper_connection(const SmoeHyper* h, const void* before, const void* out, const void* inject_in,
                                     int64_t tokens, void* mixed, void* residual, void* inject, void* workspace,
                                     size_t workspace_bytes, void* stream) {
    SMOE_REQUIRE(h, SMOE_EARG, "hyper_connection: null spec");
    SMOE_REQUIRE(h->hc >= 1 && h->hc <= 8, SMOE_ESHAPE, "hyper_connection: 1 to 8 streams");
    SMOE_REQUIRE(h->d >= 1 && h->d % 8 == 0 && h->rank >= 8 && h->rank % 8 == 0 && h->rank <= 1024, SMOE_ESHAPE,
                 "hyper_connection: d and rank must be multiples of 8 (rank 8..1024)");
    SMOE_REQUIRE(tokens >= 0 && tokens <= 65535, SMOE_ESHAPE, "hyper_connection: too many tokens");
    SMOE_REQUIRE(h->dtype == SMOE_F16 || h->dtype == SMOE_F32, SMOE_EDTYPE, "hyper_connection: float16 or float32");
    if (tokens == 0) return SMOE_OK;
    SMOE_REQUIRE(before && out && inject_in && mixed && residual && h->norm && h->down && h->up, SMOE_EARG,
                 "hyper_connection: null pointer");
    SMOE_REQUIRE(!h->inject_w || inject, SMOE_EARG, "hyper_connection: an inject weight needs an inject output");
    SMOE_REQUIRE(aligned16(h->down) && aligned16(h->up) && (!h->inject_w || aligned16(h->inject_w)), SMOE_EARG,
                 "hyper_connection: weights must be 16-byte aligned");
    SMOE_REQUIRE(workspace && workspace_bytes >= smoe_hyper_workspace_size(tokens, h->hc, h->d, h->rank),
                 SMOE_EWORKSPACE, "hyper_connection: workspace too small");
    const int hc = static_cast<int>(h->hc), d = static_cast<int>(h->d), rank = static_cast<int>(h->rank);
    const int64_t wide = int64_t(hc) * d;
    float* normed = static_cast<float*>(workspace);
    float* low = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + ((tokens * wide * 4 + 255) & ~int64_t(255)));
    const int n_inject = h->inject_w ? hc : 0;
    cudaStream_t st = as_stream(stream);
    const size_t esz = h->dtype == SMOE_F16 ? 2 : 4;
    const size_t up_smem = size_t(kDnTok) * rank * 4 + size_t(hc) * 32 * kDnTok * 4;
    auto go = [&](auto tag) -> int {
        using T = decltype(tag);
        cudaError_t e = launch_pdl(Writes().add(residual, tokens * wide * esz).add(normed, tokens * wide * 4),
                                   hc_norm_kernel<T>, dim3(hc, static_cast<unsigned>(tokens)), dim3(kDnThreads), 0, st,
                                   static_cast<const T*>(before), static_cast<const T*>(out),
                                   static_cast<const T*>(inject_in), static_cast<const T*>(h->norm), hc, d, h->eps,
                                   static_cast<T*>(residual), normed);
        if (e != cudaSuccess) return fail(-static_cast<int>(e), std::string("hc_norm: ") + cudaGetErrorString(e));
        e = launch_pdl(Writes().add(low, tokens * rank * 4).add(n_inject ? inject : nullptr, tokens * hc * esz),
                       hc_down_kernel<T>, dim3(rank + n_inject), dim3(kDnThreads), 0, st, normed,
                       static_cast<const T*>(h->down), static_cast<const T*>(h->inject_w), rank, hc, wide,
                       static_cast<int>(tokens), low, static_cast<T*>(inject));
        if (e != cudaSuccess) return fail(-static_cast<int>(e), std::string("hc_down: ") + cudaGetErrorString(e));
        if (int s = max_smem(hc_up_kernel<T>, static_cast<int>(up_smem))) return fail(s, "hc_up: shared memory");
        e = launch_pdl(Writes().add(mixed, tokens * d * esz), hc_up_kernel<T>, dim3((d + 31) / 32), dim3(32 * hc),
                       up_smem, st, normed, static_cast<const T*>(h->up), low, rank, hc, d, static_cast<int>(tokens),
                       static_cast<T*>(mixed));
        if (e != cudaSuccess) return fail(-static_cast<int>(e), std::string("hc_up: ") + cudaGetErrorString(e));
        return launch_status("hyper_connection");
    };
    return h->dtype == SMOE_F16 ? go(__half()) : go(float());
}

// ---------------------------------------------------------------- Q3_K planes entry points

extern "C" int smoe_q3k_planes(const uint8_t* blocks, int64_t rows, int64_t cols, uint32_t* hm, uint32_t* qs,
                               int8_t* sc, uint16_t* dd, void* stream) {
    SMOE_REQUIRE(rows >= 0 && cols > 0 && cols % 256 == 0, SMOE_ESHAPE, "q3k_planes: rows of whole blocks");
    const int64_t n = rows * (cols / 256);
    if (n == 0) return SMOE_OK;
    SMOE_REQUIRE(blocks && hm && qs && sc && dd, SMOE_EARG, "q3k_planes: null pointer");
    q3k_planes_kernel<<<grid_of(n, 128), 128, 0, as_stream(stream)>>>(blocks, n, hm, qs, sc, dd);
    return launch_status("q3k_planes");
}

extern "C" int smoe_q3k_planes_window(const uint32_t* hm, const uint32_t* qs, const int8_t* sc, const uint16_t* dd,
                                      int64_t rows, int64_t cols, const void* x, int64_t tokens, void* out, int dtype,
                                      void* stream) {
    SMOE_REQUIRE(rows >= 1 && cols > 0 && cols % 256 == 0 && cols <= (1 << 24), SMOE_ESHAPE,
                 "q3k_planes_window: rows of whole blocks");
    if (tokens == 0) return SMOE_OK;
    SMOE_REQUIRE(hm && qs && sc && dd && x && out && tokens > 0, SMOE_EARG, "q3k_planes_window: bad arguments");
    SMOE_REQUIRE(aligned16(x) && aligned16(hm) && aligned16(qs) && (reinterpret_cast<uintptr_t>(sc) & 7) == 0,
                 SMOE_EARG, "q3k_planes_window: activations and planes must be 16-byte aligned (sc 8-byte)");
    const unsigned grid = static_cast<unsigned>((rows * 32 + 255) / 256);
    cudaStream_t st = as_stream(stream);
    cudaError_t e;
    if (dtype == SMOE_F16)
        e = launch_pdl(Writes().add(out, tokens * rows * 2), q3k_window_kernel<__half>, dim3(grid), dim3(256), 0, st,
                       hm, qs, sc, dd, rows, static_cast<int>(cols), static_cast<const __half*>(x),
                       static_cast<int>(tokens), static_cast<__half*>(out));
    else if (dtype == SMOE_F32)
        e = launch_pdl(Writes().add(out, tokens * rows * 4), q3k_window_kernel<float>, dim3(grid), dim3(256), 0, st,
                       hm, qs, sc, dd, rows, static_cast<int>(cols), static_cast<const float*>(x),
                       static_cast<int>(tokens), static_cast<float*>(out));
    else
        return fail(SMOE_EDTYPE, "q3k_planes_window: float16 or float32 activations");
    if (e != cudaSuccess) return fail(-static_cast<int>(e), std::string("q3k_planes_window: ") + cudaGetErrorString(e));
    return launch_status("q3k_planes_window");
}

extern "C" int smoe_q3k_planes_dequant(const uint32_t* hm, const uint32_t* qs, const int8_t* sc, const uint16_t* dd,
                                       int64_t rows, int64_t cols, void* out, int dtype, void* stream) {
    SMOE_REQUIRE(rows >= 0 && cols > 0 && cols % 256 == 0, SMOE_ESHAPE, "q3k_planes_dequant: rows of whole blocks");
    const int64_t quads = rows * cols / 4;
    if (quads == 0) return SMOE_OK;
    SMOE_REQUIRE(hm && qs && sc && dd && out, SMOE_EARG, "q3k_planes_dequant: null pointer");
    SMOE_REQUIRE(aligned16(out), SMOE_EARG, "q3k_planes_dequant: the output must be 16-byte aligned");
    cudaStream_t st = as_stream(stream);
    if (dtype == SMOE_F16)
        q3k_planes_dequant_kernel<__half><<<grid_of(quads, 256), 256, 0, st>>>(hm, qs, sc, dd, quads,
                                                                               static_cast<__half*>(out));
    else if (dtype == SMOE_F32)
        q3k_planes_dequant_kernel<float><<<grid_of(quads, 256), 256, 0, st>>>(hm, qs, sc, dd, quads,
                                                                              static_cast<float*>(out));
    else
        return fail(SMOE_EDTYPE, "q3k_planes_dequant: float16 or float32");
    return launch_status("q3k_planes_dequant");
}

// ---------------------------------------------------------------- Q6_K parts entry points

extern "C" int smoe_q6k_parts(const uint8_t* blocks, int64_t rows, int64_t cols, int8_t* codes, int8_t* scales,
                              uint16_t* d, void* stream) {
    SMOE_REQUIRE(rows >= 0 && cols > 0 && cols % 256 == 0, SMOE_ESHAPE, "q6k_parts: rows of whole blocks");
    const int64_t n = rows * (cols / 256);
    if (n == 0) return SMOE_OK;
    SMOE_REQUIRE(blocks && codes && scales && d, SMOE_EARG, "q6k_parts: null pointer");
    q6k_parts_kernel<<<grid_of(n, 128), 128, 0, as_stream(stream)>>>(blocks, n, codes, scales, d);
    return launch_status("q6k_parts");
}

extern "C" int smoe_scaled_window(const int8_t* codes, const int8_t* scales, const uint16_t* d, int64_t rows,
                                  int64_t cols, int64_t d_step, const void* x, int64_t tokens, void* out, int dtype,
                                  void* stream) {
    SMOE_REQUIRE(rows >= 1 && cols > 0 && cols % 16 == 0 && cols <= (1 << 24), SMOE_ESHAPE,
                 "scaled_window: rows of whole groups of 16");
    SMOE_REQUIRE(d_step >= 16 && d_step % 16 == 0 && cols % d_step == 0, SMOE_ESHAPE,
                 "scaled_window: d must cover whole groups of 16 and divide the row");
    if (tokens == 0) return SMOE_OK;
    SMOE_REQUIRE(codes && scales && d && x && out && tokens > 0, SMOE_EARG, "scaled_window: bad arguments");
    SMOE_REQUIRE(aligned16(codes), SMOE_EARG, "scaled_window: codes must be 16-byte aligned");
    const unsigned grid = static_cast<unsigned>((rows * 32 + 255) / 256);
    cudaStream_t st = as_stream(stream);
    cudaError_t e;
    if (dtype == SMOE_F16)
        e = launch_pdl(Writes().add(out, tokens * rows * 2), scaled_window_kernel<__half>, dim3(grid), dim3(256), 0,
                       st, codes, scales, d, rows, static_cast<int>(cols), static_cast<int>(d_step),
                       static_cast<const __half*>(x), static_cast<int>(tokens), static_cast<__half*>(out));
    else if (dtype == SMOE_F32)
        e = launch_pdl(Writes().add(out, tokens * rows * 4), scaled_window_kernel<float>, dim3(grid), dim3(256), 0,
                       st, codes, scales, d, rows, static_cast<int>(cols), static_cast<int>(d_step),
                       static_cast<const float*>(x), static_cast<int>(tokens), static_cast<float*>(out));
    else
        return fail(SMOE_EDTYPE, "scaled_window: float16 or float32 activations");
    if (e != cudaSuccess) return fail(-static_cast<int>(e), std::string("scaled_window: ") + cudaGetErrorString(e));
    return launch_status("scaled_window");
}

extern "C" int smoe_scaled_floats(const int8_t* codes, const int8_t* scales, const uint16_t* d, int64_t rows,
                                  int64_t cols, int64_t d_step, void* out, int dtype, void* stream) {
    SMOE_REQUIRE(rows >= 0 && cols > 0 && cols % 16 == 0 && d_step >= 16 && d_step % 16 == 0 && cols % d_step == 0,
                 SMOE_ESHAPE, "scaled_floats: rows of whole groups of 16");
    const int64_t groups = rows * (cols / 16);
    if (groups == 0) return SMOE_OK;
    SMOE_REQUIRE(codes && scales && d && out, SMOE_EARG, "scaled_floats: null pointer");
    cudaStream_t st = as_stream(stream);
    if (dtype == SMOE_F16)
        scaled_floats_kernel<__half><<<grid_of(groups, 256), 256, 0, st>>>(codes, scales, d, rows, static_cast<int>(cols),
                                                                           static_cast<int>(d_step),
                                                                           static_cast<__half*>(out));
    else if (dtype == SMOE_F32)
        scaled_floats_kernel<float><<<grid_of(groups, 256), 256, 0, st>>>(codes, scales, d, rows, static_cast<int>(cols),
                                                                          static_cast<int>(d_step),
                                                                          static_cast<float*>(out));
    else
        return fail(SMOE_EDTYPE, "scaled_floats: float16 or float32");
    return launch_status("scaled_floats");
}
