// Device pieces of the int8 tensor-core decode matvec shared by its kernels (smoe_mv8.cu) and the fused decode
// layer (smoe_layer.cu): the block types' stage decoders, the codebook fill, the activation split.
#pragma once

#include <cuda.h>

#include "blocks.cuh"
#include "tc05.cuh"

namespace smoe {

constexpr int kM8Warps = 16;
constexpr int kM8Threads = 32 * kM8Warps;
constexpr int kM8MaxSlots = 4;
constexpr int kM8XBlock = 256;                   // columns per activation scale
constexpr uint32_t kM8WaitLimit = 1u << 22;

__device__ __forceinline__ void mma_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ uint32_t lds_u16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }
__device__ __forceinline__ uint32_t lds_u8(const uint8_t* p) { return *p; }
__device__ __forceinline__ float h2f(uint32_t bits) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits & 0xffffu)));
}

// ---------------------------------------------------------------- IQ3_S
// (110 bytes: d 0, qs 2..65, qh 66..73, signs 74..105, scales 106..109.) In run r, lane tig of a row's quad
// takes groups 2 tig and 2 tig + 1 (weights 8 tig .. 8 tig + 7 of the run): K 4 tig .. 4 tig + 3 of the MMA is
// group 2 tig, K 16 + 4 tig .. is group 2 tig + 1, the same permutation for the activations.
//
// A group's four weights are the grid word of its 9-bit index (qs byte | qh bit << 8) with the group's four
// signs applied. The grid (512 words) sits in shared memory REP times over, word i * REP + lane % REP, so a
// warp's 32 random lookups meet at most 32 / REP to a bank. Every grid value is odd, so negating a byte is xor with
// 0xFE: a sign byte's bits (two groups') become 0x00 / 0xFF bytes by one multiply per group (each bit to
// the top of a byte) and a sign-replicating byte permute.

template <int O>
__device__ __forceinline__ uint32_t ld_s16(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u16 %0, [%1+%2];" : "=r"(v) : "r"(a), "n"(O));
    return v;
}
template <int O>
__device__ __forceinline__ uint32_t ld_s8(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u8 %0, [%1+%2];" : "=r"(v) : "r"(a), "n"(O));
    return v;
}
__device__ __forceinline__ uint32_t ld_s32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
// prmt.b32 in its default mode: a selector nibble with bit 3 set replicates the top bit of the chosen byte
__device__ __forceinline__ uint32_t prmt_sr(uint32_t a, uint32_t c) {
    uint32_t d;
    asm("prmt.b32 %0, %1, 0, %2;" : "=r"(d) : "r"(a), "r"(c));
    return d;
}
constexpr int kM8GridRep = 16;  // copies of the IQ3_S grid in shared memory (the matvec kernels')

// NB blocks a stage: two (512 columns, 16 rows of 220 bytes in 240-byte rows of the ring slot) where the
// width allows, else one (110 bytes in 144)
template <int NB, int REP = kM8GridRep>
struct M8IQ3S {
    static constexpr int kKind = 21, kStageCols = 256 * NB, kStageBytes = 110 * NB, kRS = NB == 2 ? 240 : 144;
    static constexpr bool kLut = true, kTokens = false;
    // run R of the stage: the two rows' groups (bq / bs: the lane's qs / sign bytes), lutl = this lane's grid copy
    template <int R>
    __device__ static __forceinline__ void run(const uint32_t (&bq)[2], const uint32_t (&bs)[2], const uint32_t (&qh)[2][2],
                                               const uint32_t (&m)[2][2], uint32_t lutl, const uint8_t* xsrc, int tig,
                                               int gid, int (&t)[2]) {
        uint32_t a[2][2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const uint32_t q2 = ld_s16<2 + 8 * R>(bq[j]);  // qs bytes of the two groups
            const uint32_t sb = ld_s8<74 + 4 * R>(bs[j]);   // their sign nibbles
            // byte R % 4 of the shifted qh word: bits 0, 1 are the groups' (the rest never reach the index)
            const uint32_t h = __byte_perm(qh[j][R >> 2], 0u, 0x4440 + (R & 3));
            // both grid indices in one word: qs | qh << 8 in each half
            const uint32_t z = __byte_perm(q2, 0u, 0x4140) | ((h * 0x00800100u) & 0x01000100u);
            const uint32_t ga = ld_s32(lutl + (z & 0x1ffu) * (4 * REP));
            const uint32_t gb = ld_s32(lutl + (z >> 16) * (4 * REP));
            // sign masks: each of the byte's 8 bits moved to the top of a byte by one multiply (copies of sb at
            // 9-bit strides never overlap), bytes reordered and their top bits replicated by one permute
            const uint32_t ma = prmt_sr(sb * 0x80402010u, 0x89ABu);  // bits 0..3 (group 2 tig)
            const uint32_t mb = prmt_sr(sb * 0x08040201u, 0x89ABu);  // bits 4..7 (group 2 tig + 1)
            a[j][0] = ga ^ (ma & 0xFEFEFEFEu);
            a[j][1] = gb ^ (mb & 0xFEFEFEFEu);
        }
        uint2 b = make_uint2(0u, 0u);
        if (gid < 2) b = *reinterpret_cast<const uint2*>(xsrc + 32 * R + 8 * tig);
        int acc[4];
        mma_s8(acc, a[0][0], a[1][0], a[0][1], a[1][1], b.x, b.y);
        // (lanes with tig > 0 hold columns 2..7: zeros)
        const int m0 = static_cast<int>(__byte_perm(m[0][R & 1], 0u, 0x4440 + (R >> 1)));
        const int m1 = static_cast<int>(__byte_perm(m[1][R & 1], 0u, 0x4440 + (R >> 1)));
        t[0] += m0 * (acc[0] * 128 + acc[1]);
        t[1] += m1 * (acc[2] * 128 + acc[3]);
    }
    // one block of rows gid (j = 0) and gid + 8 (j = 1): partial sums of the two rows
    __device__ static __forceinline__ void block(const uint8_t* r0, const uint8_t* r1, int tig, int gid,
                                                 const uint32_t* lut, const uint8_t* xh, const uint8_t* xl, float xs,
                                                 float (&total)[2]) {
        const uint32_t rb[2] = {smem_addr(r0), smem_addr(r1)};
        const uint32_t lutl = smem_addr(lut) + 4u * static_cast<uint32_t>((4 * gid + tig) & (REP - 1));
        uint32_t m[2][2], qh[2][2], bq[2], bs[2];
        float d[2];
        int t[2] = {0, 0};
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            d[j] = h2f(ld_s16<0>(rb[j]));
            // the runs' odd sub-scales 1 + 2 s as bytes: runs 0, 2, 4, 6 in m[j][0], runs 1, 3, 5, 7 in m[j][1]
            const uint32_t sc = ld_s16<106>(rb[j]) | (ld_s16<108>(rb[j]) << 16);
            m[j][0] = ((sc & 0x0F0F0F0Fu) << 1) | 0x01010101u;
            m[j][1] = ((sc >> 3) & 0x1E1E1E1Eu) | 0x01010101u;
            // qh bits of groups 2 tig, 2 tig + 1 of run r at bits 8 (r % 4), 8 (r % 4) + 1 of word r / 4
            qh[j][0] = (ld_s16<66>(rb[j]) | (ld_s16<68>(rb[j]) << 16)) >> (2 * tig);
            qh[j][1] = (ld_s16<70>(rb[j]) | (ld_s16<72>(rb[j]) << 16)) >> (2 * tig);
            bq[j] = rb[j] + 2u * tig;
            bs[j] = rb[j] + tig;
        }
        const uint8_t* xsrc = gid == 0 ? xh : xl;
        run<0>(bq, bs, qh, m, lutl, xsrc, tig, gid, t);
        run<1>(bq, bs, qh, m, lutl, xsrc, tig, gid, t);
        run<2>(bq, bs, qh, m, lutl, xsrc, tig, gid, t);
        run<3>(bq, bs, qh, m, lutl, xsrc, tig, gid, t);
        run<4>(bq, bs, qh, m, lutl, xsrc, tig, gid, t);
        run<5>(bq, bs, qh, m, lutl, xsrc, tig, gid, t);
        run<6>(bq, bs, qh, m, lutl, xsrc, tig, gid, t);
        run<7>(bq, bs, qh, m, lutl, xsrc, tig, gid, t);
        const float k = xs * (1.0f / 128.0f);
        total[0] = fmaf(d[0] * k, static_cast<float>(t[0]), total[0]);
        total[1] = fmaf(d[1] * k, static_cast<float>(t[1]), total[1]);
    }
    // one stage: NB blocks, each with its own activation scale (xs[0], xs[1])
    __device__ static void stage(const uint8_t* r0, const uint8_t* r1, int tig, int gid, const uint32_t* lut,
                                 const uint8_t* xh, const uint8_t* xl, const float* xs, float (&total)[2]) {
        block(r0, r1, tig, gid, lut, xh, xl, xs[0], total);
        if constexpr (NB == 2) block(r0 + 110, r1 + 110, tig, gid, lut, xh + 256, xl + 256, xs[1], total);
    }
};

// the IQ3_S grid (entries 0..511 of the sign-folded table built from gguf-py's grid: sign bits 0), REP times
// over (word i * REP + copy): 2 KB x REP
template <int REP = kM8GridRep>
__device__ __forceinline__ void m8_fill_grid(uint32_t* lut) {
    for (int i = threadIdx.x; i < 512 * REP / 4; i += blockDim.x) {
        const uint32_t g = __ldg(kIq3sSigned + (4 * i) / REP);
        reinterpret_cast<uint4*>(lut)[i] = make_uint4(g, g, g, g);
    }
}

// ---------------------------------------------------------------- Q8_0
// (34 bytes: d 0, qs 2..33.) A stage is four runs; in run r lane tig takes codes 8 tig .. 8 tig + 7.
struct M8Q8_0 {
    static constexpr int kKind = 8, kStageCols = 128, kStageBytes = 136, kRS = 176;
    static constexpr bool kLut = false, kTokens = true;
    __device__ static void stage(const uint8_t* r0, const uint8_t* r1, int tig, int gid, const uint32_t*,
                                 const uint8_t* xh, const uint8_t* xl, const float* xs, float (&total)[2]) {
        const uint8_t* rb[2] = {r0, r1};
        const uint8_t* xsrc = gid == 0 ? xh : xl;
        const float k = xs[0] * (1.0f / 128.0f);  // (a stage lies within one 256-column scale block)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            uint32_t a[2][2];
            float d[2];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const uint8_t* p = rb[j] + 34 * r + 2 + 8 * tig;
                const uint32_t* w = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(p) & ~uintptr_t(3));
                const uint32_t sh = 8u * static_cast<uint32_t>(reinterpret_cast<uintptr_t>(p) & 3u);
                const uint32_t w0 = w[0], w1 = w[1], w2 = w[2];
                a[j][0] = __funnelshift_r(w0, w1, sh);
                a[j][1] = __funnelshift_r(w1, w2, sh);
                d[j] = h2f(lds_u16(rb[j] + 34 * r));
            }
            uint2 b = make_uint2(0u, 0u);
            if (gid < 2) b = *reinterpret_cast<const uint2*>(xsrc + 32 * r + 8 * tig);
            int acc[4];
            mma_s8(acc, a[0][0], a[1][0], a[0][1], a[1][1], b.x, b.y);
            total[0] = fmaf(d[0] * k, static_cast<float>(acc[0] * 128 + acc[1]), total[0]);
            total[1] = fmaf(d[1] * k, static_cast<float>(acc[2] * 128 + acc[3]), total[1]);
        }
    }
    // The same stage for nt <= 4 tokens of one expert, their activation rows xstride bytes (and xsstride
    // scales) apart: column 2t of B holds token t's hi, column 2t + 1 its lo, so lane tig of a quad receives
    // token tig's two sums, and its total is token tig's (tig < nt). One pass over the weights for all nt.
    __device__ static void stage_tokens(const uint8_t* r0, const uint8_t* r1, int tig, int gid, const uint8_t* xh,
                                        const uint8_t* xl, int64_t xstride, const float* xs, int xsstride, int nt,
                                        float (&total)[2]) {
        const uint8_t* rb[2] = {r0, r1};
        const int t = gid >> 1;
        const uint8_t* xsrc = ((gid & 1) ? xl : xh) + int64_t(t) * xstride;
        const float k = tig < nt ? xs[tig * xsstride] * (1.0f / 128.0f) : 0.0f;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            uint32_t a[2][2];
            float d[2];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const uint8_t* p = rb[j] + 34 * r + 2 + 8 * tig;
                const uint32_t* w = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(p) & ~uintptr_t(3));
                const uint32_t sh = 8u * static_cast<uint32_t>(reinterpret_cast<uintptr_t>(p) & 3u);
                const uint32_t w0 = w[0], w1 = w[1], w2 = w[2];
                a[j][0] = __funnelshift_r(w0, w1, sh);
                a[j][1] = __funnelshift_r(w1, w2, sh);
                d[j] = h2f(lds_u16(rb[j] + 34 * r));
            }
            uint2 b = make_uint2(0u, 0u);
            if (t < nt) b = *reinterpret_cast<const uint2*>(xsrc + 32 * r + 8 * tig);
            int acc[4];
            mma_s8(acc, a[0][0], a[1][0], a[0][1], a[1][1], b.x, b.y);
            total[0] = fmaf(d[0] * k, static_cast<float>(acc[0] * 128 + acc[1]), total[0]);
            total[1] = fmaf(d[1] * k, static_cast<float>(acc[2] * 128 + acc[3]), total[1]);
        }
    }
};

// Eight values a lane of one 256-column block (a warp) split into int8 hi and lo and the block's scale:
// v = s (hi + lo / 128), s = max|v| / 127.
__device__ __forceinline__ void m8_split_values(const float (&v)[8], int8_t* hi, int8_t* lo, float* scale, int lane) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float s = amax / 127.0f, inv = amax > 0.f ? 127.0f / amax : 0.f;
    uint32_t hw[2] = {0u, 0u}, lw[2] = {0u, 0u};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float hf = fminf(fmaxf(rintf(v[i] * inv), -127.f), 127.f);
        const float lf = fminf(fmaxf(rintf((v[i] - hf * s) * (128.0f * inv)), -127.f), 127.f);
        hw[i >> 2] |= (static_cast<uint32_t>(static_cast<int>(hf)) & 255u) << (8 * (i & 3));
        lw[i >> 2] |= (static_cast<uint32_t>(static_cast<int>(lf)) & 255u) << (8 * (i & 3));
    }
    *reinterpret_cast<uint2*>(hi) = make_uint2(hw[0], hw[1]);
    *reinterpret_cast<uint2*>(lo) = make_uint2(lw[0], lw[1]);
    if (lane == 0) *scale = s;
}

// One 256-column block of an activation row split into int8 hi and lo and its scale, by one warp (8 values a
// lane, from element `at`). With gate set, v = swiglu(gate, up) (the same function, so the same float16 bits,
// as the separate SwiGLU kernel).
__device__ __forceinline__ void m8_split(const __half* x, const __half* gate, const __half* up, int64_t at,
                                         int8_t* hi, int8_t* lo, float* scale, int lane) {
    float v[8];
    if (gate) {
        const uint4 gr = *reinterpret_cast<const uint4*>(gate + at);
        const uint4 ur = *reinterpret_cast<const uint4*>(up + at);
        const __half* gh = reinterpret_cast<const __half*>(&gr);
        const __half* uh = reinterpret_cast<const __half*>(&ur);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __half2float(swiglu_one(gh[i], uh[i]));
    } else {
        const uint4 raw = *reinterpret_cast<const uint4*>(x + at);
        const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(h2[i]);
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    }
    m8_split_values(v, hi, lo, scale, lane);
}

}  // namespace smoe
