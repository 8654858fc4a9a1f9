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
__device__ __forceinline__ uint32_t lds_u8_at(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u8 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds_u16_at(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=r"(v) : "r"(a));
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
    static constexpr bool kLut = true, kTokens = false, kXsum = false, kHalves = false;
    __device__ static void fill(uint32_t* lut);
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

template <int NB, int REP>
__device__ void M8IQ3S<NB, REP>::fill(uint32_t* lut) {
    m8_fill_grid<REP>(lut);
}

// ---------------------------------------------------------------- IQ4_XS
// (136 bytes: d 0, scales_h u16 2, scales_l 4..7, qs 8..135.) Run ib's weight j (< 16) is kvalues[low nibble of
// qs[16 ib + j]], weight 16 + j the high nibble's; the run's scale ls - 32 with ls = nibble ib of scales_l | two
// bits of scales_h << 4. Lane tig of a row's quad takes one qs word, bytes 4 tig .. 4 tig + 3 of the run: their
// low nibbles are weights 4 tig .. 4 tig + 3 (MMA K 4 tig ..), their high nibbles weights 16 + 4 tig .. (K 16 +
// 4 tig ..), so the activations go in their own order. A byte's two values come from one lookup in a table of the
// 256 bytes (kvalues[b & 15] | kvalues[b >> 4] << 8), 32 copies (word b * 32 + lane): no bank conflicts.
// The run sums (|128 hi + lo| < 2^27 each) are scaled in float32: their integer sum over a block could exceed
// 31 bits.
template <int NB>
struct M8IQ4XS {
    static constexpr int kKind = 23, kStageCols = 256 * NB, kStageBytes = 136 * NB, kRS = NB == 2 ? 304 : 176;
    static constexpr bool kLut = true, kTokens = false, kXsum = false, kHalves = false;
    __device__ static void fill(uint32_t* lut) {
        for (int i = threadIdx.x; i < 256 * 32 / 4; i += blockDim.x) {
            const int b = i / 8;  // (four words a store, 32 copies an entry)
            const uint32_t v = (static_cast<uint32_t>(static_cast<uint8_t>(__ldg(kKvalues + (b & 15))))) |
                               (static_cast<uint32_t>(static_cast<uint8_t>(__ldg(kKvalues + (b >> 4)))) << 8);
            reinterpret_cast<uint4*>(lut)[i] = make_uint4(v, v, v, v);
        }
    }
    __device__ static __forceinline__ void block(const uint8_t* r0, const uint8_t* r1, int tig, int gid,
                                                 const uint32_t* lut, const uint8_t* xh, const uint8_t* xl, float xs,
                                                 float (&total)[2]) {
        const uint32_t rb[2] = {smem_addr(r0), smem_addr(r1)};
        const uint32_t lutl = smem_addr(lut) + 4u * static_cast<uint32_t>(4 * gid + tig);
        float d[2], tot[2] = {0.f, 0.f};
        uint32_t sh[2], sl[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            d[j] = h2f(ld_s16<0>(rb[j]));
            sh[j] = ld_s16<2>(rb[j]);
            sl[j] = ld_s16<4>(rb[j]) | (ld_s16<6>(rb[j]) << 16);
        }
        const uint8_t* xsrc = gid == 0 ? xh : xl;
#pragma unroll
        for (int R = 0; R < 8; ++R) {
            uint32_t lo[2], hi[2];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const uint32_t w = ld_s32(rb[j] + 8 + 16 * R + 4 * tig);
                const uint32_t v0 = ld_s32(lutl + __byte_perm(w, 0u, 0x4440) * 128u);
                const uint32_t v1 = ld_s32(lutl + __byte_perm(w, 0u, 0x4441) * 128u);
                const uint32_t v2 = ld_s32(lutl + __byte_perm(w, 0u, 0x4442) * 128u);
                const uint32_t v3 = ld_s32(lutl + __byte_perm(w, 0u, 0x4443) * 128u);
                const uint32_t p01 = __byte_perm(v0, v1, 0x5140), p23 = __byte_perm(v2, v3, 0x5140);
                lo[j] = __byte_perm(p01, p23, 0x5410);
                hi[j] = __byte_perm(p01, p23, 0x7632);
            }
            uint32_t b0 = 0u, b1 = 0u;
            if (gid < 2) {
                b0 = *reinterpret_cast<const uint32_t*>(xsrc + 32 * R + 4 * tig);
                b1 = *reinterpret_cast<const uint32_t*>(xsrc + 32 * R + 16 + 4 * tig);
            }
            int acc[4];
            mma_s8(acc, lo[0], lo[1], hi[0], hi[1], b0, b1);
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int m = static_cast<int>(((sl[j] >> (4 * R)) & 15u) | (((sh[j] >> (2 * R)) & 3u) << 4)) - 32;
                tot[j] = fmaf(static_cast<float>(m), static_cast<float>(acc[2 * j] * 128 + acc[2 * j + 1]), tot[j]);
            }
        }
        const float k = xs * (1.0f / 128.0f);
        total[0] = fmaf(d[0] * k, tot[0], total[0]);
        total[1] = fmaf(d[1] * k, tot[1], total[1]);
    }
    __device__ static void stage(const uint8_t* r0, const uint8_t* r1, int tig, int gid, const uint32_t* lut,
                                 const uint8_t* xh, const uint8_t* xl, const float* xs, float (&total)[2]) {
        block(r0, r1, tig, gid, lut, xh, xl, xs[0], total);
        if constexpr (NB == 2) block(r0 + 136, r1 + 136, tig, gid, lut, xh + 256, xl + 256, xs[1], total);
    }
};

// ---------------------------------------------------------------- IQ3_XXS
// (98 bytes: d 0, qs 2..65 (a grid index a group of 4), 8 words at 66 + 4 ib: run ib's four 7-bit sign indices
// and its scale s in the top 4 bits.) As IQ3_S: lane tig takes groups 2 tig, 2 tig + 1 of run R (weights 8 tig ..
// 8 tig + 7), the grid word of each (16 copies of the 256-word grid, word i * 16 + lane % 16), its signs from
// ksigns[sign index tig] (the table's byte in 32 copies, word i * 32 + lane). The grid values are even, so a sign
// is applied as (g ^ m) + (m & 1) per byte (never a carry out of a byte). The run's scale (0.5 + s) / 2 is
// (2 s + 1) / 4, its float sum scaled once per block by d / 4. Fields are read by halves: the block is not 4-byte
// aligned in general.
template <int NB>
struct M8IQ3XXS {
    static constexpr int kKind = 18, kStageCols = 256 * NB, kStageBytes = 98 * NB, kRS = NB == 2 ? 208 : 112;
    static constexpr bool kLut = true, kTokens = false, kXsum = false, kHalves = false;
    __device__ static void fill(uint32_t* lut) {
        for (int i = threadIdx.x; i < 256 * 16 / 4; i += blockDim.x) {
            const uint32_t g = __ldg(kIq3xxsGrid + i / 4);
            reinterpret_cast<uint4*>(lut)[i] = make_uint4(g, g, g, g);
        }
        uint32_t* signs = lut + 4096;
        for (int i = threadIdx.x; i < 128 * 32 / 4; i += blockDim.x) {
            const uint32_t v = __ldg(kKsigns + i / 8);
            reinterpret_cast<uint4*>(signs)[i] = make_uint4(v, v, v, v);
        }
    }
    __device__ static __forceinline__ uint32_t signed_bytes(uint32_t g, uint32_t m) {
        return (g ^ m) + (m & 0x01010101u);
    }
    __device__ static __forceinline__ void block(const uint8_t* r0, const uint8_t* r1, int tig, int gid,
                                                 const uint32_t* lut, const uint8_t* xh, const uint8_t* xl, float xs,
                                                 float (&total)[2]) {
        const uint32_t rb[2] = {smem_addr(r0), smem_addr(r1)};
        const int lane = 4 * gid + tig;
        const uint32_t gridl = smem_addr(lut) + 4u * static_cast<uint32_t>(lane & 15);
        const uint32_t signl = smem_addr(lut + 4096) + 4u * static_cast<uint32_t>(lane);
        float d[2], tot[2] = {0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 2; ++j) d[j] = h2f(ld_s16<0>(rb[j]));
        const uint8_t* xsrc = gid == 0 ? xh : xl;
#pragma unroll
        for (int R = 0; R < 8; ++R) {
            uint32_t a[2][2];
            int ms[2];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const uint32_t q2 = lds_u16_at(rb[j] + 2 + 8 * R + 2 * tig);
                const uint32_t aux = lds_u16_at(rb[j] + 66 + 4 * R) | (lds_u16_at(rb[j] + 68 + 4 * R) << 16);
                const uint32_t ga = ld_s32(gridl + (q2 & 0xffu) * 64u);
                const uint32_t gb = ld_s32(gridl + (q2 >> 8) * 64u);
                const uint32_t sb = ld_s32(signl + ((aux >> (7 * tig)) & 127u) * 128u);
                const uint32_t ma = prmt_sr(sb * 0x80402010u, 0x89ABu);  // bits 0..3 (group 2 tig)
                const uint32_t mb = prmt_sr(sb * 0x08040201u, 0x89ABu);  // bits 4..7 (group 2 tig + 1)
                a[j][0] = signed_bytes(ga, ma);
                a[j][1] = signed_bytes(gb, mb);
                ms[j] = 2 * static_cast<int>(aux >> 28) + 1;
            }
            uint2 b = make_uint2(0u, 0u);
            if (gid < 2) b = *reinterpret_cast<const uint2*>(xsrc + 32 * R + 8 * tig);
            int acc[4];
            mma_s8(acc, a[0][0], a[1][0], a[0][1], a[1][1], b.x, b.y);
#pragma unroll
            for (int j = 0; j < 2; ++j)
                tot[j] = fmaf(static_cast<float>(ms[j]), static_cast<float>(acc[2 * j] * 128 + acc[2 * j + 1]), tot[j]);
        }
        const float k = xs * (1.0f / 512.0f);  // (d / 4) (xs / 128)
        total[0] = fmaf(d[0] * k, tot[0], total[0]);
        total[1] = fmaf(d[1] * k, tot[1], total[1]);
    }
    __device__ static void stage(const uint8_t* r0, const uint8_t* r1, int tig, int gid, const uint32_t* lut,
                                 const uint8_t* xh, const uint8_t* xl, const float* xs, float (&total)[2]) {
        block(r0, r1, tig, gid, lut, xh, xl, xs[0], total);
        if constexpr (NB == 2) block(r0 + 98, r1 + 98, tig, gid, lut, xh + 256, xl + 256, xs[1], total);
    }
};

// ---------------------------------------------------------------- Q8_0
// (34 bytes: d 0, qs 2..33.) A stage is NB runs (blocks); in run r lane tig takes codes 8 tig .. 8 tig + 7. Eight
// blocks a stage (256 columns: one activation scale block), so a warp's loop turns half as often as with four.
template <int NB>
struct M8Q8_0N {
    static constexpr int kKind = 8, kStageCols = 32 * NB, kStageBytes = 34 * NB, kRS = NB == 8 ? 304 : 176;
    static constexpr bool kLut = false, kTokens = true, kXsum = false, kHalves = false;
    __device__ static void fill(uint32_t*) {}
    __device__ static void stage(const uint8_t* r0, const uint8_t* r1, int tig, int gid, const uint32_t*,
                                 const uint8_t* xh, const uint8_t* xl, const float* xs, float (&total)[2]) {
        const uint32_t rb[2] = {smem_addr(r0), smem_addr(r1)};  // (32-bit shared addresses: plain LDS)
        const uint8_t* xsrc = gid == 0 ? xh : xl;
        const float k = xs[0] * (1.0f / 128.0f);  // (a stage lies within one 256-column scale block)
#pragma unroll
        for (int r = 0; r < NB; ++r) {
            uint32_t a[2][2];
            float d[2];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const uint32_t p = rb[j] + 34 * r + 2 + 8 * tig;
                const uint32_t wa = p & ~3u, sh = 8u * (p & 3u);
                const uint32_t w0 = ld_s32(wa), w1 = ld_s32(wa + 4), w2 = ld_s32(wa + 8);
                a[j][0] = __funnelshift_r(w0, w1, sh);
                a[j][1] = __funnelshift_r(w1, w2, sh);
                d[j] = h2f(lds_u16_at(rb[j] + 34 * r));
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
        const uint32_t rb[2] = {smem_addr(r0), smem_addr(r1)};
        const int t = gid >> 1;
        const uint8_t* xsrc = ((gid & 1) ? xl : xh) + int64_t(t) * xstride;
        const float k = tig < nt ? xs[tig * xsstride] * (1.0f / 128.0f) : 0.0f;
#pragma unroll
        for (int r = 0; r < NB; ++r) {
            uint32_t a[2][2];
            float d[2];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const uint32_t p = rb[j] + 34 * r + 2 + 8 * tig;
                const uint32_t wa = p & ~3u, sh = 8u * (p & 3u);
                const uint32_t w0 = ld_s32(wa), w1 = ld_s32(wa + 4), w2 = ld_s32(wa + 8);
                a[j][0] = __funnelshift_r(w0, w1, sh);
                a[j][1] = __funnelshift_r(w1, w2, sh);
                d[j] = h2f(lds_u16_at(rb[j] + 34 * r));
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
using M8Q8_0 = M8Q8_0N<8>;

// ---------------------------------------------------------------- Q2_0
// (18 bytes: d 0, codes 2..17; weight j of the block is d (q_j - 1) with q_j bits 2 (j % 4) .. + 1 of byte
// 2 + j / 4.) A stage is four blocks: 256 columns, one activation scale. In run h (32 weights) of a block, lane
// tig of a row's quad takes weights 8 tig .. 8 tig + 7 (two code bytes): K 4 tig .. 4 tig + 3 of the MMA are the
// first four, K 16 + 4 tig .. the last four, the activations in the same order (as Q8_0's runs). The codes enter
// the MMA as the exact int8 values q - 1 (-1 .. 2); a block's two runs add up in int32 before its d.
struct M8Q2_0 {
    static constexpr int kKind = 42, kStageCols = 256, kStageBytes = 72, kRS = 112;
    static constexpr bool kLut = false, kTokens = false, kXsum = false, kHalves = false;
    __device__ static void fill(uint32_t*) {}
    // a byte's four codes as four int8 values q - 1: each 2-bit field moved to the bottom of its own byte (the
    // copies at bit offsets 0, 6, 12 and 18 put field i at bit 8 i), then 1 taken from each byte without a
    // borrow between bytes (every byte is first raised by 0x80)
    __device__ static __forceinline__ uint32_t expand(uint32_t c) {
        const uint32_t t = c | (c << 12);
        const uint32_t x = (t | (t << 6)) & 0x03030303u;
        return ((x | 0x80808080u) - 0x01010101u) ^ 0x80808080u;
    }
    __device__ static void stage(const uint8_t* r0, const uint8_t* r1, int tig, int gid, const uint32_t*,
                                 const uint8_t* xh, const uint8_t* xl, const float* xs, float (&total)[2]) {
        const uint32_t rb[2] = {smem_addr(r0), smem_addr(r1)};  // (even addresses: 16-bit loads)
        const uint8_t* xsrc = gid == 0 ? xh : xl;
        const float k = xs[0] * (1.0f / 128.0f);
#pragma unroll
        for (int blk = 0; blk < 4; ++blk) {
            float d[2];
            int t[2] = {0, 0};
#pragma unroll
            for (int j = 0; j < 2; ++j) d[j] = h2f(lds_u16_at(rb[j] + 18 * blk));
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint32_t a[2][2];
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const uint32_t c = lds_u16_at(rb[j] + 18 * blk + 2 + 8 * h + 2 * tig);
                    a[j][0] = expand(c & 255u);
                    a[j][1] = expand(c >> 8);
                }
                uint2 b = make_uint2(0u, 0u);
                if (gid < 2) b = *reinterpret_cast<const uint2*>(xsrc + 64 * blk + 32 * h + 8 * tig);
                int acc[4];
                mma_s8(acc, a[0][0], a[1][0], a[0][1], a[1][1], b.x, b.y);
                // (lanes with tig > 0 hold columns 2..7: zeros)
                t[0] += acc[0] * 128 + acc[1];
                t[1] += acc[2] * 128 + acc[3];
            }
            total[0] = fmaf(d[0] * k, static_cast<float>(t[0]), total[0]);
            total[1] = fmaf(d[1] * k, static_cast<float>(t[1]), total[1]);
        }
    }
};

// Eight values a lane of one 256-column block (a warp) split into int8 hi and lo and the block's scale:
// v = s (hi + lo / 128), s = max|v| / 127. With sum16 set, sum16[c] receives the block's 16-column group c's
// sum of 128 hi + lo (exact in float32): its split values' sum in units of s / 128.
__device__ __forceinline__ void m8_split_values(const float (&v)[8], int8_t* hi, int8_t* lo, float* scale, int lane,
                                                float* sum16 = nullptr) {
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
    if (sum16) {
        int t = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int h = static_cast<int8_t>((hw[i >> 2] >> (8 * (i & 3))) & 255u);
            const int l = static_cast<int8_t>((lw[i >> 2] >> (8 * (i & 3))) & 255u);
            t += 128 * h + l;
        }
        t += __shfl_xor_sync(0xffffffffu, t, 1);
        if ((lane & 1) == 0) sum16[lane >> 1] = static_cast<float>(t);
    }
}

// One 256-column block of an activation row split into int8 hi and lo and its scale, by one warp (8 values a
// lane, from element `at`). With gate set, v = swiglu(gate, up) (the same function, so the same float16 bits,
// as the separate SwiGLU kernel).
__device__ __forceinline__ void m8_split(const __half* x, const __half* gate, const __half* up, int64_t at,
                                         int8_t* hi, int8_t* lo, float* scale, int lane, float* sum16 = nullptr) {
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
    m8_split_values(v, hi, lo, scale, lane, sum16);
}

// ---------------------------------------------------------------- the K-types
// Their codes enter the MMA as small unsigned integers (Q2_K 0..3, Q3_K q + 4 h in 0..7, Q4_K 0..15, Q5_K 0..31,
// Q6_K 0..63) and each sub-block's sum is scaled on its own: w = a q - b per sub-block (a = d scale, b = dmin
// min, or a times the code's offset: 4 for Q3_K, 32 for Q6_K), so sum w x = a sum q x - b sum x, with sum x from
// the split's 16-column sums (in the same units, s / 128, as the MMA's 128 hi + lo). Types with sub-blocks of 32
// (Q4_K, Q5_K) use B's columns 0 / 1 (hi / lo) and lane tig 0 holds a run's sums; types with sub-blocks of 16
// (Q2_K, Q3_K, Q6_K) put the run's first 16 activations in columns 0 / 1 and its last 16 in columns 2 / 3, so
// lane tig 0 holds the first sub-block's sums and lane tig 1 the second's (kHalves: the two lanes' totals are
// added at the end of a job). In both, a lane takes weights 4 tig .. 4 tig + 3 and 16 + 4 tig .. of each run
// (one block word each), the activations in their own order.

// a word of the staged block at a 4-byte (A4) or only 2-byte aligned address
template <bool A4>
__device__ __forceinline__ uint32_t ld_word(uint32_t a) {
    if constexpr (A4) return ld_s32(a);
    return lds_u16_at(a) | (lds_u16_at(a + 2) << 16);
}

// B of a whole-run MMA: columns 0 / 1 = the run's 32 activations (hi / lo)
__device__ __forceinline__ void m8_run_b(const uint8_t* xh, const uint8_t* xl, int R, int tig, int gid, uint32_t& b0,
                                         uint32_t& b1) {
    b0 = b1 = 0u;
    if (gid < 2) {
        const uint8_t* src = gid ? xl : xh;
        b0 = *reinterpret_cast<const uint32_t*>(src + 32 * R + 4 * tig);
        b1 = *reinterpret_cast<const uint32_t*>(src + 32 * R + 16 + 4 * tig);
    }
}
// B of a two-halves MMA: columns 0 / 1 = the run's first 16 activations (hi / lo), columns 2 / 3 its last 16
__device__ __forceinline__ void m8_halves_b(const uint8_t* xh, const uint8_t* xl, int R, int tig, int gid, uint32_t& b0,
                                            uint32_t& b1) {
    b0 = b1 = 0u;
    if (gid < 4) {
        const uint32_t v = *reinterpret_cast<const uint32_t*>(((gid & 1) ? xl : xh) + 32 * R + (gid < 2 ? 0 : 16) + 4 * tig);
        if (gid < 2) b0 = v;
        else b1 = v;
    }
}

// the 6-bit scale and min of sub-block j of a Q4_K / Q5_K block from its 12 scale bytes (three words)
__device__ __forceinline__ void k4_scale_min(int j, uint32_t s0, uint32_t s1, uint32_t s2, float& sc, float& mn) {
    auto byte = [&](int i) { return ((i < 4 ? s0 : i < 8 ? s1 : s2) >> (8 * (i & 3))) & 255u; };
    if (j < 4) {
        sc = static_cast<float>(byte(j) & 63u);
        mn = static_cast<float>(byte(j + 4) & 63u);
    } else {
        sc = static_cast<float>((byte(j + 4) & 15u) | ((byte(j - 4) >> 6) << 4));
        mn = static_cast<float>((byte(j + 4) >> 4) | ((byte(j) >> 6) << 4));
    }
}

// Q4_K (144 bytes: d 0, dmin 2, scales 4..15, qs 16..143) and Q5_K (176: d, dmin, scales, qh 16..47, qs 48..175):
// run r's code i: the nibble r % 2 of qs[32 (r / 2) + i], Q5_K with bit r of qh[i] as its fifth bit.
template <bool Q5>
struct M8Q45K {
    // one block a stage: the blocks are 16-byte multiples, so a stage starts 16-byte aligned
    static constexpr int kKind = Q5 ? 13 : 12, kBlock = Q5 ? 176 : 144, kQs = Q5 ? 48 : 16;
    static constexpr int kStageCols = 256, kStageBytes = kBlock, kRS = kBlock;
    static constexpr bool kLut = false, kTokens = false, kXsum = true, kHalves = false;
    __device__ static void fill(uint32_t*) {}
    __device__ static __forceinline__ void block(const uint8_t* r0, const uint8_t* r1, int tig, int gid,
                                                 const uint8_t* xh, const uint8_t* xl, float xs, const float* xsum,
                                                 float (&total)[2]) {
        const uint32_t rb[2] = {smem_addr(r0), smem_addr(r1)};
        float d[2], dmin[2], tot[2] = {0.f, 0.f};
        uint32_t s0[2], s1[2], s2[2], qh[2][2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            d[j] = h2f(ld_s16<0>(rb[j]));
            dmin[j] = h2f(ld_s16<2>(rb[j]));
            s0[j] = ld_s32(rb[j] + 4);
            s1[j] = ld_s32(rb[j] + 8);
            s2[j] = ld_s32(rb[j] + 12);
            if constexpr (Q5) {
                qh[j][0] = ld_s32(rb[j] + 16 + 4 * tig);
                qh[j][1] = ld_s32(rb[j] + 32 + 4 * tig);
            }
        }
#pragma unroll
        for (int R = 0; R < 8; ++R) {
            uint32_t a[2][2];
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint32_t q = (ld_s32(rb[j] + kQs + 32 * (R >> 1) + 16 * h + 4 * tig) >> (4 * (R & 1))) & 0x0F0F0F0Fu;
                    if constexpr (Q5) q |= ((qh[j][h] >> R) & 0x01010101u) << 4;
                    a[j][h] = q;
                }
            uint32_t b0, b1;
            m8_run_b(xh, xl, R, tig, gid, b0, b1);
            int acc[4];
            mma_s8(acc, a[0][0], a[1][0], a[0][1], a[1][1], b0, b1);
            const float sx = tig == 0 ? xsum[2 * R] + xsum[2 * R + 1] : 0.f;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                float sc, mn;
                k4_scale_min(R, s0[j], s1[j], s2[j], sc, mn);
                tot[j] = fmaf(d[j] * sc, static_cast<float>(acc[2 * j] * 128 + acc[2 * j + 1]), tot[j]);
                tot[j] = fmaf(-dmin[j] * mn, sx, tot[j]);
            }
        }
        const float k = xs * (1.0f / 128.0f);
        total[0] = fmaf(k, tot[0], total[0]);
        total[1] = fmaf(k, tot[1], total[1]);
    }
    __device__ static void stage(const uint8_t* r0, const uint8_t* r1, int tig, int gid, const uint8_t* xh,
                                 const uint8_t* xl, const float* xs, const float* xsum, float (&total)[2]) {
        block(r0, r1, tig, gid, xh, xl, xs[0], xsum, total);
    }
};

// Q2_K (84 bytes: scales 0..15 (scale | min << 4 per 16), qs 16..79, d 80, dmin 82): run r's code i is the two bits
// at 2 (r % 4) of qs[32 (r / 4) + i]; w = d (s & 15) q - dmin (s >> 4).
struct M8Q2K {
    static constexpr int kKind = 10, kStageCols = 512, kStageBytes = 168, kRS = 208;
    static constexpr bool kLut = false, kTokens = false, kXsum = true, kHalves = true;
    __device__ static void fill(uint32_t*) {}
    __device__ static __forceinline__ void block(const uint8_t* r0, const uint8_t* r1, int tig, int gid,
                                                 const uint8_t* xh, const uint8_t* xl, float xs, const float* xsum,
                                                 float (&total)[2]) {
        const uint32_t rb[2] = {smem_addr(r0), smem_addr(r1)};
        float d[2], dmin[2], tot[2] = {0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            d[j] = h2f(ld_s16<80>(rb[j]));
            dmin[j] = h2f(ld_s16<82>(rb[j]));
        }
        const int sub = tig & 1;  // (lanes tig 0 / 1: the run's first / second 16)
#pragma unroll
        for (int R = 0; R < 8; ++R) {
            uint32_t a[2][2];
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
                for (int h = 0; h < 2; ++h)
                    a[j][h] = (ld_s32(rb[j] + 16 + 32 * (R >> 2) + 16 * h + 4 * tig) >> (2 * (R & 3))) & 0x03030303u;
            uint32_t b0, b1;
            m8_halves_b(xh, xl, R, tig, gid, b0, b1);
            int acc[4];
            mma_s8(acc, a[0][0], a[1][0], a[0][1], a[1][1], b0, b1);
            const float sx = tig < 2 ? xsum[2 * R + sub] : 0.f;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const uint32_t sb = lds_u8_at(rb[j] + 2 * R + sub);
                tot[j] = fmaf(d[j] * static_cast<float>(sb & 15u), static_cast<float>(acc[2 * j] * 128 + acc[2 * j + 1]),
                              tot[j]);
                tot[j] = fmaf(-dmin[j] * static_cast<float>(sb >> 4), sx, tot[j]);
            }
        }
        const float k = xs * (1.0f / 128.0f);
        total[0] = fmaf(k, tot[0], total[0]);
        total[1] = fmaf(k, tot[1], total[1]);
    }
    __device__ static void stage(const uint8_t* r0, const uint8_t* r1, int tig, int gid, const uint8_t* xh,
                                 const uint8_t* xl, const float* xs, const float* xsum, float (&total)[2]) {
        block(r0, r1, tig, gid, xh, xl, xs[0], xsum, total);
        block(r0 + 84, r1 + 84, tig, gid, xh + 256, xl + 256, xs[1], xsum + 16, total);
    }
};

// Q3_K (110 bytes: hmask 0..31, qs 32..95, scales 96..107 (sixteen 6-bit, less 32), d 108): run r's code i is the two
// bits at 2 (r % 4) of qs[32 (r / 4) + i] plus 4 times bit r of hmask[i], less 4 (a clear high bit subtracts 4).
// The second block of a stage is only 2-byte aligned.
struct M8Q3K {
    static constexpr int kKind = 11, kStageCols = 512, kStageBytes = 220, kRS = 240;
    static constexpr bool kLut = false, kTokens = false, kXsum = true, kHalves = true;
    __device__ static void fill(uint32_t*) {}
    template <bool A4>
    __device__ static __forceinline__ void block(const uint8_t* r0, const uint8_t* r1, int tig, int gid,
                                                 const uint8_t* xh, const uint8_t* xl, float xs, const float* xsum,
                                                 float (&total)[2]) {
        const uint32_t rb[2] = {smem_addr(r0), smem_addr(r1)};
        float d[2], tot[2] = {0.f, 0.f};
        uint32_t hm[2][2], sw[2][3];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            d[j] = h2f(lds_u16_at(rb[j] + 108));
            hm[j][0] = ld_word<A4>(rb[j] + 4 * tig);
            hm[j][1] = ld_word<A4>(rb[j] + 16 + 4 * tig);
#pragma unroll
            for (int w = 0; w < 3; ++w) sw[j][w] = ld_word<A4>(rb[j] + 96 + 4 * w);
        }
        const int sub = tig & 1;
#pragma unroll
        for (int R = 0; R < 8; ++R) {
            uint32_t a[2][2];
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
                for (int h = 0; h < 2; ++h)
                    a[j][h] = ((ld_word<A4>(rb[j] + 32 + 32 * (R >> 2) + 16 * h + 4 * tig) >> (2 * (R & 3))) & 0x03030303u) |
                              (((hm[j][h] >> R) & 0x01010101u) << 2);
            uint32_t b0, b1;
            m8_halves_b(xh, xl, R, tig, gid, b0, b1);
            int acc[4];
            mma_s8(acc, a[0][0], a[1][0], a[0][1], a[1][1], b0, b1);
            const float sx = tig < 2 ? xsum[2 * R + sub] : 0.f;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                // scale k = 2 R + sub: its low four bits from byte k % 8 (the high nibble from the second eight),
                // two high bits from byte 8 + k % 4 at 2 (k / 4)
                const int kk = 2 * R + sub;
                auto byte = [&](int i) { return (sw[j][i >> 2] >> (8 * (i & 3))) & 255u; };
                const uint32_t low = kk < 8 ? (byte(kk & 7) & 15u) : (byte(kk & 7) >> 4);
                const uint32_t high = (byte(8 + (kk & 3)) >> (2 * (kk >> 2))) & 3u;
                const float dl = d[j] * static_cast<float>(static_cast<int>(low | (high << 4)) - 32);
                tot[j] = fmaf(dl, static_cast<float>(acc[2 * j] * 128 + acc[2 * j + 1]) - 4.0f * sx, tot[j]);
            }
        }
        const float k = xs * (1.0f / 128.0f);
        total[0] = fmaf(k, tot[0], total[0]);
        total[1] = fmaf(k, tot[1], total[1]);
    }
    __device__ static void stage(const uint8_t* r0, const uint8_t* r1, int tig, int gid, const uint8_t* xh,
                                 const uint8_t* xl, const float* xs, const float* xsum, float (&total)[2]) {
        block<true>(r0, r1, tig, gid, xh, xl, xs[0], xsum, total);
        block<false>(r0 + 110, r1 + 110, tig, gid, xh + 256, xl + 256, xs[1], xsum + 16, total);
    }
};

// Q6_K (210 bytes: ql 0..127, qh 128..191, scales 192..207 (int8 per 16), d 208): run r = 4 h + s, code i: the
// nibble s / 2 of ql[64 h + 32 (s % 2) + i] with the two bits at 2 s of qh[32 h + i] above it, less 32. One block a
// stage (two would not leave room for the ring), 2-byte aligned in general: words are read by halves.
struct M8Q6K {
    static constexpr int kKind = 14, kStageCols = 256, kStageBytes = 210, kRS = 240;
    static constexpr bool kLut = false, kTokens = false, kXsum = true, kHalves = true;
    __device__ static void fill(uint32_t*) {}
    template <bool A4>
    __device__ static __forceinline__ void block(const uint8_t* r0, const uint8_t* r1, int tig, int gid,
                                                 const uint8_t* xh, const uint8_t* xl, float xs, const float* xsum,
                                                 float (&total)[2]) {
        const uint32_t rb[2] = {smem_addr(r0), smem_addr(r1)};
        float d[2], tot[2] = {0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 2; ++j) d[j] = h2f(lds_u16_at(rb[j] + 208));
        const int sub = tig & 1;
#pragma unroll
        for (int R = 0; R < 8; ++R) {
            const int hh = R >> 2, ss = R & 3;
            uint32_t a[2][2];
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t ql = ld_word<A4>(rb[j] + 64 * hh + 32 * (ss & 1) + 16 * h + 4 * tig);
                    const uint32_t qh = ld_word<A4>(rb[j] + 128 + 32 * hh + 16 * h + 4 * tig);
                    a[j][h] = ((ql >> (4 * (ss >> 1))) & 0x0F0F0F0Fu) | (((qh >> (2 * ss)) & 0x03030303u) << 4);
                }
            uint32_t b0, b1;
            m8_halves_b(xh, xl, R, tig, gid, b0, b1);
            int acc[4];
            mma_s8(acc, a[0][0], a[1][0], a[0][1], a[1][1], b0, b1);
            const float sx = tig < 2 ? xsum[2 * R + sub] : 0.f;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const float dsc = d[j] * static_cast<float>(static_cast<int8_t>(lds_u8_at(rb[j] + 192 + 2 * R + sub)));
                tot[j] = fmaf(dsc, static_cast<float>(acc[2 * j] * 128 + acc[2 * j + 1]) - 32.0f * sx, tot[j]);
            }
        }
        const float k = xs * (1.0f / 128.0f);
        total[0] = fmaf(k, tot[0], total[0]);
        total[1] = fmaf(k, tot[1], total[1]);
    }
    __device__ static void stage(const uint8_t* r0, const uint8_t* r1, int tig, int gid, const uint8_t* xh,
                                 const uint8_t* xl, const float* xs, const float* xsum, float (&total)[2]) {
        block<false>(r0, r1, tig, gid, xh, xl, xs[0], xsum, total);
    }
};

}  // namespace smoe
