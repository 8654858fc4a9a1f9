// Decoders of the grouped GEMM's A operand: 128 weights of one row (a thread's half of a 256-column stage)
// to exact float16 pairs in TMEM.
//
// A stage's raw blocks are staged row by row (the 16-byte aligned cover of each row's bytes, rows an odd number
// of 16-byte chunks apart). A thread reads its row with 16-byte loads — 8 consecutive rows hit the 32 banks
// once — and aligns the words in registers to the row's byte offset, so every field of the block is then a
// register picked at compile time. Each decoder produces the float16 weights in column order and stores them
// with tcgen05.st 32x32b (16 registers = 32 weights at a time). Every weight is the float32 weight of gguf-py
// rounded to float16 once (the reference's tiles round to the activations' type, strata_mlx/blocks.py:610).
#pragma once

#include "blocks.cuh"
#include "tc05.cuh"

namespace smoe {

// Bytes [base, base + 4 NW) of a staged row (16-byte aligned) as NW words, for any byte offset `base`.
template <int NW>
__device__ __forceinline__ void row_words(const uint8_t* row, int base, uint32_t (&w)[NW]) {
    constexpr int NR = 4 * ((NW + 4 + 3) / 4);  // words read: enough for a shift of up to 3 words and a funnel
    uint32_t r[NR];
    const uint4* c = reinterpret_cast<const uint4*>(row + (base & ~15));
#pragma unroll
    for (int i = 0; i < NR / 4; ++i) {
        const uint4 v = c[i];
        r[4 * i] = v.x;
        r[4 * i + 1] = v.y;
        r[4 * i + 2] = v.z;
        r[4 * i + 3] = v.w;
    }
    const int k = (base >> 2) & 3;
    if (k & 2) {
#pragma unroll
        for (int i = 0; i + 2 < NR; ++i) r[i] = r[i + 2];
    }
    if (k & 1) {
#pragma unroll
        for (int i = 0; i + 1 < NR; ++i) r[i] = r[i + 1];
    }
    const int b = 8 * (base & 3);
    if (b) {
#pragma unroll
        for (int i = 0; i < NW; ++i) w[i] = __funnelshift_r(r[i], r[i + 1], b);
    } else {
#pragma unroll
        for (int i = 0; i < NW; ++i) w[i] = r[i];
    }
}

// The 4 bytes at byte P of the words w (P known at compile time).
template <int P, int NW>
__device__ __forceinline__ uint32_t bytes4(const uint32_t (&w)[NW]) {
    static_assert((P >> 2) < NW, "field outside the staged words");
    if constexpr ((P & 3) == 0) return w[P >> 2];
    else {
        static_assert((P >> 2) + 1 < NW, "field outside the staged words");
        return __funnelshift_r(w[P >> 2], w[(P >> 2) + 1], 8 * (P & 3));
    }
}
template <int P, int NW>
__device__ __forceinline__ uint32_t bytes2(const uint32_t (&w)[NW]) {
    if constexpr ((P & 3) == 3) return bytes4<P, NW>(w) & 0xffffu;
    else return (w[P >> 2] >> (8 * (P & 3))) & 0xffffu;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t s) { return __byte_perm(a, b, s); }
__device__ __forceinline__ uint32_t h2fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t h2mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;\n" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t h2sub(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;\n" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t dup_half(uint32_t lo16) { return (lo16 & 0xffffu) * 0x00010001u; }

constexpr int kGmLutRep = 16;  // copies of the IQ3_S codebook in shared memory (lane & 15 reads its own)

// Q2_K (84 bytes: scales 0..15, qs 16..79, d 80, dmin 82): half H of the block is qs bytes 16 + 32 H .. + 31 at
// four shifts; sub-block 8 H + 2 s + (byte >= 16) scales 16 weights. Per sub-block the four possible weights
// (code 0..3) are worked out once in float32, rounded to float16, and every weight is then a byte-permute
// lookup of its code.
struct GdQ2K {
    static constexpr int kKind = 10;
    static constexpr bool kLut = false;
    template <int H>
    __device__ static void decode(const uint8_t* row, int off, uint32_t tbase, const uint32_t*, const uint32_t*) {
        uint32_t w[21];
        row_words(row, off, w);
        const uint32_t dd = w[20];
        const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(dd & 0xffffu)));
        const float dmin = __half2float(__ushort_as_half(static_cast<unsigned short>(dd >> 16)));
        const uint32_t sc0 = w[2 * H], sc1 = w[2 * H + 1];
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            uint32_t v[16];
#pragma unroll
            for (int half16 = 0; half16 < 2; ++half16) {
                const int sub = 2 * s + half16;
                const uint32_t sb = ((sub < 4 ? sc0 : sc1) >> (8 * (sub & 3))) & 255u;
                const float dl = __fmul_rn(d, float(sb & 15u)), ml = __fmul_rn(dmin, float(sb >> 4));
                const uint32_t t01 = tc::pack_half2(fmaf(dl, 0.f, -ml), fmaf(dl, 1.f, -ml));
                const uint32_t t23 = tc::pack_half2(fmaf(dl, 2.f, -ml), fmaf(dl, 3.f, -ml));
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint32_t c = (w[4 + 8 * H + 4 * half16 + kk] >> (2 * s)) & 0x03030303u;  // four codes
                    const uint32_t sel = c * 34u + 0x10101010u;  // nibbles 2q, 2q+1
                    v[2 * (4 * half16 + kk)] = prmt(t01, t23, sel);
                    v[2 * (4 * half16 + kk) + 1] = prmt(t01, t23, sel >> 16);
                }
            }
            tc::tmem_st16(tbase + 16u * s, v);
        }
    }
};

// IQ3_S (110 bytes: d 0, qs 2..65, qh 66..73, signs 74..105, scales 106..109): runs 4 H .. 4 H + 3; a group of
// four weights is a codebook word (lane-replicated table), expanded to the exact float16 integers
// grid * (1 + 2 sub-scale) with the signs, then one rounding d * that.
struct GdIQ3S {
    static constexpr int kKind = 21;
    static constexpr bool kLut = true;
    template <int IB, int NW>
    __device__ static void run(const uint32_t (&w)[NW], uint32_t d2, uint32_t qh, uint32_t sc, uint32_t tbase,
                               const uint32_t* lut, const uint32_t* mc) {
        const uint32_t q0 = bytes4<2 + 8 * IB>(w), q1 = bytes4<6 + 8 * IB>(w);
        const uint32_t sg = bytes4<74 + 4 * IB>(w);
        const uint2 mcv = reinterpret_cast<const uint2*>(mc)[sc & 15u];
        uint32_t v[16];
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            const uint32_t qsb = ((l < 4 ? q0 : q1) >> (8 * (l & 3))) & 255u;
            const uint32_t idx = qsb | (((qh >> l) & 1u) << 8);
            const uint32_t g = lut[idx * kGmLutRep];
            const uint32_t t = (sg >> (4 * l)) & 15u;
            const uint32_t lo = h2fma(prmt(g, 0x6464u, 0x4140), mcv.x, mcv.y) ^ ((t * 0x40008000u) & 0x80008000u);
            const uint32_t hi = h2fma(prmt(g, 0x6464u, 0x4342), mcv.x, mcv.y) ^ ((t * 0x10002000u) & 0x80008000u);
            v[2 * l] = h2mul(lo, d2);
            v[2 * l + 1] = h2mul(hi, d2);
        }
        tc::tmem_st16(tbase + 16u * (IB & 3), v);
    }
    template <int H>
    __device__ static void decode(const uint8_t* row, int off, uint32_t tbase, const uint32_t* lut, const uint32_t* mc) {
        uint32_t w[28];
        row_words(row, off, w);
        const uint32_t d2 = dup_half(w[0]);
        const uint32_t qh4 = bytes4<66 + 4 * H>(w);             // qh bytes of runs 4H .. 4H + 3
        const uint32_t sc2 = bytes2<106 + 2 * H>(w);            // sub-scale nibbles of runs 4H .. 4H + 3
        run<4 * H + 0>(w, d2, qh4 & 255u, sc2, tbase, lut, mc);
        run<4 * H + 1>(w, d2, (qh4 >> 8) & 255u, sc2 >> 4, tbase, lut, mc);
        run<4 * H + 2>(w, d2, (qh4 >> 16) & 255u, sc2 >> 8, tbase, lut, mc);
        run<4 * H + 3>(w, d2, qh4 >> 24, sc2 >> 12, tbase, lut, mc);
    }
};

// Q8_0 (34 bytes: d 0, qs 2..33): blocks 4 H .. 4 H + 3 of the stage's eight; a weight is d * q rounded once
// to float16.
struct GdQ8_0 {
    static constexpr int kKind = 8;
    static constexpr bool kLut = false;
    template <int BB, int NW>
    __device__ static void block(const uint32_t (&w)[NW], uint32_t tbase) {
        const uint32_t d2 = dup_half(bytes2<34 * BB>(w));
        uint32_t v[16];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            uint32_t q;
            switch (k) {  // the compile-time byte position of word k of block BB
                case 0: q = bytes4<34 * BB + 2>(w); break;
                case 1: q = bytes4<34 * BB + 6>(w); break;
                case 2: q = bytes4<34 * BB + 10>(w); break;
                case 3: q = bytes4<34 * BB + 14>(w); break;
                case 4: q = bytes4<34 * BB + 18>(w); break;
                case 5: q = bytes4<34 * BB + 22>(w); break;
                case 6: q = bytes4<34 * BB + 26>(w); break;
                default: q = bytes4<34 * BB + 30>(w); break;
            }
            q ^= 0x80808080u;  // int8 -> code + 128
            v[2 * k] = h2mul(h2sub(prmt(q, 0x6464u, 0x4140), 0x64806480u), d2);
            v[2 * k + 1] = h2mul(h2sub(prmt(q, 0x6464u, 0x4342), 0x64806480u), d2);
        }
        tc::tmem_st16(tbase + 16u * BB, v);
    }
    template <int H>
    __device__ static void decode(const uint8_t* row, int off, uint32_t tbase, const uint32_t*, const uint32_t*) {
        uint32_t w[34];
        row_words(row, off + 136 * H, w);
        block<0>(w, tbase);
        block<1>(w, tbase);
        block<2>(w, tbase);
        block<3>(w, tbase);
    }
};

}  // namespace smoe
