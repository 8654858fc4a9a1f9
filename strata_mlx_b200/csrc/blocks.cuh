// Decoders of GGUF quant blocks, one struct per type.
//
// `run(row, n, w)` writes the n-th run of 32 weights of a row (float32, exact products, in gguf-py's
// operation order where a rounding happens) into w. Field positions restate the reference's `_UNPACK`
// bodies (strata_mlx/blocks.py:57-194) and gguf-py 0.19.0's dequantize_blocks (gguf/quants.py) for the
// K-types the reference decodes on the CPU only (strata_mlx/gguf.py:182-276). Weight j of a 256-block
// sits in run j / 32; the comment on each type gives its byte/bit layout.
#pragma once

#include "_tables.cuh"
#include "common.cuh"

namespace smoe {

// Rounding-exact helpers: no contraction across a rounding point that gguf-py (numpy) has.
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }

// Q8_0: [d f16][32 x int8]; w = d * q (gguf-py quants.py:378, reference gguf.py:203-206)
struct Q8_0 {
    static constexpr int kKind = 8, kPer = 32, kBytes = 34;
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + n * kBytes;
        const float d = half_at(b);
#pragma unroll
        for (int j = 0; j < 32; ++j) w[j] = mul_rn(d, float(int8_t(b[2 + j])));
    }
};

// Q2_K: [scales 16][qs 64][d f16 @80][dmin f16 @82]; weight j: q = (qs[32(j/128) + j%32] >> 2((j%128)/32)) & 3,
// sub-block j/16 with scale byte s: w = (d*(s&15))*q - dmin*(s>>4) (gguf-py quants.py:404-428)
struct Q2_K {
    static constexpr int kKind = 10, kPer = 256, kBytes = 84;
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + (n >> 3) * kBytes;
        const int r = n & 7;
        const uint8_t* q = b + 16 + 32 * (r >> 2);
        const int shift = 2 * (r & 3);
        const float d = half_at(b + 80), dmin = half_at(b + 82);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t s = b[2 * r + h];
            const float dl = mul_rn(d, float(s & 15)), ml = mul_rn(dmin, float(s >> 4));
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float v = float((q[16 * h + i] >> shift) & 3);
                w[16 * h + i] = sub_rn(mul_rn(dl, v), ml);
            }
        }
    }
};

// Q3_K: [hmask 32][qs 64 @32][scales 12 @96][d f16 @108]; run r: two bits from qs[32(r/4) + i] >> 2(r%4),
// less 4 where bit r of hmask[i] is clear; 6-bit scales less 32 per 16 (reference blocks.py:45-50,164-175)
struct Q3_K {
    static constexpr int kKind = 11, kPer = 256, kBytes = 110;
    __device__ static float scale(const uint8_t* s, int k) {
        const int p = k & 3, word = k >> 2;
        const uint32_t low = word < 2 ? (s[4 * word + p] & 15u) : (uint32_t(s[4 * (word - 2) + p]) >> 4);
        return float(int(low | (((uint32_t(s[8 + p]) >> (2 * word)) & 3u) << 4)) - 32);
    }
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + (n >> 3) * kBytes;
        const int r = n & 7;
        const uint8_t* q = b + 32 + 32 * (r >> 2);
        const int shift = 2 * (r & 3);
        const float d = half_at(b + 108);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float dl = mul_rn(d, scale(b + 96, 2 * r + h));
#pragma unroll
            for (int i = 16 * h; i < 16 * h + 16; ++i) {
                const int v = int((q[i] >> shift) & 3u) - (((b[i] >> r) & 1u) ? 0 : 4);
                w[i] = mul_rn(dl, float(v));
            }
        }
    }
};

// The eight 6-bit (scale, min) pairs of a Q4_K / Q5_K block from its 12 bytes (reference gguf.py:174-179)
__device__ __forceinline__ void k4_scale_min(const uint8_t* s, int t, float& sc, float& mn) {
    if (t < 4) {
        sc = float(s[t] & 63);
        mn = float(s[t + 4] & 63);
    } else {
        sc = float((s[t + 4] & 15) | ((s[t - 4] >> 6) << 4));
        mn = float((s[t + 4] >> 4) | ((s[t] >> 6) << 4));
    }
}

// Q4_K: [d][dmin][scales 12 @4][qs 128 @16]; sub-block t = run: q = (qs[32(t/2) + i] >> 4(t%2)) & 15,
// w = (d*sc)*q - dmin*mn (gguf-py quants.py:475, reference gguf.py:207-216)
struct Q4_K {
    static constexpr int kKind = 12, kPer = 256, kBytes = 144;
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + (n >> 3) * kBytes;
        const int t = n & 7;
        float sc, mn;
        k4_scale_min(b + 4, t, sc, mn);
        const float dl = mul_rn(half_at(b), sc), ml = mul_rn(half_at(b + 2), mn);
        const uint8_t* q = b + 16 + 32 * (t >> 1);
        const int shift = 4 * (t & 1);
#pragma unroll
        for (int i = 0; i < 32; ++i) w[i] = sub_rn(mul_rn(dl, float((q[i] >> shift) & 15)), ml);
    }
};

// Q5_K: [d][dmin][scales 12 @4][qh 32 @16][qs 128 @48]; as Q4_K with a fifth bit, bit t of qh[i]
struct Q5_K {
    static constexpr int kKind = 13, kPer = 256, kBytes = 176;
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + (n >> 3) * kBytes;
        const int t = n & 7;
        float sc, mn;
        k4_scale_min(b + 4, t, sc, mn);
        const float dl = mul_rn(half_at(b), sc), ml = mul_rn(half_at(b + 2), mn);
        const uint8_t* q = b + 48 + 32 * (t >> 1);
        const int shift = 4 * (t & 1);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const uint32_t v = ((q[i] >> shift) & 15u) | (((b[16 + i] >> t) & 1u) << 4);
            w[i] = sub_rn(mul_rn(dl, float(v)), ml);
        }
    }
};

// Q6_K: [ql 128][qh 64 @128][scales int8 16 @192][d f16 @208]; weight j = 128h + 32s + i (run r = 4h + s):
// low nibble of ql[64h + 32(s%2) + i] >> 4(s/2), two high bits qh[32h + i] >> 2s; q - 32;
// w = (d*scale)*q in that order, the product can need 25 bits (gguf-py quants.py:552, gguf.py:135-165)
struct Q6_K {
    static constexpr int kKind = 14, kPer = 256, kBytes = 210;
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + (n >> 3) * kBytes;
        const int r = n & 7, h = r >> 2, s = r & 3;
        const uint8_t* ql = b + 64 * h + 32 * (s & 1);
        const uint8_t* qh = b + 128 + 32 * h;
        const int lshift = 4 * (s >> 1), hshift = 2 * s;
        const float d = half_at(b + 208);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const float dsc = mul_rn(d, float(int8_t(b[192 + 2 * r + half])));
#pragma unroll
            for (int i = 16 * half; i < 16 * half + 16; ++i) {
                const int q = int(((ql[i] >> lshift) & 15u) | (((qh[i] >> hshift) & 3u) << 4)) - 32;
                w[i] = mul_rn(dsc, float(q));
            }
        }
    }
};

// IQ3_XXS: [d][qs 64 @2][8 x u32 @66]; run ib: aux = word ib, db = d*(0.5 + aux>>28)*0.5; group l of 4
// weights: iq3xxs_grid[qs[8ib + l]]; sign bits ksigns[(aux >> 7(l/2)) & 127] >> 4(l%2) (blocks.py:103-116)
struct IQ3_XXS {
    static constexpr int kKind = 18, kPer = 256, kBytes = 98;
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + (n >> 3) * kBytes;
        const int ib = n & 7;
        const uint32_t aux = u32le(b + 66 + 4 * ib);
        const float db = mul_rn(mul_rn(half_at(b), 0.5f + float(aux >> 28)), 0.5f);
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            const uint32_t g = __ldg(&kIq3xxsGrid[b[2 + 8 * ib + l]]);
            const uint32_t sign = uint32_t(__ldg(&kKsigns[(aux >> (7 * (l >> 1))) & 127])) >> (4 * (l & 1));
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float v = mul_rn(db, float((g >> (8 * j)) & 255));
                w[4 * l + j] = ((sign >> j) & 1) ? -v : v;
            }
        }
    }
};

// IQ3_S: [d][qs 64 @2][qh 8 @66][signs 32 @74][scales 4 @106]; run ib: db = d*(1 + 2*nibble ib of scales);
// group l: iq3s_grid[qs[8ib + l] | bit l of qh[ib] << 8]; sign bits signs[4ib + l/2] >> 4(l%2)
// (reference blocks.py:89-102)
struct IQ3_S {
    static constexpr int kKind = 21, kPer = 256, kBytes = 110;
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + (n >> 3) * kBytes;
        const int ib = n & 7;
        const float db = mul_rn(half_at(b), float(1 + 2 * ((b[106 + (ib >> 1)] >> (4 * (ib & 1))) & 15)));
        const uint32_t high = b[66 + ib];
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            const uint32_t g = __ldg(&kIq3sGrid[b[2 + 8 * ib + l] | (((high >> l) & 1u) << 8)]);
            const uint32_t sign = uint32_t(b[74 + 4 * ib + (l >> 1)]) >> (4 * (l & 1));
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float v = mul_rn(db, float((g >> (8 * j)) & 255));
                w[4 * l + j] = ((sign >> j) & 1) ? -v : v;
            }
        }
    }
};

// IQ4_XS: [d][scales_h u16 @2][scales_l 4 @4][qs 128 @8]; run ib: ls = nibble ib of scales_l | two bits
// 2ib of scales_h << 4; dl = d*(ls - 32); 16 bytes qs[16ib..]: low nibbles then high (blocks.py:78-88)
struct IQ4_XS {
    static constexpr int kKind = 23, kPer = 256, kBytes = 136;
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + (n >> 3) * kBytes;
        const int ib = n & 7;
        const uint32_t ls = ((b[4 + (ib >> 1)] >> (4 * (ib & 1))) & 15u) | (((u16le(b + 2) >> (2 * ib)) & 3u) << 4);
        const float dl = mul_rn(half_at(b), float(int(ls) - 32));
        const uint8_t* q = b + 8 + 16 * ib;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            w[i] = mul_rn(dl, float(__ldg(&kKvalues[q[i] & 15])));
            w[16 + i] = mul_rn(dl, float(__ldg(&kKvalues[q[i] >> 4])));
        }
    }
};

// IQ4_NL: [d][qs 16]; w[i] = d*kvalues[qs[i] & 15], w[16+i] = d*kvalues[qs[i] >> 4] (blocks.py:69-77)
struct IQ4_NL {
    static constexpr int kKind = 20, kPer = 32, kBytes = 18;
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + n * kBytes;
        const float d = half_at(b);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            w[i] = mul_rn(d, float(__ldg(&kKvalues[b[2 + i] & 15])));
            w[16 + i] = mul_rn(d, float(__ldg(&kKvalues[b[2 + i] >> 4])));
        }
    }
};

// Q2_0: [d][16 bytes of 2-bit codes], 64 weights: w[4i + j] = d*(((q[i] >> 2j) & 3) - 1) (blocks.py:58-68)
struct Q2_0 {
    static constexpr int kKind = 42, kPer = 64, kBytes = 18;
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + (n >> 1) * kBytes;
        const uint8_t* q = b + 2 + 8 * (n & 1);
        const float d = half_at(b);
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) w[4 * i + j] = mul_rn(d, float(int((q[i] >> (2 * j)) & 3u) - 1));
    }
};

// IQ2_XXS: [d][8 x (4 grid bytes, u32 aux)] per run ib at 2 + 8ib; db = d*(0.5 + aux>>28)*0.25;
// group l of 8: iq2xxs_grid[q[l]], sign ksigns[(aux >> 7l) & 127] (blocks.py:148-161)
struct IQ2_XXS {
    static constexpr int kKind = 16, kPer = 256, kBytes = 66;
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + (n >> 3) * kBytes;
        const uint8_t* q = b + 2 + 8 * (n & 7);
        const uint32_t aux = u32le(q + 4);
        const float db = mul_rn(mul_rn(half_at(b), 0.5f + float(aux >> 28)), 0.25f);
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint64_t g = __ldg(&kIq2xxsGrid[q[l]]);
            const uint32_t sign = __ldg(&kKsigns[(aux >> (7 * l)) & 127]);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float v = mul_rn(db, float(uint32_t(g >> (8 * j)) & 255));
                w[8 * l + j] = ((sign >> j) & 1) ? -v : v;
            }
        }
    }
};

// IQ2_XS: [d][32 x u16 @2][scales 8 @66]; group l of run ib: q = u16 4ib + l: grid q & 511, ksigns[q >> 9];
// dl = d*0.25*(0.5 + nibble l/2 of scales[ib]) (blocks.py:133-147)
struct IQ2_XS {
    static constexpr int kKind = 17, kPer = 256, kBytes = 74;
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + (n >> 3) * kBytes;
        const int ib = n & 7;
        const float d = mul_rn(half_at(b), 0.25f);
        const uint32_t scales = b[66 + ib];
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t q = u16le(b + 2 + 2 * (4 * ib + l));
            const uint64_t g = __ldg(&kIq2xsGrid[q & 511]);
            const uint32_t sign = __ldg(&kKsigns[q >> 9]);
            const float dl = mul_rn(d, 0.5f + float(l < 2 ? (scales & 15) : (scales >> 4)));
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float v = mul_rn(dl, float(uint32_t(g >> (8 * j)) & 255));
                w[8 * l + j] = ((sign >> j) & 1) ? -v : v;
            }
        }
    }
};

// IQ2_S: [d][qs 32 @2][signs 32 @34][qh 8 @66][scales 8 @74]; group l of run ib:
// iq2s_grid[qs[4ib + l] | two bits 2l of qh[ib] << 8], signs[4ib + l] (blocks.py:117-132)
struct IQ2_S {
    static constexpr int kKind = 22, kPer = 256, kBytes = 82;
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + (n >> 3) * kBytes;
        const int ib = n & 7;
        const float d = mul_rn(half_at(b), 0.25f);
        const uint32_t high = b[66 + ib], scales = b[74 + ib];
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint64_t g = __ldg(&kIq2sGrid[b[2 + 4 * ib + l] | (((high >> (2 * l)) & 3u) << 8)]);
            const uint32_t sign = b[34 + 4 * ib + l];
            const float dl = mul_rn(d, 0.5f + float(l < 2 ? (scales & 15) : (scales >> 4)));
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float v = mul_rn(dl, float(uint32_t(g >> (8 * j)) & 255));
                w[8 * l + j] = ((sign >> j) & 1) ? -v : v;
            }
        }
    }
};

// IQ1_M: [qs 32][qh 16 @32][scales 4 x u16 @48, the block's f16 scale in their top nibbles]; group l of
// run ib: grid iq1_grid[qs[4ib + l] | (h & 7) << 8] (held as 0,1,2), h = nibble l%2 of qh[2ib + l/2];
// dl = d*(2*s + 1) with 3-bit s; w = dl*(g - 1 -/+ 0.125) (blocks.py:177-193)
struct IQ1_M {
    static constexpr int kKind = 29, kPer = 256, kBytes = 56;
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + (n >> 3) * kBytes;
        const int ib = n & 7;
        const uint32_t packed = (u16le(b + 48) >> 12) | ((u16le(b + 50) >> 8) & 0x00f0u) |
                                ((u16le(b + 52) >> 4) & 0x0f00u) | (u16le(b + 54) & 0xf000u);
        const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(packed)));
        const uint32_t scales = u16le(b + 48 + 2 * (ib >> 1)) >> (6 * (ib & 1));
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t high = (uint32_t(b[32 + 2 * ib + (l >> 1)]) >> (4 * (l & 1))) & 15u;
            const uint64_t g = __ldg(&kIq1Grid[b[4 * ib + l] | ((high & 7u) << 8)]);
            const float dl = mul_rn(d, float(2 * ((scales >> (3 * (l >> 1))) & 7u) + 1));
            const float delta = (high & 8u) ? -1.125f : -0.875f;
#pragma unroll
            for (int j = 0; j < 8; ++j) w[8 * l + j] = mul_rn(dl, __fadd_rn(float(uint32_t(g >> (8 * j)) & 255), delta));
        }
    }
};

// ---- Staged forms: `Staged<B>::run` writes the same floats as `B::run` (the same operations in the same order)
// for a row held in shared memory with at least 4 bytes after its end that may be read (the matvec's row slots).
// It reads the row four bytes at a time (two aligned words and a funnel shift, whatever the row's alignment)
// and turns small integers into floats without a conversion instruction: a byte v placed in the mantissa of
// 2^23 is the float 2^23 + v, and subtracting 2^23 + c gives v - c exactly (|v - c| < 2^23).

__device__ __forceinline__ uint32_t word_at(const uint8_t* p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
    return __funnelshift_r(w[0], w[1], static_cast<uint32_t>(a & 3u) * 8u);
}
// byte j of w, less c, as a float (base = 2^23 + c)
template <int J>
__device__ __forceinline__ float byte_less(uint32_t w, float base) {
    return __fsub_rn(__int_as_float(static_cast<int>(__byte_perm(w, 0x4B000000u, 0x7540u + J))), base);
}
constexpr float kF0 = 8388608.0f;  // 2^23

template <class B>
struct Staged {
    __device__ static void run(const uint8_t* row, int n, float* w) { B::run(row, n, w); }
};

template <>
struct Staged<Q8_0> {
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + n * Q8_0::kBytes;
        const float d = half_at(b);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t u = word_at(b + 2 + 4 * i) ^ 0x80808080u;  // int8 q as q + 128
            w[4 * i + 0] = mul_rn(d, byte_less<0>(u, kF0 + 128.0f));
            w[4 * i + 1] = mul_rn(d, byte_less<1>(u, kF0 + 128.0f));
            w[4 * i + 2] = mul_rn(d, byte_less<2>(u, kF0 + 128.0f));
            w[4 * i + 3] = mul_rn(d, byte_less<3>(u, kF0 + 128.0f));
        }
    }
};

template <>
struct Staged<Q2_K> {
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + (n >> 3) * Q2_K::kBytes;
        const int r = n & 7;
        const uint8_t* q = b + 16 + 32 * (r >> 2);
        const int shift = 2 * (r & 3);
        const float d = half_at(b + 80), dmin = half_at(b + 82);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t s = b[2 * r + h];
            const float dl = mul_rn(d, float(s & 15)), ml = mul_rn(dmin, float(s >> 4));
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t v = (word_at(q + 16 * h + 4 * i) >> shift) & 0x03030303u;
                w[16 * h + 4 * i + 0] = sub_rn(mul_rn(dl, byte_less<0>(v, kF0)), ml);
                w[16 * h + 4 * i + 1] = sub_rn(mul_rn(dl, byte_less<1>(v, kF0)), ml);
                w[16 * h + 4 * i + 2] = sub_rn(mul_rn(dl, byte_less<2>(v, kF0)), ml);
                w[16 * h + 4 * i + 3] = sub_rn(mul_rn(dl, byte_less<3>(v, kF0)), ml);
            }
        }
    }
};

template <>
struct Staged<Q3_K> {
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + (n >> 3) * Q3_K::kBytes;
        const int r = n & 7;
        const uint8_t* q = b + 32 + 32 * (r >> 2);
        const int shift = 2 * (r & 3);
        const float d = half_at(b + 108);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float dl = mul_rn(d, Q3_K::scale(b + 96, 2 * r + h));
#pragma unroll
            for (int i = 16 * h; i < 16 * h + 16; i += 4) {
                // q + 4 where bit r of hmask is set, q where it is clear; less 4
                const uint32_t v = ((word_at(q + i) >> shift) & 0x03030303u) |
                                   (((word_at(b + i) >> r) & 0x01010101u) << 2);
                w[i + 0] = mul_rn(dl, byte_less<0>(v, kF0 + 4.0f));
                w[i + 1] = mul_rn(dl, byte_less<1>(v, kF0 + 4.0f));
                w[i + 2] = mul_rn(dl, byte_less<2>(v, kF0 + 4.0f));
                w[i + 3] = mul_rn(dl, byte_less<3>(v, kF0 + 4.0f));
            }
        }
    }
};

template <>
struct Staged<Q4_K> {
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + (n >> 3) * Q4_K::kBytes;
        const int t = n & 7;
        float sc, mn;
        k4_scale_min(b + 4, t, sc, mn);
        const float dl = mul_rn(half_at(b), sc), ml = mul_rn(half_at(b + 2), mn);
        const uint8_t* q = b + 16 + 32 * (t >> 1);
        const int shift = 4 * (t & 1);
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
            const uint32_t v = (word_at(q + i) >> shift) & 0x0F0F0F0Fu;
            w[i + 0] = sub_rn(mul_rn(dl, byte_less<0>(v, kF0)), ml);
            w[i + 1] = sub_rn(mul_rn(dl, byte_less<1>(v, kF0)), ml);
            w[i + 2] = sub_rn(mul_rn(dl, byte_less<2>(v, kF0)), ml);
            w[i + 3] = sub_rn(mul_rn(dl, byte_less<3>(v, kF0)), ml);
        }
    }
};

template <>
struct Staged<Q5_K> {
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + (n >> 3) * Q5_K::kBytes;
        const int t = n & 7;
        float sc, mn;
        k4_scale_min(b + 4, t, sc, mn);
        const float dl = mul_rn(half_at(b), sc), ml = mul_rn(half_at(b + 2), mn);
        const uint8_t* q = b + 48 + 32 * (t >> 1);
        const int shift = 4 * (t & 1);
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
            const uint32_t v = ((word_at(q + i) >> shift) & 0x0F0F0F0Fu) | (((word_at(b + 16 + i) >> t) & 0x01010101u) << 4);
            w[i + 0] = sub_rn(mul_rn(dl, byte_less<0>(v, kF0)), ml);
            w[i + 1] = sub_rn(mul_rn(dl, byte_less<1>(v, kF0)), ml);
            w[i + 2] = sub_rn(mul_rn(dl, byte_less<2>(v, kF0)), ml);
            w[i + 3] = sub_rn(mul_rn(dl, byte_less<3>(v, kF0)), ml);
        }
    }
};

template <>
struct Staged<Q6_K> {
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + (n >> 3) * Q6_K::kBytes;
        const int r = n & 7, h = r >> 2, s = r & 3;
        const uint8_t* ql = b + 64 * h + 32 * (s & 1);
        const uint8_t* qh = b + 128 + 32 * h;
        const int lshift = 4 * (s >> 1), hshift = 2 * s;
        const float d = half_at(b + 208);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const float dsc = mul_rn(d, float(int8_t(b[192 + 2 * r + half])));
#pragma unroll
            for (int i = 16 * half; i < 16 * half + 16; i += 4) {
                const uint32_t v = ((word_at(ql + i) >> lshift) & 0x0F0F0F0Fu) |
                                   (((word_at(qh + i) >> hshift) & 0x03030303u) << 4);  // q + 32
                w[i + 0] = mul_rn(dsc, byte_less<0>(v, kF0 + 32.0f));
                w[i + 1] = mul_rn(dsc, byte_less<1>(v, kF0 + 32.0f));
                w[i + 2] = mul_rn(dsc, byte_less<2>(v, kF0 + 32.0f));
                w[i + 3] = mul_rn(dsc, byte_less<3>(v, kF0 + 32.0f));
            }
        }
    }
};

// four grid bytes times db, each negated where its sign bit is set
__device__ __forceinline__ void grid4(uint32_t g, float db, uint32_t sign, float* w) {
    const float v0 = mul_rn(db, byte_less<0>(g, kF0)), v1 = mul_rn(db, byte_less<1>(g, kF0));
    const float v2 = mul_rn(db, byte_less<2>(g, kF0)), v3 = mul_rn(db, byte_less<3>(g, kF0));
    w[0] = (sign & 1u) ? -v0 : v0;
    w[1] = (sign & 2u) ? -v1 : v1;
    w[2] = (sign & 4u) ? -v2 : v2;
    w[3] = (sign & 8u) ? -v3 : v3;
}

template <>
struct Staged<IQ3_XXS> {
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + (n >> 3) * IQ3_XXS::kBytes;
        const int ib = n & 7;
        const uint32_t aux = word_at(b + 66 + 4 * ib);
        const float db = mul_rn(mul_rn(half_at(b), 0.5f + float(aux >> 28)), 0.5f);
        const uint32_t q0 = word_at(b + 2 + 8 * ib), q1 = word_at(b + 6 + 8 * ib);
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            const uint32_t qb = ((l < 4 ? q0 : q1) >> (8 * (l & 3))) & 255u;
            const uint32_t sign = uint32_t(__ldg(&kKsigns[(aux >> (7 * (l >> 1))) & 127])) >> (4 * (l & 1));
            grid4(__ldg(&kIq3xxsGrid[qb]), db, sign, w + 4 * l);
        }
    }
};

template <>
struct Staged<IQ3_S> {
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + (n >> 3) * IQ3_S::kBytes;
        const int ib = n & 7;
        const float db = mul_rn(half_at(b), float(1 + 2 * ((b[106 + (ib >> 1)] >> (4 * (ib & 1))) & 15)));
        const uint32_t high = b[66 + ib];
        const uint32_t q0 = word_at(b + 2 + 8 * ib), q1 = word_at(b + 6 + 8 * ib);
        const uint32_t signs = word_at(b + 74 + 4 * ib);
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            const uint32_t qb = ((l < 4 ? q0 : q1) >> (8 * (l & 3))) & 255u;
            const uint32_t sign = signs >> (4 * l);
            grid4(__ldg(&kIq3sGrid[qb | (((high >> l) & 1u) << 8)]), db, sign, w + 4 * l);
        }
    }
};

template <>
struct Staged<IQ4_XS> {
    __device__ static void run(const uint8_t* row, int n, float* w) {
        const uint8_t* b = row + (n >> 3) * IQ4_XS::kBytes;
        const int ib = n & 7;
        const uint32_t ls = ((b[4 + (ib >> 1)] >> (4 * (ib & 1))) & 15u) | (((u16le(b + 2) >> (2 * ib)) & 3u) << 4);
        const float dl = mul_rn(half_at(b), float(int(ls) - 32));
        const uint8_t* q = b + 8 + 16 * ib;
        // the codebook value k as the float (2^23 + k + 128) - (2^23 + 128)
        const auto kv = [](uint32_t i) {
            return __fsub_rn(__int_as_float(0x4B000000 | (int(__ldg(&kKvalues[i])) + 128)), kF0 + 128.0f);
        };
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
            const uint32_t v = word_at(q + i);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t byte = (v >> (8 * j)) & 255u;
                w[i + j] = mul_rn(dl, kv(byte & 15u));
                w[16 + i + j] = mul_rn(dl, kv(byte >> 4));
            }
        }
    }
};

// Dispatch a GGML type id to a functor templated on the block struct. Returns SMOE_EKIND if unknown.
template <typename F>
inline int dispatch_kind(int kind, F&& f) {
    switch (kind) {
        case Q8_0::kKind: f(Q8_0{}); return SMOE_OK;
        case Q2_K::kKind: f(Q2_K{}); return SMOE_OK;
        case Q3_K::kKind: f(Q3_K{}); return SMOE_OK;
        case Q4_K::kKind: f(Q4_K{}); return SMOE_OK;
        case Q5_K::kKind: f(Q5_K{}); return SMOE_OK;
        case Q6_K::kKind: f(Q6_K{}); return SMOE_OK;
        case IQ3_XXS::kKind: f(IQ3_XXS{}); return SMOE_OK;
        case IQ3_S::kKind: f(IQ3_S{}); return SMOE_OK;
        case IQ4_XS::kKind: f(IQ4_XS{}); return SMOE_OK;
        case IQ4_NL::kKind: f(IQ4_NL{}); return SMOE_OK;
        case Q2_0::kKind: f(Q2_0{}); return SMOE_OK;
        case IQ2_XXS::kKind: f(IQ2_XXS{}); return SMOE_OK;
        case IQ2_XS::kKind: f(IQ2_XS{}); return SMOE_OK;
        case IQ2_S::kKind: f(IQ2_S{}); return SMOE_OK;
        case IQ1_M::kKind: f(IQ1_M{}); return SMOE_OK;
        default: return SMOE_EKIND;
    }
}

inline bool block_info(int kind, int& per, int& bytes) {
    return dispatch_kind(kind, [&](auto blk) {
               per = decltype(blk)::kPer;
               bytes = decltype(blk)::kBytes;
           }) == SMOE_OK;
}

}  // namespace smoe
