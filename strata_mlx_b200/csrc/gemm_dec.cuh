// Decoders of the grouped GEMM's A operand: 64 weights of one row (a thread's quarter of a 256-column stage)
// to exact float16 pairs.
//
// A stage's raw blocks are staged row by row (the 16-byte aligned cover of each row's bytes, rows an odd number
// of 16-byte chunks apart); a thread reads the fields its quarter needs as 32-bit words (BlockWords). A
// decoder leaves its 64 weights, in column order, as 32 float16 pairs in registers; the converged warp then
// stores them with tcgen05.st (a .sync.aligned instruction). Every weight is the float32 weight of gguf-py
// rounded to float16 once (the reference's tiles round to the activations' type, strata_mlx/blocks.py:610).
#pragma once

#include "blocks.cuh"
#include "tc05.cuh"

namespace smoe {

// The bytes of one block staged in shared memory, read as 32-bit words: the block starts `A` bytes past the
// 4-byte aligned `base` (A = the block's offset mod 4, a template argument: 0 for Q2_K and Q8_0 rows, 0 or 2
// for IQ3_S), so the word and the shift of every field are known at compile time. Rows are an odd number of
// 16-byte chunks apart: a warp's 32 rows read a word 4 banks to a row, 4-way conflicted, with no register
// realignment.
template <int A>
struct BlockWords {
    const uint32_t* base;
    template <int P>
    __device__ __forceinline__ uint32_t at() const {  // the 4 bytes at byte P of the block
        constexpr int t = A + P;
        if constexpr ((t & 3) == 0) return base[t >> 2];
        else return __funnelshift_r(base[t >> 2], base[(t >> 2) + 1], 8 * (t & 3));
    }
    template <int P>
    __device__ __forceinline__ uint32_t half_at() const {  // the 2 bytes at byte P (low half)
        constexpr int t = A + P;
        if constexpr ((t & 3) == 3) return at<P>() & 0xffffu;
        else return (base[t >> 2] >> (8 * (t & 3))) & 0xffffu;
    }
};

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

// Q2_K (84 bytes: scales 0..15, qs 16..79, d 80, dmin 82): quarter Q of the block is half H = Q / 2 (qs bytes
// 16 + 32 H .. + 31) at shifts 2 (Q % 2) and 2 (Q % 2) + 1; sub-block 8 H + 2 shift + (byte >= 16) scales 16
// weights. Per sub-block the four possible weights (code 0..3) are worked out once in float32, rounded to
// float16, and every weight is then a byte-permute lookup of its code.
struct GdQ2K {
    static constexpr int kKind = 10, kOffStep = 4;
    static constexpr bool kLut = false;
    template <int Q, int A>
    __device__ static void decode(const BlockWords<A>& bw, uint32_t (&out)[32], const uint32_t*, const uint32_t*) {
        constexpr int H = Q >> 1;
        const uint32_t dd = bw.template at<80>();
        const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(dd & 0xffffu)));
        const float dmin = __half2float(__ushort_as_half(static_cast<unsigned short>(dd >> 16)));
        const uint32_t sc = bw.template at<4 * (2 * H + (Q & 1))>();  // scales of sub-blocks 8 H + 4 (Q % 2) .. + 3
        uint32_t qs[8];
        qs[0] = bw.template at<16 + 32 * H>();
        qs[1] = bw.template at<20 + 32 * H>();
        qs[2] = bw.template at<24 + 32 * H>();
        qs[3] = bw.template at<28 + 32 * H>();
        qs[4] = bw.template at<32 + 32 * H>();
        qs[5] = bw.template at<36 + 32 * H>();
        qs[6] = bw.template at<40 + 32 * H>();
        qs[7] = bw.template at<44 + 32 * H>();
#pragma unroll
        for (int ss = 0; ss < 2; ++ss) {
            const int s = 2 * (Q & 1) + ss;
            uint32_t* v = out + 16 * ss;
#pragma unroll
            for (int half16 = 0; half16 < 2; ++half16) {
                const uint32_t sb = (sc >> (8 * (2 * ss + half16))) & 255u;
                const float dl = __fmul_rn(d, float(sb & 15u)), ml = __fmul_rn(dmin, float(sb >> 4));
                const uint32_t t01 = tc::pack_half2(fmaf(dl, 0.f, -ml), fmaf(dl, 1.f, -ml));
                const uint32_t t23 = tc::pack_half2(fmaf(dl, 2.f, -ml), fmaf(dl, 3.f, -ml));
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint32_t c = (qs[4 * half16 + kk] >> (2 * s)) & 0x03030303u;  // four codes
                    const uint32_t sel = c * 34u + 0x10101010u;  // nibbles 2q, 2q+1
                    v[2 * (4 * half16 + kk)] = prmt(t01, t23, sel);
                    v[2 * (4 * half16 + kk) + 1] = prmt(t01, t23, sel >> 16);
                }
            }
        }
    }
};

// IQ3_S (110 bytes: d 0, qs 2..65, qh 66..73, signs 74..105, scales 106..109): runs 2 Q, 2 Q + 1; a group of
// four weights is a codebook word (lane-replicated table), expanded to the exact float16 integers
// grid * (1 + 2 sub-scale) with the signs, then one rounding d * that.
struct GdIQ3S {
    static constexpr int kKind = 21, kOffStep = 2;
    static constexpr bool kLut = true;
    template <int IB, int A>
    __device__ static void run(const BlockWords<A>& bw, uint32_t d2, uint32_t qh, uint32_t sc, uint32_t* v,
                               const uint32_t* lut, const uint32_t* mc) {
        const uint32_t q0 = bw.template at<2 + 8 * IB>(), q1 = bw.template at<6 + 8 * IB>();
        const uint32_t sg = bw.template at<74 + 4 * IB>();
        const uint2 mcv = reinterpret_cast<const uint2*>(mc)[sc & 15u];
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
    }
    template <int Q, int A>
    __device__ static void decode(const BlockWords<A>& bw, uint32_t (&out)[32], const uint32_t* lut, const uint32_t* mc) {
        const uint32_t d2 = dup_half(bw.template half_at<0>());
        const uint32_t qh2 = bw.template half_at<66 + 2 * Q>();  // qh bytes of runs 2Q, 2Q + 1
        const uint32_t sc = bw.template half_at<106 + Q>() & 255u;  // sub-scale nibbles of runs 2Q, 2Q + 1
        run<2 * Q + 0>(bw, d2, qh2 & 255u, sc, out, lut, mc);
        run<2 * Q + 1>(bw, d2, qh2 >> 8, sc >> 4, out + 16, lut, mc);
    }
};

// Q8_0 (34 bytes: d 0, qs 2..33): blocks 2 Q, 2 Q + 1 of the stage's eight; a weight is d * q rounded once
// to float16.
struct GdQ8_0 {
    static constexpr int kKind = 8, kOffStep = 4;
    static constexpr bool kLut = false;
    template <int P, int A>
    __device__ static void block(const BlockWords<A>& bw, uint32_t* v) {  // the block at byte P
        const uint32_t d2 = dup_half(bw.template half_at<P>());
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            uint32_t q;
            switch (k) {  // the compile-time byte position of word k of the block
                case 0: q = bw.template at<P + 2>(); break;
                case 1: q = bw.template at<P + 6>(); break;
                case 2: q = bw.template at<P + 10>(); break;
                case 3: q = bw.template at<P + 14>(); break;
                case 4: q = bw.template at<P + 18>(); break;
                case 5: q = bw.template at<P + 22>(); break;
                case 6: q = bw.template at<P + 26>(); break;
                default: q = bw.template at<P + 30>(); break;
            }
            q ^= 0x80808080u;  // int8 -> code + 128
            v[2 * k] = h2mul(h2sub(prmt(q, 0x6464u, 0x4140), 0x64806480u), d2);
            v[2 * k + 1] = h2mul(h2sub(prmt(q, 0x6464u, 0x4342), 0x64806480u), d2);
        }
    }
    template <int Q, int A>
    __device__ static void decode(const BlockWords<A>& bw, uint32_t (&out)[32], const uint32_t*, const uint32_t*) {
        block<68 * Q>(bw, out);
        block<68 * Q + 34>(bw, out + 16);
    }
};

}  // namespace smoe
