// The int8 tensor-core decode matvec (smoe_mv8.cu) as the entry points of smoe_blocks.cu call it.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace smoe {

// One matvec problem: out[p, r] = W[idx[p], r, :] . a[p / share, :], a = x, or the SwiGLU of (gate, up).
struct M8Spec {
    int kind;
    const uint8_t* blocks;
    int64_t experts, rows, cols, row_bytes;
    const uint32_t* idx;
    int64_t pairs, share;
    const __half *x, *gate, *up;
    __half* out;
};

// A later launch's weights to fetch into L2 meanwhile: the blocks of experts idx[0 .. pairs) of a stack whose
// experts are expert_bytes apart.
struct M8Pref {
    const uint8_t* blocks;
    int64_t expert_bytes;
    const uint32_t* idx;
    int pairs;
    uint32_t experts;
};

// The route of the tokens whose products a launch takes (smoe_route / smoe_route_local in the same launch):
// router rows w (experts, hidden) and the shared gate row gw (or null) against x (tokens, hidden) float16 ->
// logits, idx, weights, gate_out, and with lidx set the pairs' local expert numbers (idx - lo where below
// count, else count). counters[0] counts the CTAs whose router rows are in; counters[1] is the launch number
// the CTA that takes the top-k moves on once idx is written. Problems whose idx is this idx or lidx read it
// once that number has moved.
struct M8Route {
    const __half *w, *gw, *x;
    float* logits;
    uint32_t* idx;
    float* weights;
    __half* gate_out;
    uint32_t* counters;
    uint32_t* lidx;
    uint32_t lo, count;
    int tokens, experts, hidden, k;
};

// n <= 4 problems in one launch (and up to two stacks' weights fetched into L2 for later launches, and the
// route of their tokens): 0 launched, 1 not taken (the caller runs them another way), else an error.
int mv8_batch(int n, const M8Spec* specs, cudaStream_t st, int npf = 0, const M8Pref* pf = nullptr,
              const M8Route* route = nullptr);

// the gate / up problems (nprob 1 or 2) of one stack pair: 0 launched, 1 not taken, else an error
int mv8_try(int kind0, int kind1, const uint8_t* b0, const uint8_t* b1, int64_t experts, int64_t rows, int64_t cols,
            int64_t row_bytes, const uint32_t* idx, int64_t pairs, int64_t share, const __half* x, const __half* gate,
            const __half* up, __half* o0, __half* o1, int nprob, cudaStream_t st);

// the shared expert's down product with the block's combine as its epilogue: 0 launched, 1 not taken, else an
// error (out[t, r] = the combine of y (tokens, k, rows), w (tokens, k), g (tokens) and the product)
int mv8_glu_combine(int kind, const uint8_t* blocks, int64_t rows, int64_t cols, int64_t row_bytes,
                    const uint32_t* idx, int64_t tokens, const __half* gate, const __half* up, const __half* y,
                    const float* w, const __half* g, int k, __half* out, cudaStream_t st);

}  // namespace smoe
