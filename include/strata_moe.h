/*
 * strata_moe.h: C ABI of the B200 (sm_100a) mixture-of-experts hot path on GGUF quant blocks.
 *
 * Every entry point replaces one kernel-launching function of yibie/strata-mlx's Python modules
 * `strata_mlx/blocks.py` and `strata_mlx/fused.py` (cited beside each declaration). The Python facade
 * `strata_mlx_b200.blocks` / `strata_mlx_b200.fused` binds them with ctypes; any other host language binds
 * the same symbols (plain C types only: pointers, sizes, int codes).
 *
 * Conventions
 *   - Pointers are CUDA device pointers unless named `host_*`. Blocks are the GGUF file's raw bytes of a
 *     stack (experts, rows, cols): row r of expert e starts at (e*rows + r) * row_bytes, with
 *     row_bytes = cols / per_block * block_bytes (strata_mlx/blocks.py:296-297).
 *   - `kind` is the GGML type id of the blocks (8 Q8_0, 10 Q2_K, 11 Q3_K, 12 Q4_K, 13 Q5_K, 14 Q6_K,
 *     16 IQ2_XXS, 17 IQ2_XS, 18 IQ3_XXS, 20 IQ4_NL, 21 IQ3_S, 22 IQ2_S, 23 IQ4_XS, 29 IQ1_M, 42 Q2_0).
 *   - `dtype` codes: SMOE_F32 = 0, SMOE_F16 = 1. Activations and results take the activations' type unless
 *     a declaration says float32.
 *   - `stream` is a cudaStream_t (0 = legacy default stream). Every call that takes a stream is asynchronous
 *     on it, allocates nothing, synchronises nothing and so can be captured in a CUDA graph. The calls without
 *     a stream (the *_status reads, smoe_matvec_wait_test, the exchange buffers' alloc / open / close /
 *     free) synchronise or allocate and belong outside capture.
 *   - Return value: 0 on success; > 0 an invalid argument (SMOE_E*), with a message from
 *     smoe_last_error(); < 0 the negated cudaError_t of a failed launch.
 */
#ifndef STRATA_MOE_H
#define STRATA_MOE_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SMOE_API __attribute__((visibility("default")))
#else
#define SMOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum { SMOE_F32 = 0, SMOE_F16 = 1 };
enum {
    SMOE_OK = 0,
    SMOE_EKIND = 1,      /* block type not supported by this entry point */
    SMOE_ESHAPE = 2,     /* a dimension does not divide into blocks / tiles, or is out of range */
    SMOE_EDTYPE = 3,     /* activation type not supported */
    SMOE_EARG = 4,       /* null pointer, misaligned pointer, or an inconsistent count */
    SMOE_EWORKSPACE = 5, /* workspace missing or smaller than the *_workspace_size query asked for */
    SMOE_ETIMEOUT = 6    /* a bounded device-side wait gave up (status read back by the host) */
};

/* Human-readable message of the last error returned on this host thread. */
SMOE_API const char* smoe_last_error(void);

/* Library version and the CUDA architecture it was built for (e.g. 1000 for sm_100a). */
SMOE_API int smoe_version(void);
SMOE_API int smoe_built_arch(void);

/* Weights per block and bytes per block of a GGML type id (strata_mlx/blocks.py:36-38 BLOCK,
 * strata_mlx/gguf.py:25-33 TYPES). Returns SMOE_EKIND for types without a decoder here. */
SMOE_API int smoe_block_info(int kind, int* per_block, int* block_bytes);

/* Every weight of `n_rows` rows of `cols` weights as float16/float32: out[r, c].
 * Replaces `dequantize` / the `_DEQUANT` kernel (strata_mlx/blocks.py:261-270, 515-522). The float16
 * result is the float32 weight rounded to nearest even once, bit-equal to gguf-py's dequantize. */
SMOE_API int smoe_dequant(int kind, const uint8_t* blocks, int64_t n_rows, int64_t cols, void* out, int out_dtype,
                 void* stream);

/* out[p, r] = W[idx[p], r, :] . x[p / share, :] for p < pairs, r < rows; float32 sums.
 * W is a stack (experts, rows, cols) of `kind` blocks. x and out are `dtype`.
 * Replaces `BlockSwitchLinear.__call__` / the `_MATVEC` kernel (strata_mlx/blocks.py:196-220, 525-554):
 * share = 1 gives a row of x to every pair (down), share = k one to each run of k pairs (gate, up).
 * Indices >= experts are an error on the host side only if detected there; the kernel skips such pairs
 * (their output rows are left as they were). Kernels by type and dtype: IQ3_S and Q8_0 with float16 x on the
 * int8 tensor cores (x split into int8 hi / lo; up to four pairs of a one-expert stack in one pass over its
 * weights; pairs whose activations do not fit one launch in several), the K-types with float16 x on int8
 * dot products on the CUDA cores, everything else (and float32 x) on float32 CUDA-core sums; the int8 forms
 * stay within 1e-3 of the largest value of the exact product. */
SMOE_API int smoe_matvec(int kind, const uint8_t* blocks, int64_t experts, int64_t rows, int64_t cols,
                const uint32_t* idx, int64_t pairs, int64_t share, const void* x, void* out, int dtype,
                void* stream);

/* The int8 tensor-core decode kernels (the IQ3_S / Q8_0 paths of smoe_matvec, smoe_matvec_gate_up,
 * smoe_matvec_glu, smoe_matvec_batch and smoe_matvec_glu_combine) bound every wait for a weight copy (about a
 * second). A wait that gives up stops the warp's copies, records SMOE_ETIMEOUT in a status word on the device,
 * and leaves that launch's outputs not valid. smoe_matvec_status synchronizes the current device and reads the
 * word (0 or SMOE_ETIMEOUT); `clear` zeroes it. smoe_matvec_wait_test is for tests that make a wait run out:
 * it sets, on the current device, the bound in polls (each suspends the waiting thread up to 1 ms; < 0 restores
 * the default) and, with `withhold` 1, has every warp leave its first weight copy unissued, so that the wait for it
 * runs out, or with `withhold` 2 has smoe_route_matvec_batch's fused launch never announce its route, so that
 * the routed products' waits for it run out; it synchronizes the device. No counterpart in the reference (its
 * kernels have no device-side waits). */
SMOE_API int smoe_matvec_status(int* status, int clear);
SMOE_API int smoe_matvec_wait_test(int64_t polls, int withhold);

/* The gate and up products of the same pairs in one launch: two smoe_matvec calls sharing idx and x
 * (strata_mlx/blocks.py:971 `g, u = gate(x5, indices), up(x5, indices)`). The two stacks may differ in
 * kind but have the same shape. */
SMOE_API int smoe_matvec_gate_up(int gate_kind, const uint8_t* gate_blocks, int up_kind, const uint8_t* up_blocks,
                        int64_t experts, int64_t rows, int64_t cols, const uint32_t* idx, int64_t pairs,
                        int64_t share, const void* x, void* gate_out, void* up_out, int dtype, void* stream);

/* out[p, :] = W[idx[p]] . swiglu(gate[p, :], up[p, :]) with swiglu formed as mlx-lm forms it in the
 * activations' type (sigmoid in float32 rounded to the type, then two products in the type).
 * Replaces `matvec_glu` / `_MATVEC_GLU` (strata_mlx/blocks.py:225-259, 939-955); unlike the reference it
 * takes any pair count. gate/up are (pairs, cols), out (pairs, rows), all `dtype`. */
SMOE_API int smoe_matvec_glu(int kind, const uint8_t* blocks, int64_t experts, int64_t rows, int64_t cols,
                    const uint32_t* idx, int64_t pairs, const void* gate, const void* up, void* out, int dtype,
                    void* stream);

/* Several products of the decode path in one launch (the routed experts' gate and up with the shared
 * expert's gate and up; or the two down products): each problem is an smoe_matvec (x set, gate and up null)
 * or an smoe_matvec_glu (x null, gate and up set; share is then 1). Problems that name the same activations
 * read them once. All problems are done when the call returns to the stream, in one int8 tensor-core launch
 * when it takes all of them (float16 activations, IQ3_S / Q8_0, at most 4), else one launch per problem.
 * A problem with out, x, gate and up all null is not computed: it names weights a later launch reads (the
 * blocks of experts idx[0 .. pairs) of its stack), which the one launch fetches into L2 while it streams its
 * own (at most two such; a hint, dropped when the batch is not one launch).
 * No single reference counterpart: it batches the calls of `_Routed.__call__` (strata_mlx/fused.py:492-494)
 * that do not depend on one another. */
typedef struct SmoeMatvec {
    int kind;
    const uint8_t* blocks;
    int64_t experts, rows, cols;
    const uint32_t* idx;
    int64_t pairs, share;
    const void *x, *gate, *up;
    void* out;
    int dtype;
} SmoeMatvec;
SMOE_API int smoe_matvec_batch(int n, const SmoeMatvec* problems, void* stream);

/* The shared expert's down product with the end of the MoE block as its epilogue: for t < tokens,
 * out[t, r] = half(sum_j y[t,j,r] w[t,j]) + half(half(sigmoid(g[t])) half(W . swiglu(gate[t], up[t]))[r]),
 * exactly smoe_matvec_glu into s followed by smoe_combine(y, w, g, s) (the same functions, so the same bits for
 * the same product). W is one expert's stack (1, rows, cols), idx `tokens` zeros; float16 activations, IQ3_S
 * or Q8_0 blocks with cols a multiple of 256 (SMOE_ESHAPE otherwise). No single reference counterpart: it
 * fuses `shared_expert(x)` (strata_mlx/load.py:419-421) with `moe_combine` (strata_mlx/fused.py:448-481). */
SMOE_API int smoe_matvec_glu_combine(int kind, const uint8_t* blocks, int64_t rows, int64_t cols, const uint32_t* idx,
                                     int64_t tokens, const void* gate, const void* up, const void* y, const float* w,
                                     const void* g, int64_t k, void* out, int dtype, void* stream);

/* h = swiglu(gate, up) elementwise over n values of `dtype`: mlx-lm's `swiglu` as restated at
 * strata_mlx/blocks.py:222-237 (the unfused form `down(swiglu(g, u), indices)`, blocks.py:976). */
SMOE_API int smoe_swiglu(const void* gate, const void* up, int64_t n, void* out, int dtype, void* stream);

/* smoe_swiglu from float32 gate and up (a tile product's sums) to float16 out: the float32 SwiGLU rounded once,
 * `swiglu(g, u).astype(x.dtype)` of the tiled path (strata_mlx/blocks.py:690-692); with out_dtype == dtype it is
 * smoe_swiglu. */
SMOE_API int smoe_swiglu_to(const void* gate, const void* up, int64_t n, int dtype, void* out, int out_dtype,
                            void* stream);

/* Router product: logits[t, e] = W[e, :] . x[t, :], W float16 (experts, hidden), x `x_dtype`
 * (tokens, hidden), float32 sums and result. A token's sum does not depend on `tokens`.
 * Replaces `WindowLinear.__call__` / `_MATVEC` of fused.py (strata_mlx/fused.py:334-390). */
SMOE_API int smoe_router_logits(const uint16_t* weight, const void* x, int x_dtype, int64_t tokens, int64_t experts,
                       int64_t hidden, float* logits, void* stream);

/* idx[t, :] = the k largest of logits[t, :] (float32, n per row), largest first, ties to the lower index:
 * `mx.argpartition(-logits, k - 1)[..., :k]`. Replaces `top_k` / `_TOPK` (strata_mlx/fused.py:400-436);
 * any n <= 2048 and k <= 32, rows of any count. If `weights` is not null it also receives
 * softmax(logits[t, idx[t, :]]) in float32 (strata_mlx/fused.py:491, `mx.softmax(..., precise=True)`). */
SMOE_API int smoe_top_k(const float* logits, int64_t rows, int64_t n, int64_t k, uint32_t* idx, float* weights,
               void* stream);

/* The start of the MoE block in one launch: smoe_router_logits into `logits` (tokens, experts), then
 * smoe_top_k with weights into idx / weights (tokens, k), and, when `gate_weight` (1, hidden, float16) is
 * given, the shared expert's gate value gate_out[t] = (gate_weight . x[t]) rounded to x's type: the first
 * three lines of `_Routed.__call__` (strata_mlx/fused.py:487-491, `shared_expert_gate(x).to(x.dtype)`) with the
 * same sums and choice as the separate calls. experts <= 2048, k <= 32. `counters`: smoe_route_counters(tokens)
 * bytes of device memory, zero before the first call; every call leaves them zero. Calls that share counters
 * must not overlap on the GPU. No single reference counterpart: it fuses the three. */
SMOE_API size_t smoe_route_counters(int64_t tokens);
SMOE_API int smoe_route(const uint16_t* weight, const uint16_t* gate_weight, const void* x, int x_dtype,
                        int64_t tokens, int64_t experts, int64_t hidden, int64_t k, float* logits, uint32_t* idx,
                        float* weights, void* gate_out, uint32_t* counters, void* stream);
/* smoe_route that also writes the expert-parallel rank's view of the choice in the same launch: lidx[t, j] =
 * idx[t, j] - lo for the rank's experts [lo, lo + count), else `count` (what smoe_localize writes). No counterpart
 * in the reference (one device): it fuses smoe_localize into the start of `_Routed.__call__`. */
SMOE_API int smoe_route_local(const uint16_t* weight, const uint16_t* gate_weight, const void* x, int x_dtype,
                              int64_t tokens, int64_t experts, int64_t hidden, int64_t k, float* logits, uint32_t* idx,
                              float* weights, void* gate_out, uint32_t* counters, int64_t lo, int64_t count,
                              uint32_t* lidx, void* stream);

/* The route of a decode step and the products that read it, in one launch where the kernel takes them:
 * smoe_route (lidx NULL) or smoe_route_local (lidx set), then smoe_matvec_batch(n, problems) -- the same
 * logits, idx, weights, gate_out and lidx, and the same products within the batch's rounding (its teams may
 * group a product's partial sums differently from another batch). A problem whose idx points into the route's
 * idx or lidx reads the route's choice: the launch's CTAs each take two router rows, the last CTA in takes the
 * top-k, and the copies of the routed experts' weights start once it has; the other problems' (the shared
 * expert's) run meanwhile. Taken for float16 x, at most 8 tokens and 256 experts and the batch's one-launch
 * problems; otherwise the two calls run one after the other. `counters`: smoe_route_step_counters(tokens)
 * bytes, zero before the first call (calls sharing them must not overlap on the GPU): two words for the fused
 * launch, then smoe_route's counters for the two calls' form. No single reference
 * counterpart: it fuses the start of `_Routed.__call__` (strata_mlx/fused.py:487-491) with the first products
 * of `switch_mlp` and `shared_expert` (strata_mlx/blocks.py:939-986, strata_mlx/load.py:419-421). */
typedef struct SmoeRouteStep {
    const uint16_t* weight;       /* router (experts, hidden), float16 */
    const uint16_t* gate_weight;  /* the shared gate (1, hidden), float16, or NULL */
    const void* x;                /* (tokens, hidden) of x_dtype */
    int x_dtype;
    int64_t tokens, experts, hidden, k;
    float* logits;                /* (tokens, experts) */
    uint32_t* idx;                /* (tokens, k) */
    float* weights;               /* (tokens, k) */
    void* gate_out;               /* (tokens) of x_dtype; NULL with gate_weight NULL */
    uint32_t* counters;
    int64_t lo, count;            /* with lidx: this rank's experts [lo, lo + count) */
    uint32_t* lidx;               /* (tokens, k), or NULL */
} SmoeRouteStep;
SMOE_API size_t smoe_route_step_counters(int64_t tokens);
SMOE_API int smoe_route_matvec_batch(const SmoeRouteStep* route, int n, const SmoeMatvec* problems, void* stream);

/* The end of the MoE block: out[t, d] = half(sum_k y[t,k,d] w[t,k]) + half(half(sigmoid(g[t])) s[t,d]),
 * the sum in float32 in MLX's col_reduce_small order (partials j = k mod 8, then in order), every product
 * rounded, contraction off. y (tokens, k, d) `dtype`, w (tokens, k) float32, g (tokens) `dtype`,
 * s (tokens, d) `dtype`. Replaces `moe_combine` / `_COMBINE` (strata_mlx/fused.py:448-481) for any token
 * count and any d. */
SMOE_API int smoe_combine(const void* y, const float* w, const void* g, const void* s, int64_t tokens, int64_t k,
                 int64_t d, void* out, int dtype, void* stream);

/* Expert parallelism (N ranks, each holding the experts [lo, lo + count) of every layer and a 1/N slice of the
 * shared expert's ffn): the pieces around the one all-reduce of a decode step. No counterpart in the
 * reference, which runs on one device (strata_mlx has no multi-device code); they split
 * `_Routed.__call__` (strata_mlx/fused.py:487-497) at its combine.
 *   smoe_localize:     lidx = idx - lo for this rank's experts, else `count` (a pair the kernels leave out).
 *   smoe_partial_sums: sums[t, 0:d] = sum over this rank's pairs of y * w (MLX's order among them), float32;
 *                      sums[t, d:2d] = float(s[t]) (this rank's slice of the shared expert) or 0 if s is null.
 *   smoe_combine_sums: after the all-reduce of sums over ranks, out = half(routed) + half(half(sigmoid(g))
 *                      half(shared)), the combine of strata_mlx/fused.py:448-462 on the summed partials. */
SMOE_API int smoe_localize(const uint32_t* idx, int64_t n, int64_t lo, int64_t count, uint32_t* out, void* stream);
SMOE_API int smoe_partial_sums(const void* y, const float* w, const uint32_t* lidx, int64_t experts, const void* s,
                               int64_t tokens, int64_t k, int64_t d, float* sums, int dtype, void* stream);
SMOE_API int smoe_combine_sums(const float* sums, const void* g, int64_t tokens, int64_t d, void* out, int dtype,
                               void* stream);

/* The decode step's one exchange over NVLink peer memory, fused with the end of the block: it replaces the
 * smoe_partial_sums -> all-reduce -> smoe_combine_sums sequence above with one launch. No counterpart in the
 * reference (one device only); it is the same split of `_Routed.__call__` (strata_mlx/fused.py:487-497) at its
 * combine, with the same rounding points as smoe_combine_sums.
 *   smoe_ep_exchange_bytes:  bytes of one rank's exchange buffer for `ranks` ranks, up to max_tokens tokens of
 *                            d values (0 for sizes out of range: 1..16 ranks).
 *   smoe_ep_exchange_alloc:  cudaMalloc (zeroed) on the current device, and its CUDA IPC handle (64 bytes) for
 *                            the other ranks of the node; smoe_ep_exchange_free releases it.
 *   smoe_ep_exchange_open:   map another rank's buffer from its handle; smoe_ep_exchange_close unmaps it.
 *   smoe_ep_reduce_combine:  every rank calls it with the same shape, in the same order: rank r forms its float32
 *                            partials (routed: its pairs' y w in MLX's order; shared: float(s)), stores them into
 *                            every rank's buffer, waits for every rank's (bounded: about a second, or wait_polls
 *                            polls when not 0), adds them in rank order and writes
 *                            out = half(routed) + half(half(sigmoid(g)) half(shared)) -- the same bits on every
 *                            rank. Calls that share buffers must be ordered on the GPU (one stream). Each launch
 *                            counts itself in the buffer, so it can be captured in a CUDA graph and replayed.
 *   smoe_ep_exchange_status: synchronizes the device and reads this rank's status word (SMOE_ETIMEOUT when a wait
 *                            gave up; the outputs of that call were not written); `clear` zeroes it.
 *   smoe_ep_reduce_combine_emulated: every rank's call in one cooperative launch on one GPU (ranks 2..8, each
 *                            spec's peers naming the other specs' buffers): the exchange's arithmetic and order
 *                            on a machine with one GPU (tests). */
typedef struct SmoeEpReduce {
    int rank, ranks;
    void* peers[16];        /* every rank's exchange buffer as mapped here (peers[rank]: this rank's own) */
    const void* y;          /* (tokens, k, d) this rank's experts' outputs; rows of other ranks' pairs are not read */
    const float* w;         /* (tokens, k) */
    const uint32_t* lidx;   /* (tokens, k) local expert of each pair (smoe_localize), >= experts for another rank's */
    int64_t experts;        /* experts of this rank */
    const void* s;          /* (tokens, d) this rank's slice of the shared expert, or null */
    const void* g;          /* (tokens) the shared expert's gate value */
    int64_t tokens, k, d;
    int64_t capacity;       /* max_tokens x d of the buffers */
    void* out;              /* (tokens, d) */
    int dtype;
    uint32_t wait_polls;    /* 0: the default bound */
} SmoeEpReduce;
SMOE_API size_t smoe_ep_exchange_bytes(int64_t ranks, int64_t max_tokens, int64_t d);
SMOE_API int smoe_ep_exchange_alloc(size_t bytes, void** buffer, void* ipc_handle);
SMOE_API int smoe_ep_exchange_open(const void* ipc_handle, void** peer_buffer);
SMOE_API int smoe_ep_exchange_close(void* peer_buffer);
SMOE_API int smoe_ep_exchange_free(void* buffer);
SMOE_API int smoe_ep_exchange_status(void* buffer, int* failed, int clear);
SMOE_API int smoe_ep_reduce_combine(const SmoeEpReduce* r, void* stream);
SMOE_API int smoe_ep_reduce_combine_emulated(int ranks, const SmoeEpReduce* r, void* stream);

/* Expert parallelism for a prompt chunk (each rank holds its own tokens; rank r owns experts [r E/N, (r+1) E/N)):
 * the two ends of the all-to-all exchanges that carry the pairs to their experts' ranks and the outputs back.
 * Like the decode pieces above, no counterpart in the reference; together they split `_Routed.__call__`
 * (strata_mlx/fused.py:487-497) between the top-k and the combine.
 *   smoe_ep_dispatch:  from idx (pairs = tokens * k expert indices, flat), counts[ranks] = the pairs per
 *                      destination rank (idx / (experts / ranks)); where[pairs] = each pair's place in the send
 *                      order (destinations in rank order, one destination's pairs in pair order; -1 for an
 *                      index not below `experts`, which is not sent); send_expert[place] = the expert in its
 *                      owner's numbering; send_x[place] = the pair's token row of x (tokens, hidden) `dtype`.
 *                      send_expert and send_x hold `pairs` entries / rows; the first sum(counts) are written.
 *   smoe_combine_rows: smoe_combine with the experts' outputs read at y[where[t * k + j]] (the rows returned
 *                      by the exchange, in the send order) instead of y[t, j]; a pair with where -1 adds 0. */
SMOE_API int smoe_ep_dispatch(const uint32_t* idx, int64_t pairs, int64_t k, int64_t experts, int64_t ranks,
                              const void* x, int64_t hidden, int dtype, int32_t* counts, int32_t* where,
                              uint32_t* send_expert, void* send_x, void* stream);
SMOE_API int smoe_combine_rows(const void* y, const int32_t* where, const float* w, const void* g, const void* s,
                               int64_t tokens, int64_t k, int64_t d, void* out, int dtype, void* stream);

/* The hyper-connection around a block: the write of the block before it folded into the read of the residual
 * streams (strata_mlx/fused.py:46-146 `_NORM`, `_DOWN`, `_UP`; `FusedResidual.__call__`, 280-323), for `tokens`
 * tokens, hc streams of d values, a low rank of `rank`:
 *   residual = before + out * inject_in (before (tokens, hc d), out (tokens, d), inject_in (tokens, hc)), in the
 *              activations' type; normed = residual rsqrt(mean of its squares per stream + eps) norm, float32;
 *   total_j  = (row j of down, or of inject_w, . normed) / hc; low = total sigmoid(total) (rows of down, float32),
 *              inject = 2 sigmoid(total) (rows of inject_w, the activations' type), when inject_w is given;
 *   mixed[c] = sum over streams s of normed[s d + c] sigmoid(up[s d + c] . low) / hc, the activations' type.
 * Sums in float32 in an order fixed by the shapes, so a token gets the same bits alone as in a window. Weights
 * and activations share `dtype` (float16 or float32); down (rank, hc d), up (hc d, rank), inject_w (hc, hc d)
 * or null, norm (hc d), weights 16-byte aligned; d and rank multiples of 8, hc <= 8. Three launches;
 * smoe_hyper_workspace_size() bytes of device workspace (normed and low). */
typedef struct SmoeHyper {
    const void* norm;
    const void* down;
    const void* up;
    const void* inject_w;  /* or null: no inject output (the caller keeps inject_in) */
    int64_t hc, d, rank;
    float eps;
    int dtype;
} SmoeHyper;
SMOE_API size_t smoe_hyper_workspace_size(int64_t tokens, int64_t hc, int64_t d, int64_t rank);
SMOE_API int smoe_hyper_connection(const SmoeHyper* h, const void* before, const void* out, const void* inject_in,
                                   int64_t tokens, void* mixed, void* residual, void* inject, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* A Q3_K tensor held as planes (strata_mlx/blocks.py:399-512): its blocks (rows, cols) rearranged once into
 * hm (8 words a block: the high-bit mask), qs (16 words: the two-bit codes), sc (16 int8: the six-bit scales
 * less 32) and dd (the float16 d), 114 bytes a block for the file's 110; the same weights.
 *   smoe_q3k_planes:         the rearrangement (`q3k_planes`, blocks.py:403-414).
 *   smoe_q3k_planes_window:  out[t, r] = W . x[t] for tokens x (tokens, cols) -> (tokens, rows) in x's type
 *                            (`q3k_planes_window`, blocks.py:482-499); a token's bits do not depend on the window.
 *   smoe_q3k_planes_dequant: every weight (d scale) value as the block decoder forms it, rounded once
 *                            (`q3k_planes_dequantize`, blocks.py:502-512). */
SMOE_API int smoe_q3k_planes(const uint8_t* blocks, int64_t rows, int64_t cols, uint32_t* hm, uint32_t* qs,
                             int8_t* sc, uint16_t* dd, void* stream);
SMOE_API int smoe_q3k_planes_window(const uint32_t* hm, const uint32_t* qs, const int8_t* sc, const uint16_t* dd,
                                    int64_t rows, int64_t cols, const void* x, int64_t tokens, void* out, int dtype,
                                    void* stream);
SMOE_API int smoe_q3k_planes_dequant(const uint32_t* hm, const uint32_t* qs, const int8_t* sc, const uint16_t* dd,
                                     int64_t rows, int64_t cols, void* out, int dtype, void* stream);

/* A Q6_K tensor as ScaledLinear holds it (strata_mlx/dense.py:109-167): a weight is code * scale * d with codes
 * int8 (rows, cols) (the six bits less 32), scales int8 (rows, cols / 16), d float16 (rows, cols / d_step).
 *   smoe_q6k_parts:     the three parts from the file's blocks (`q6k_parts`, strata_mlx/gguf.py:150-165; d_step 256).
 *   smoe_scaled_window: out[t, r] = sum over groups of 16 of (d scale) (codes . x[t]), float32 sums, for tokens
 *                       x (tokens, cols) -> (tokens, rows) in x's type (`ScaledLinear.__call__`, dense.py:147-167);
 *                       codes 16-byte aligned; a token's bits do not depend on the window.
 *   smoe_scaled_floats: every weight (float(d) float(scale)) float(code) rounded once (`ScaledLinear.floats`,
 *                       dense.py:128-145). */
SMOE_API int smoe_q6k_parts(const uint8_t* blocks, int64_t rows, int64_t cols, int8_t* codes, int8_t* scales,
                            uint16_t* d, void* stream);
SMOE_API int smoe_scaled_window(const int8_t* codes, const int8_t* scales, const uint16_t* d, int64_t rows,
                                int64_t cols, int64_t d_step, const void* x, int64_t tokens, void* out, int dtype,
                                void* stream);
SMOE_API int smoe_scaled_floats(const int8_t* codes, const int8_t* scales, const uint16_t* d, int64_t rows,
                                int64_t cols, int64_t d_step, void* out, int dtype, void* stream);

/* The dispatch permutation of `pairs` = tokens * k expert indices (int32, flat) into tiles of 16 slots,
 * each tile one expert's: tile_expert[most] (experts for a tile nothing fills), token[most * 16] (0 in an
 * unfilled slot), where[pairs] (the slot of each pair), most = pairs / 16 + min(experts, pairs).
 * A pair's place within its expert follows its flat index. Replaces `tiles_of`
 * (strata_mlx/blocks.py:657-681). Needs smoe_tiles_of_workspace_size() bytes of device workspace. */
SMOE_API size_t smoe_tiles_of_workspace_size(int64_t pairs, int64_t experts);
SMOE_API int smoe_tiles_of(const int32_t* indices, int64_t pairs, int64_t k, int64_t experts, uint32_t* tile_expert,
                  uint32_t* token, uint32_t* where, void* workspace, size_t workspace_bytes, void* stream);

/* smoe_tiles_of for callers that cannot allocate device memory (a host framework that owns every device
 * allocation and gives a plugin only its inputs and outputs, or a loop that must not call cudaMalloc because it
 * can synchronize the device). No counterpart in the reference: it is an addition of this library. Same
 * arguments and results as smoe_tiles_of, without the workspace: its scratch is a fixed array of 1 MiB + 256
 * bytes in the library's device image (held by every GPU that loads the library until the process exits),
 * which limits it to smoe_tiles_of_workspace_size(pairs, experts) <= 1,048,832 bytes (131,072 pairs at 1,024
 * experts; 209,664 at 256) and returns SMOE_ESHAPE beyond. It allocates nothing. The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress) and keeps it for the life of the process; make that first call before
 * any stream capture, and make no call on a device after resetting it (the kept address is then stale). All
 * calls share the array: calls that overlap on the GPU race on it. */
SMOE_API int smoe_tiles_of_noalloc(const int32_t* indices, int64_t pairs, int64_t k, int64_t experts,
                                   uint32_t* tile_expert, uint32_t* token, uint32_t* where, void* stream);

/* Whether smoe_tile_matmul takes a stack of such rows (strata_mlx/blocks.py:629-631 `tileable`). */
SMOE_API int smoe_tileable(int kind, int64_t rows, int64_t cols);

/* out[p, :] = W[tile_expert[p / 16]] . a[p, :] for p < p16 (a multiple of 16), the weights rounded to a's
 * type (float16) before they multiply, float32 sums, out float32 (p16, rows). Tiles whose expert is
 * >= experts are left out (their rows of out are not written). Grouped GEMM on the 5th-generation tensor
 * cores (tcgen05, accumulators in TMEM). Replaces `tile_matmul` / `_TILES`
 * (strata_mlx/blocks.py:583-654). Needs smoe_tile_matmul_workspace_size() bytes of device workspace. */
SMOE_API size_t smoe_tile_matmul_workspace_size(int64_t p16);
SMOE_API int smoe_tile_matmul(int kind, const uint8_t* blocks, int64_t experts, int64_t rows, int64_t cols,
                     const void* a, int a_dtype, int64_t p16, const uint32_t* tile_expert, float* out,
                     void* workspace, size_t workspace_bytes, void* stream);

/* smoe_tile_matmul with its result read back in the caller's order and type: the sums of slot s, rounded once
 * to float16, go to row slot_row[s] of out (out_rows, rows) float16, or to row s without slot_row; rows at or past
 * out_rows are not written. Float16 activations a (a_rows <= p16 rows: the slots past a_rows multiply zeros, so a
 * dense layer's tokens need no padding to a whole tile), cols a multiple of 256 (the tensor-core kernel;
 * SMOE_ESHAPE otherwise). No single reference counterpart: it is `tile_matmul` followed by the read-back of the
 * tiled path, `out[where].astype(x.dtype)` (strata_mlx/blocks.py:684-694), in one launch. */
SMOE_API int smoe_tile_matmul_rows(int kind, const uint8_t* blocks, int64_t experts, int64_t rows, int64_t cols,
                                   const void* a, int64_t a_rows, int64_t p16, const uint32_t* tile_expert,
                                   const uint32_t* slot_row, int64_t out_rows, void* out, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* Two stacks of the same type and shape (a layer's gate and up) through the same tiles and activations in one
 * launch: out_a from blocks_a, out_b from blocks_b, each as smoe_tile_matmul gives it (float32, slot order) or,
 * the _rows form, as smoe_tile_matmul_rows gives it (float16 at slot_row's rows). Float16 activations and cols a
 * multiple of 256 (SMOE_EARG otherwise). Replaces the reference's two `product(gate, a)`, `product(up, a)` calls
 * of the tiled path (strata_mlx/blocks.py:690-692); one launch has one tail where two had two. Workspace as
 * smoe_tile_matmul's. */
SMOE_API int smoe_tile_matmul_pair(int kind, const uint8_t* blocks_a, const uint8_t* blocks_b, int64_t experts,
                                   int64_t rows, int64_t cols, const void* a, int64_t p16, const uint32_t* tile_expert,
                                   float* out_a, float* out_b, void* workspace, size_t workspace_bytes, void* stream);
SMOE_API int smoe_tile_matmul_pair_rows(int kind, const uint8_t* blocks_a, const uint8_t* blocks_b, int64_t experts,
                                        int64_t rows, int64_t cols, const void* a, int64_t a_rows, int64_t p16,
                                        const uint32_t* tile_expert, const uint32_t* slot_row, int64_t out_rows,
                                        void* out_a, void* out_b, void* workspace, size_t workspace_bytes,
                                        void* stream);

/* slot_row[s] = p for the pair p with where[p] = s (smoe_tiles_of's `where` inverted), 0xffffffff for slots no
 * pair fills: the map smoe_tile_matmul_rows takes to write a tiled product in pair order. slots entries. */
SMOE_API int smoe_slot_rows(const uint32_t* where, int64_t pairs, int64_t slots, uint32_t* slot_row, void* stream);

/* One MoE block's decode step for one float16 token in a single persistent launch: smoe_route (with the
 * shared gate), the four gate / up products of smoe_matvec_batch, the routed down product of smoe_matvec_glu
 * and smoe_matvec_glu_combine, as `_Routed.__call__` (strata_mlx/fused.py:487-497) runs them for one token.
 * Routed experts IQ3_S (gate / up (experts, ffn, hidden), down (experts, hidden, ffn)), the shared expert
 * Q8_0 (gate / up (1, sffn, hidden), down (1, hidden, sffn)); hidden and ffn multiples of 512, sffn of 256,
 * experts <= 256, k <= 32 (SMOE_EKIND / SMOE_ESHAPE otherwise). Outputs: logits [experts] float32, idx and
 * weights [k], gate_out (1 float16), out [hidden] float16 -- the same choice, and products within the int8
 * split's rounding of the separate calls. `scratch`: smoe_decode_layer_scratch() bytes of device memory,
 * zero before the first call and then left to the library (the launches count their grid barriers in it);
 * calls sharing a scratch must not overlap on the GPU. One CTA per SM, all resident together (a cooperative
 * launch); every wait on another CTA gives up after a second, leaving a flag that
 * smoe_decode_layer_status() reads (1: some wait gave up, the outputs are not valid). After a wait gave up the
 * scratch's barrier count is off: zero the scratch again before the next call. smoe_decode_layer_wait_test(1)
 * (for tests; it synchronizes the device) has one CTA skip its first arrival, so that the waits run out;
 * smoe_decode_layer_wait_test(0) restores it. No single reference counterpart: it fuses the four calls above. */
typedef struct SmoeDecodeLayer {
    const uint16_t* router;      /* [experts][hidden] float16 */
    const uint16_t* shared_gate; /* [hidden] float16, the shared expert's gate row */
    int64_t experts, hidden, k;
    int kind;                    /* 21 (IQ3_S) */
    const uint8_t *gate, *up, *down;
    int64_t ffn;
    int shared_kind;             /* 8 (Q8_0) */
    const uint8_t *sgate, *sup, *sdown;
    int64_t sffn;
    float* logits;
    uint32_t* idx;
    float* weights;
    void* gate_out;
    void* out;
    void* scratch;
} SmoeDecodeLayer;
SMOE_API size_t smoe_decode_layer_scratch(int64_t hidden, int64_t k, int64_t ffn, int64_t sffn);
SMOE_API int smoe_decode_layer(const SmoeDecodeLayer* layer, const void* x, void* stream);
SMOE_API int smoe_decode_layer_status(const void* scratch, int64_t hidden, int64_t k, int64_t ffn, int64_t sffn,
                                      int* failed);
SMOE_API int smoe_decode_layer_wait_test(int withhold);

#ifdef __cplusplus
}
#endif
#endif /* STRATA_MOE_H */
