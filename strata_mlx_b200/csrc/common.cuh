// Shared helpers of the strata_moe CUDA library: status handling, float16 I/O, async copies.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <string>
#include <utility>

#include "../../include/strata_moe.h"

namespace smoe {

// ---- host side: errors

void set_error(const std::string& msg);  // defined in smoe_api.cu, thread-local message

inline int fail(int code, const std::string& msg) {
    set_error(msg);
    return code;
}

inline int launch_status(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error(std::string(what) + ": " + cudaGetErrorString(e));
        return -static_cast<int>(e);
    }
    return SMOE_OK;
}

#define SMOE_REQUIRE(cond, code, msg) \
    do {                              \
        if (!(cond)) return ::smoe::fail((code), (msg)); \
    } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Raise a kernel's dynamic shared-memory limit once per (kernel, device) instead of at every launch.
int set_max_smem(const void* kernel, int bytes);  // defined in smoe_api.cu
template <typename K>
inline int max_smem(K* kernel, int bytes) {
    return set_max_smem(reinterpret_cast<const void*>(kernel), bytes);
}

// ---- programmatic dependent launch
//
// A kernel launched with launch_pdl may start while the kernel before it in the stream is still running (its
// CTAs are placed as that kernel's CTAs finish). Before pdl_wait() it may only set up its own shared memory and
// read data that the launch before it does not write; pdl_wait() returns once that launch has completed and
// its writes are visible. Every kernel launched here calls pdl_release() only after its own pdl_wait(), so when
// a launch starts, every launch before the one just ahead of it has completed: data older than the previous
// launch (weights, codebooks, the router's choice two launches back) may be read before the wait, which
// pdl_early() tells the host. Outputs are written only after the wait. Launched without the attribute, or
// behind a kernel that never releases (any other library's), a kernel starts after its predecessor completed
// and pdl_wait() returns at once.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_release() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// The device memory one launch writes.
struct Writes {
    static constexpr int kMax = 12;
    const void* p[kMax] = {};
    size_t n[kMax] = {};
    int count = 0;
    bool all = false;  // more ranges than kMax: the launch counts as writing everything
    Writes& add(const void* ptr, size_t bytes) {
        if (ptr != nullptr && bytes > 0) {
            if (count < kMax) {
                p[count] = ptr;
                n[count] = bytes;
                ++count;
            } else {
                all = true;
            }
        }
        return *this;
    }
};
// Record what the launch just made on `st` with launch_pdl writes (the next launch on `st` may overlap it).
void pdl_note(cudaStream_t st, const Writes& w);  // defined in smoe_api.cu
// Whether the next launch on `st` may read [p, p + n) before its pdl_wait(): the last launch_pdl launch on
// `st` does not write it. (A record older than the stream's true last launch errs safe: that launch is then
// another kernel, which the next launch waits for in full.)
bool pdl_early(cudaStream_t st, const void* p, size_t n);  // defined in smoe_api.cu

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(const Writes& writes, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
    pdl_note(st, writes);
    return e;
}

// ---- device side: loads of little-endian fields of a block (any alignment)

__device__ __forceinline__ uint32_t u8(const uint8_t* p) { return p[0]; }
__device__ __forceinline__ uint32_t u16le(const uint8_t* p) { return uint32_t(p[0]) | (uint32_t(p[1]) << 8); }
__device__ __forceinline__ uint32_t u32le(const uint8_t* p) { return u16le(p) | (u16le(p + 2) << 16); }
__device__ __forceinline__ float half_at(const uint8_t* p) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(u16le(p))));
}

// activation types: float32 or float16, converted to/from float32
template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// ---- async copies (sm_80+ cp.async; 16-byte granularity, zero-fill past `valid` bytes)

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src, int valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_addr(smem_dst)), "l"(gmem_src),
                 "r"(valid));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}
__device__ __forceinline__ void cp_async_wait_dyn(int n) {
    // wait_group takes an immediate: dispatch the few depths used here
    switch (n) {
        case 0: cp_async_wait<0>(); break;
        case 1: cp_async_wait<1>(); break;
        case 2: cp_async_wait<2>(); break;
        case 3: cp_async_wait<3>(); break;
        case 4: cp_async_wait<4>(); break;
        case 5: cp_async_wait<5>(); break;
        case 6: cp_async_wait<6>(); break;
        default: cp_async_wait<7>(); break;
    }
}

// Copy bytes [src, src + n) of a blob that ends at `end` into smem starting at dst (16-byte aligned) with
// 16-byte copies from the aligned address at or below src; the bytes land at dst + (src & 15). Lanes
// `lane` of `width` share the work. Copies never read at or beyond `end`.
__device__ __forceinline__ int stage_bytes(uint8_t* dst, const uint8_t* src, int64_t n, const uint8_t* end,
                                           int lane, int width) {
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(src) & ~uintptr_t(15);
    const int off = static_cast<int>(reinterpret_cast<uintptr_t>(src) - a0);
    const int chunks = static_cast<int>((off + n + 15) >> 4);
    const uintptr_t e = reinterpret_cast<uintptr_t>(end);
    for (int c = lane; c < chunks; c += width) {
        const uintptr_t g = a0 + 16 * uintptr_t(c);
        int valid = e > g ? static_cast<int>(e - g < 16 ? e - g : 16) : 0;
        cp_async16(dst + 16 * c, reinterpret_cast<const void*>(g), valid);
    }
    return off;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float sigmoid_branch(float g) {
    // MLX's form: 1 / (1 + exp(|g|)) taken on the side that cannot overflow
    const float y = 1.0f / (1.0f + expf(fabsf(g)));
    return g < 0.0f ? y : 1.0f - y;
}

// silu(gate) * up in the activations' type T, as mlx-lm's swiglu works it out (strata_mlx/blocks.py:222-224):
// sigmoid in float32 rounded to T, then two products in T
template <typename T>
__device__ __forceinline__ T swiglu_one(T g, T u) {
    const float gf = to_f32(g);
    const T sig = from_f32<T>(sigmoid_branch(gf));
    const T a = from_f32<T>(__fmul_rn(gf, to_f32(sig)));
    return from_f32<T>(__fmul_rn(to_f32(a), to_f32(u)));
}

template <typename T> __device__ __forceinline__ T mul_t(T a, T b);
// the _rn forms: a product or sum rounded on its own, never contracted into a half FMA with its neighbour
template <> __device__ __forceinline__ __half mul_t<__half>(__half a, __half b) { return __hmul_rn(a, b); }
template <> __device__ __forceinline__ float mul_t<float>(float a, float b) { return __fmul_rn(a, b); }
template <typename T> __device__ __forceinline__ T add_t(T a, T b);
template <> __device__ __forceinline__ __half add_t<__half>(__half a, __half b) { return __hadd_rn(a, b); }
template <> __device__ __forceinline__ float add_t<float>(float a, float b) { return __fadd_rn(a, b); }

// One element of the MoE block's end (strata_mlx/fused.py:448-462): half(sum_j y_j w_j) + half(half(sigmoid(g))
// s), the sum in float32 in MLX's col_reduce_small order (partials j = k mod 8, then in order), every product
// and sum rounded on its own. y points at expert 0's value, the experts' values `stride` apart.
template <typename T>
__device__ __forceinline__ T combine_one(const T* __restrict__ y, int64_t stride, const float* __restrict__ w, int k,
                                         T g, T s) {
    const T gate = from_f32<T>(1.0f / (1.0f + expf(-to_f32(g))));
    float acc = 0.0f;
    if (k == 8) {
        // (the common case, its eight loads in flight together; the same sums in the same order)
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = to_f32(y[int64_t(j) * stride]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float part = __fadd_rn(__fmul_rn(v[j], w[j]), 0.0f);
            acc = j == 0 ? part : __fadd_rn(part, acc);
        }
    } else {
        for (int j = 0; j < 8 && j < k; ++j) {
            float part = 0.0f;
            for (int kk = j; kk < k; kk += 8) part = __fadd_rn(__fmul_rn(to_f32(y[int64_t(kk) * stride]), w[kk]), part);
            acc = j == 0 ? part : __fadd_rn(part, acc);
        }
    }
    const T routed = from_f32<T>(acc);
    return add_t<T>(routed, mul_t<T>(gate, s));
}

}  // namespace smoe
