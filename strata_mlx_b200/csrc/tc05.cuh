// Thin inline-PTX wrappers for sm_100a: mbarriers with bounded waits, TMEM allocation, tcgen05 MMA / load /
// store / commit, and the shared-memory matrix descriptor. Only what the grouped GEMM uses.
#pragma once

#include <cstdint>

namespace smoe {
namespace tc {

// ---- mbarrier

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar))),
                 "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}\n" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar))), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

constexpr uint64_t kWaitNs = 1000000000ull;  // a wait gives up after one second

// try_wait that may suspend the thread until the phase completes, for at most `hint_ns`
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar))), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Wait for the phase of `parity` to complete, at most `limit` polls (each suspends the thread until the phase
// completes or 1 ms passes) and at most kWaitNs in all. Returns false when it gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t limit) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 0; i < limit; ++i) {
        if (mbar_try_wait_hint(bar, parity, 1000000u)) return true;
        if (globaltimer_ns() - t0 > kWaitNs) return false;
    }
    return false;
}

// Arrive once on `bar` and raise its expected transaction count by `bytes` (bulk copies complete against it).
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(bar))),
                 "r"(bytes)
                 : "memory");
}

// Arrive once on `bar` when every cp.async this thread issued before has landed (counted in the init count).
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
                 : "memory");
}

// 2-D tiled TMA load of this GPU's global memory into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(uint32_t dst_smem, const void* tmap, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
            dst_smem),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y),
        "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
        : "memory");
}

// L2 eviction policies (createpolicy): evict_first for data read once (streamed weights), evict_last for data
// fetched ahead of the launch that reads it
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// tma_load_2d with an L2 cache policy
__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst_smem, const void* tmap, int x, int y, uint64_t* bar,
                                                 uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, %3}], "
        "[%4], %5;\n" ::"r"(dst_smem),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar))),
        "l"(policy)
        : "memory");
}

// Fetch [src, src + bytes) of global memory into L2 (no destination; 16-byte aligned, a multiple of 16 bytes)
__device__ __forceinline__ void prefetch_l2_bulk(const void* src, uint32_t bytes, uint64_t policy) {
    asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;\n" ::"l"(src), "r"(bytes), "l"(policy)
                 : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

__device__ __forceinline__ void named_barrier(int id, int threads) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(threads) : "memory");
}

// bar.sync on named barrier `id` over `threads` threads that also and-reduces a predicate
__device__ __forceinline__ bool bar_and(int id, int threads, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "barrier.cta.red.and.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}\n"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(v)), "r"(id), "r"(threads)
        : "memory");
    return r != 0;
}

// ---- tensor memory

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(dst_smem))),
                 "r"(cols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// 16 consecutive 32-bit columns of this thread's TMEM lane (32x32b shape: warp w reaches lanes 32(w%4)..+31)
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

// ---- MMA: D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16, one CTA

__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// The same, called by a whole converged warp: one elected lane issues. A warp-uniform issue keeps the MMA
// operands in the uniform datapath, which sustains one MMA per tensor-pipe slot (a branch on one lane does not).
__device__ __forceinline__ void mma_f16_ts_warp(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t.reg .b32 r;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "elect.sync r|e, 0xffffffff;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive once on `bar` when every MMA this thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
                 : "memory");
}

// The same, called by the whole converged warp that issued with mma_f16_ts_warp (the same lane is elected).
__device__ __forceinline__ void mma_commit_warp(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t.reg .b32 r;\n\t"
        "elect.sync r|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}\n" ::"r"(
            static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
        : "memory");
}

// Instruction descriptor, kind::f16: D float32, A and B float16, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n) {
    return (1u << 4)                              // D format: float32
           | (0u << 7) | (0u << 10)               // A, B format: float16
           | (0u << 15) | (0u << 16)              // A, B K-major
           | (uint32_t(n >> 3) << 17)             // N / 8
           | (uint32_t(m >> 4) << 24);            // M / 16
}

// Shared-memory descriptor of a K-major operand without swizzle: 8-row x 16-byte core matrices, rows of a
// core matrix 16 bytes apart; `lbo` bytes between the two 8-element halves of K, `sbo` bytes between groups
// of 8 rows. Version 1 (sm_100), base offset 0, layout type 0 (no swizzle).
__device__ __forceinline__ uint64_t smem_desc(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
    return uint64_t((smem_addr >> 4) & 0x3fff) | (uint64_t((lbo >> 4) & 0x3fff) << 16) |
           (uint64_t((sbo >> 4) & 0x3fff) << 32) | (uint64_t(1) << 46);
}

// Shared-memory descriptor of a K-major operand in the 128-byte swizzle layout that TMA writes with
// CU_TENSOR_MAP_SWIZZLE_128B: rows of 128 bytes (64 float16 of K), 8-row groups 1024 bytes apart, the atom
// 1024-byte aligned; a K step of 16 inside the atom advances the start address by 32 bytes. Version 1,
// layout type 2 (128-byte swizzle), leading byte offset unused (1).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t smem_addr) {
    return uint64_t((smem_addr >> 4) & 0x3fff) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
           (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;\n" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

}  // namespace tc
}  // namespace smoe
