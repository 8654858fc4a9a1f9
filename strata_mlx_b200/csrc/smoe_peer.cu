// The one exchange of an expert-parallel decode step, over NVLink / NVSwitch peer memory, fused with the end of
// the MoE block.
//
// Every rank holds an exchange buffer (cudaMalloc'd here, shared with the other ranks of the node through CUDA
// IPC handles). A launch of ex_reduce_kernel on rank r, each thread for its own output elements:
//   1. works out rank r's float32 partials of the element: the weighted sum of its own experts' outputs (MLX's
//      combine order among them) and its slice of the shared expert;
//   2. stores them into every other rank's inbox as two 8-byte words (value, launch sequence number): each word
//      is written by one single-copy-atomic 64-bit store, so a reader that sees the sequence number sees the
//      value with it -- no fence, no flag, no barrier between the threads;
//   3. reads every other rank's two words of the element until their sequence numbers are this launch's
//      (bounded polls of local memory);
//   4. adds the ranks' partials in rank order (so every rank forms the same bits) and applies the combine's
//      rounding: out = half(routed) + half(half(sigmoid(g)) half(shared)).
// The inbox is double-buffered by the sequence number's parity: a rank writes launch v + 1's words into the half
// another rank read in launch v - 1 only after receiving that rank's launch v words, which it writes after its
// launch v - 1 has completed. Each CTA keeps its own sequence counter in its rank's buffer, so CUDA graph replays
// need no host work. A wait that gives up records SMOE_ETIMEOUT in the buffer's status word
// (smoe_ep_exchange_status) and leaves that element's output unwritten.
//
// No TMA and no multicast: peer memory is only ever touched by plain loads and stores.
#include <algorithm>
#include <cstring>

#include "common.cuh"

namespace smoe {
namespace {

constexpr int kExMaxRanks = 16;  // ranks of one node
constexpr int kExMaxCtas = 128;  // CTAs of one launch (each owns a slice of the outputs)
constexpr int kExThreads = 128;
constexpr int kExMaxEmulated = 8;
constexpr uint32_t kExDefaultPolls = 1u << 26;
constexpr uint64_t kExWaitNs = 1000000000ull;  // a wait gives up after one second at most

// A rank's exchange buffer: status word, the CTAs' launch counters, the inbox: [2 halves][rank][element] of two
// 8-byte words (routed value, sequence number) and (shared value, sequence number).
constexpr size_t kExSeqOff = 256;
constexpr size_t kExInboxOff = (kExSeqOff + 4 * kExMaxCtas + 255) & ~size_t(255);
constexpr size_t kExSlot = 16;  // bytes per element per rank

struct ExRank {
    const void* y;          // (tokens, k, d): this rank's experts' outputs (rows of other ranks' pairs unread)
    const float* w;         // (tokens, k) combine weights
    const uint32_t* lidx;   // (tokens, k) local expert of each pair, >= experts for another rank's
    const void* s;          // (tokens, d) this rank's slice of the shared expert, or null
    const void* g;          // (tokens) the shared expert's gate value
    void* out;              // (tokens, d)
    uint8_t* peers[kExMaxRanks];  // every rank's exchange buffer as this rank maps it
    int rank;
};
struct ExLaunch {
    ExRank r[kExMaxEmulated];  // one, or (one GPU, a test) every emulated rank's
    int ranks, k;
    int64_t tokens, d, capacity;  // capacity: tokens x d values an inbox holds per rank
    uint32_t experts, polls;
    int release;  // trigger the next launch at the end (programmatic dependent launch)
};

__device__ __forceinline__ void st_word(uint2* p, float v, uint32_t seq) {
    asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(v)), "r"(seq) : "memory");
}
__device__ __forceinline__ uint2 ld_word(const uint2* p) {
    uint2 v;
    asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// the value of a word once its sequence number is `seq` (false: the wait gave up)
__device__ __forceinline__ bool wait_word(const uint2* p, uint32_t seq, uint32_t polls, float& v) {
    uint2 w = ld_word(p);
    if (w.y == seq) {
        v = __uint_as_float(w.x);
        return true;
    }
    const uint64_t t0 = now_ns();
    for (uint32_t i = 0; i < polls; ++i) {
        w = ld_word(p);
        if (w.y == seq) {
            v = __uint_as_float(w.x);
            return true;
        }
        if ((i & 255u) == 255u && now_ns() - t0 > kExWaitNs) break;
    }
    return false;
}

template <typename T>
__global__ void __launch_bounds__(kExThreads) ex_reduce_kernel(const __grid_constant__ ExLaunch L) {
    const ExRank& R = L.r[blockIdx.y];
    const int c = blockIdx.x;
    const int64_t n = L.tokens * L.d;
    const int64_t per = (n + gridDim.x - 1) / gridDim.x;
    const int64_t e0 = int64_t(c) * per, e1 = min(n, e0 + per);
    uint8_t* mine = R.peers[R.rank];
    __shared__ uint32_t s_seq;
    pdl_wait();
    if (threadIdx.x == 0) {
        uint32_t* seqp = reinterpret_cast<uint32_t*>(mine + kExSeqOff) + c;
        s_seq = *seqp + 1u;
        *seqp = s_seq;
    }
    __syncthreads();
    const uint32_t seq = s_seq;
    const int64_t half = seq & 1u;
    const T* y = static_cast<const T*>(R.y);
    const T* s = static_cast<const T*>(R.s);
    const T* g = static_cast<const T*>(R.g);
    T* out = static_cast<T*>(R.out);
    const int k = L.k;
    const int64_t row = 2 * L.capacity;  // words of one rank's part of a half
    bool ok = true;
    for (int64_t e = e0 + threadIdx.x; e < e1; e += blockDim.x) {
        const int64_t t = e / L.d, i = e - t * L.d;
        // 1. this rank's partials
        float acc = 0.0f;
        for (int j = 0; j < 8 && j < k; ++j) {
            float part = 0.0f;
            for (int kk = j; kk < k; kk += 8)
                if (R.lidx[t * k + kk] < L.experts)
                    part = __fadd_rn(__fmul_rn(to_f32(y[(t * k + kk) * L.d + i]), R.w[t * k + kk]), part);
            acc = j == 0 ? part : __fadd_rn(part, acc);
        }
        const float sh = s ? to_f32(s[e]) : 0.0f;
        // 2. to every other rank
        for (int p = 0; p < L.ranks; ++p) {
            if (p == R.rank) continue;
            uint2* box = reinterpret_cast<uint2*>(R.peers[p] + kExInboxOff) + (half * L.ranks + R.rank) * row + 2 * e;
            st_word(box, acc, seq);
            st_word(box + 1, sh, seq);
        }
        // 3-4. every rank's, in rank order
        const uint2* inbox = reinterpret_cast<const uint2*>(mine + kExInboxOff) + half * L.ranks * row + 2 * e;
        float routed = 0.0f, shared = 0.0f;
        bool have = true;
        for (int p = 0; p < L.ranks; ++p) {
            float vr = acc, vs = sh;
            if (p != R.rank) {
                have = have && wait_word(inbox + p * row, seq, L.polls, vr);
                have = have && wait_word(inbox + p * row + 1, seq, L.polls, vs);
            }
            routed = p == 0 ? vr : __fadd_rn(routed, vr);
            shared = p == 0 ? vs : __fadd_rn(shared, vs);
        }
        if (!have) {
            ok = false;
            continue;
        }
        const T gate = from_f32<T>(1.0f / (1.0f + expf(-to_f32(g[t]))));
        out[e] = add_t<T>(from_f32<T>(routed), mul_t<T>(gate, from_f32<T>(shared)));
    }
    if (!ok) atomicExch(reinterpret_cast<int*>(mine), SMOE_ETIMEOUT);
    if (L.release) pdl_release();
}

int ex_check(const SmoeEpReduce& r, int emulated_rank) {
    SMOE_REQUIRE(r.ranks >= 1 && r.ranks <= kExMaxRanks, SMOE_EARG, "ep_reduce: 1 to 16 ranks");
    SMOE_REQUIRE(r.rank >= 0 && r.rank < r.ranks, SMOE_EARG, "ep_reduce: rank out of range");
    SMOE_REQUIRE(emulated_rank < 0 || r.rank == emulated_rank, SMOE_EARG, "ep_reduce: emulated ranks in rank order");
    SMOE_REQUIRE(r.tokens >= 0 && r.k >= 1 && r.k <= 32 && r.d >= 1, SMOE_ESHAPE, "ep_reduce: bad shape");
    SMOE_REQUIRE(r.tokens * r.d <= r.capacity, SMOE_ESHAPE, "ep_reduce: more tokens than the buffers were made for");
    SMOE_REQUIRE(r.experts > 0 && r.experts <= 0xffffffffLL, SMOE_EARG, "ep_reduce: bad expert count");
    SMOE_REQUIRE(r.dtype == SMOE_F16 || r.dtype == SMOE_F32, SMOE_EDTYPE, "ep_reduce: float16 or float32 activations");
    if (r.tokens == 0) return SMOE_OK;
    SMOE_REQUIRE(r.y && r.w && r.lidx && r.g && r.out, SMOE_EARG, "ep_reduce: null pointer");
    for (int p = 0; p < r.ranks; ++p) {
        SMOE_REQUIRE(r.peers[p] != nullptr, SMOE_EARG, "ep_reduce: a rank's buffer is not mapped");
        SMOE_REQUIRE((reinterpret_cast<uintptr_t>(r.peers[p]) & 255) == 0, SMOE_EARG, "ep_reduce: misaligned buffer");
    }
    return SMOE_OK;
}

ExRank ex_rank(const SmoeEpReduce& r) {
    ExRank x = {};
    x.y = r.y;
    x.w = r.w;
    x.lidx = r.lidx;
    x.s = r.s;
    x.g = r.g;
    x.out = r.out;
    for (int p = 0; p < r.ranks; ++p) x.peers[p] = static_cast<uint8_t*>(r.peers[p]);
    x.rank = r.rank;
    return x;
}

int ex_launch(int emulated, const SmoeEpReduce* r, void* stream) {
    const SmoeEpReduce& r0 = r[0];
    ExLaunch L = {};
    for (int i = 0; i < emulated; ++i) {
        if (int s = ex_check(r[i], emulated > 1 ? i : -1)) return s;
        SMOE_REQUIRE(r[i].ranks == r0.ranks && r[i].tokens == r0.tokens && r[i].k == r0.k && r[i].d == r0.d &&
                         r[i].capacity == r0.capacity && r[i].experts == r0.experts && r[i].dtype == r0.dtype,
                     SMOE_EARG, "ep_reduce: emulated ranks differ in shape");
        L.r[i] = ex_rank(r[i]);
    }
    if (r0.tokens == 0) return SMOE_OK;
    L.ranks = r0.ranks;
    L.k = static_cast<int>(r0.k);
    L.tokens = r0.tokens;
    L.d = r0.d;
    L.capacity = r0.capacity;
    L.experts = static_cast<uint32_t>(r0.experts);
    L.polls = r0.wait_polls ? r0.wait_polls : kExDefaultPolls;
    L.release = emulated == 1;
    const int64_t n = r0.tokens * r0.d;
    // every rank must cut the outputs into the same slices: the CTA count depends on the shape alone (an
    // emulated launch, all ranks' CTAs resident together, takes fewer where they would not fit)
    int ctas = static_cast<int>(std::min<int64_t>(kExMaxCtas, (n + kExThreads - 1) / kExThreads));
    const void* fn = r0.dtype == SMOE_F16 ? reinterpret_cast<const void*>(ex_reduce_kernel<__half>)
                                          : reinterpret_cast<const void*>(ex_reduce_kernel<float>);
    int dev = 0, sms = 0, per_sm = 0;
    if (emulated > 1) {
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kExThreads, 0);
        ctas = std::max(1, std::min(ctas, sms * per_sm / emulated));
    }
    cudaStream_t st = as_stream(stream);
    Writes wr;
    wr.add(r0.out, size_t(n) * (r0.dtype == SMOE_F16 ? 2 : 4));
    const dim3 grid(ctas, emulated);
    if (emulated == 1) {
        const cudaError_t e = r0.dtype == SMOE_F16
                                  ? launch_pdl(wr, ex_reduce_kernel<__half>, grid, dim3(kExThreads), 0, st, L)
                                  : launch_pdl(wr, ex_reduce_kernel<float>, grid, dim3(kExThreads), 0, st, L);
        if (e != cudaSuccess) return fail(-static_cast<int>(e), std::string("ep_reduce: ") + cudaGetErrorString(e));
        return launch_status("ep_reduce");
    }
    // emulated ranks wait on one another inside one launch: all CTAs must be resident together
    SMOE_REQUIRE(ctas * emulated <= sms * per_sm, SMOE_ESHAPE, "ep_reduce (emulated): more CTAs than fit at once");
    void* args[] = {&L};
    // (launched without the programmatic attribute and never triggering one: the next launch waits for it in full)
    const cudaError_t e = cudaLaunchCooperativeKernel(fn, grid, dim3(kExThreads), args, 0, st);
    if (e != cudaSuccess) return fail(-static_cast<int>(e), std::string("ep_reduce: ") + cudaGetErrorString(e));
    return launch_status("ep_reduce (emulated)");
}

}  // namespace
}  // namespace smoe

using namespace smoe;

extern "C" size_t smoe_ep_exchange_bytes(int64_t ranks, int64_t max_tokens, int64_t d) {
    if (ranks < 1 || ranks > kExMaxRanks || max_tokens < 1 || d < 1) return 0;
    return kExInboxOff + size_t(2) * ranks * max_tokens * d * kExSlot;
}

extern "C" int smoe_ep_exchange_alloc(size_t bytes, void** buffer, void* ipc_handle) {
    SMOE_REQUIRE(buffer && ipc_handle && bytes > kExInboxOff, SMOE_EARG, "ep_exchange_alloc: bad arguments");
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return fail(-static_cast<int>(e), std::string("ep_exchange_alloc: ") + cudaGetErrorString(e));
    e = cudaMemset(p, 0, bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return fail(-static_cast<int>(e), std::string("ep_exchange_alloc: ") + cudaGetErrorString(e));
    }
    std::memcpy(ipc_handle, &h, sizeof(h));
    *buffer = p;
    return SMOE_OK;
}

extern "C" int smoe_ep_exchange_open(const void* ipc_handle, void** peer_buffer) {
    SMOE_REQUIRE(ipc_handle && peer_buffer, SMOE_EARG, "ep_exchange_open: bad arguments");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, ipc_handle, sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return fail(-static_cast<int>(e), std::string("ep_exchange_open: ") + cudaGetErrorString(e));
    *peer_buffer = p;
    return SMOE_OK;
}

extern "C" int smoe_ep_exchange_close(void* peer_buffer) {
    if (!peer_buffer) return SMOE_OK;
    const cudaError_t e = cudaIpcCloseMemHandle(peer_buffer);
    if (e != cudaSuccess) return fail(-static_cast<int>(e), std::string("ep_exchange_close: ") + cudaGetErrorString(e));
    return SMOE_OK;
}

extern "C" int smoe_ep_exchange_free(void* buffer) {
    if (!buffer) return SMOE_OK;
    const cudaError_t e = cudaFree(buffer);
    if (e != cudaSuccess) return fail(-static_cast<int>(e), std::string("ep_exchange_free: ") + cudaGetErrorString(e));
    return SMOE_OK;
}

extern "C" int smoe_ep_exchange_status(void* buffer, int* failed, int clear) {
    SMOE_REQUIRE(buffer && failed, SMOE_EARG, "ep_exchange_status: bad arguments");
    int v = 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(&v, buffer, sizeof(int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && clear) e = cudaMemset(buffer, 0, sizeof(int));
    if (e != cudaSuccess) return fail(-static_cast<int>(e), std::string("ep_exchange_status: ") + cudaGetErrorString(e));
    *failed = v;
    return SMOE_OK;
}

extern "C" int smoe_ep_reduce_combine(const SmoeEpReduce* r, void* stream) {
    SMOE_REQUIRE(r, SMOE_EARG, "ep_reduce: null spec");
    return ex_launch(1, r, stream);
}

extern "C" int smoe_ep_reduce_combine_emulated(int ranks, const SmoeEpReduce* r, void* stream) {
    SMOE_REQUIRE(r && ranks >= 2 && ranks <= kExMaxEmulated, SMOE_EARG, "ep_reduce (emulated): 2 to 8 ranks");
    SMOE_REQUIRE(r[0].ranks == ranks, SMOE_EARG, "ep_reduce (emulated): every rank of the exchange in one launch");
    return ex_launch(ranks, r, stream);
}
