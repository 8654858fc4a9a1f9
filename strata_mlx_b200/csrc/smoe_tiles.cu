// The dispatch permutation of a prompt's (token, expert) pairs into tiles of 16 slots, each tile one
// expert's (strata_mlx/blocks.py:657-681 `tiles_of`), computed on the GPU without a host sync.
//
// Two launches over chunks of 1024 pairs. The first ranks every pair among the pairs of its expert earlier
// in its chunk (warp match + per-warp histograms in shared memory, so the ranks follow the flat index and
// the result is deterministic) and writes the chunk's histogram; it also clears `token`. The second gives
// each expert its tiles (a scan of ceil(count / 16) over experts) and each pair its slot:
// slot = 16 * first_tile[e] + (pairs of e in earlier chunks) + rank in chunk.
#include <mutex>

#include "common.cuh"

namespace smoe {

constexpr int kTsChunk = 1024;
constexpr int kTsWarps = kTsChunk / 32;
constexpr int kTile = 16;
constexpr int kTsMaxExperts = 1024;

__global__ void __launch_bounds__(kTsChunk) tiles_rank_kernel(const int32_t* __restrict__ indices, int64_t pairs,
                                                             int experts, int32_t* __restrict__ hist,
                                                             int32_t* __restrict__ rank, uint32_t* __restrict__ token,
                                                             int64_t token_len) {
    extern __shared__ int32_t wh[];  // [kTsWarps][experts] counts, then exclusive prefixes over warps
    const int c = blockIdx.x, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < kTsWarps * experts; i += kTsChunk) wh[i] = 0;
    for (int64_t i = int64_t(blockIdx.x) * kTsChunk + threadIdx.x; i < token_len; i += int64_t(gridDim.x) * kTsChunk)
        token[i] = 0;
    __syncthreads();
    const int64_t p = int64_t(c) * kTsChunk + threadIdx.x;
    int e = p < pairs ? indices[p] : -1;
    if (e >= experts) e = -1;  // names no expert: not placed
    const unsigned same = __match_any_sync(0xffffffffu, e);
    const int in_warp = __popc(same & ((1u << lane) - 1u));
    if (e >= 0 && in_warp == 0) wh[w * experts + e] = __popc(same);
    __syncthreads();
    for (int x = threadIdx.x; x < experts; x += kTsChunk) {
        int run = 0;
        for (int v = 0; v < kTsWarps; ++v) {
            const int n = wh[v * experts + x];
            wh[v * experts + x] = run;
            run += n;
        }
        hist[int64_t(c) * experts + x] = run;
    }
    __syncthreads();
    if (p < pairs) rank[p] = e >= 0 ? wh[w * experts + e] + in_warp : -1;
}

__global__ void __launch_bounds__(kTsChunk) tiles_place_kernel(const int32_t* __restrict__ indices, int64_t pairs,
                                                              int k, int experts, const int32_t* __restrict__ hist,
                                                              const int32_t* __restrict__ rank, int64_t most,
                                                              uint32_t* __restrict__ tile_expert,
                                                              uint32_t* __restrict__ token, uint32_t* __restrict__ where) {
    __shared__ int32_t before[kTsMaxExperts];   // pairs of expert e in chunks before this one
    __shared__ int32_t tile_end[kTsMaxExperts];  // inclusive scan of tiles over experts
    __shared__ int32_t warp_tot[kTsWarps];
    const int c = blockIdx.x, chunks = gridDim.x;
    // per expert: its count in earlier chunks, its total, its tiles
    const int x = threadIdx.x;  // experts <= kTsMaxExperts == kTsChunk: one expert a thread
    int tiles = 0;
    if (x < experts) {
        int b = 0, total = 0;
        for (int cc = 0; cc < chunks; ++cc) {
            const int n = hist[int64_t(cc) * experts + x];
            if (cc < c) b += n;
            total += n;
        }
        before[x] = b;
        tiles = (total + kTile - 1) / kTile;
    }
    // inclusive scan of tiles over the experts: warp scans, then the warps' totals
    int v = tiles;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
    }
    if (lane == 31) warp_tot[w] = v;
    __syncthreads();
    if (w == 0) {
        int t = warp_tot[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += u;
        }
        warp_tot[lane] = t;  // inclusive over warps
    }
    __syncthreads();
    const int incl = v + (w > 0 ? warp_tot[w - 1] : 0);
    if (x < experts) tile_end[x] = incl;
    __syncthreads();

    // every pair of this chunk to its slot
    const int64_t p = int64_t(c) * kTsChunk + threadIdx.x;
    if (p < pairs) {
        const int e = indices[p];
        const int r = rank[p];
        if (e >= 0 && e < experts && r >= 0) {
            const int64_t first = e > 0 ? tile_end[e - 1] : 0;
            const int64_t slot = first * kTile + before[e] + r;
            where[p] = static_cast<uint32_t>(slot);
            token[slot] = static_cast<uint32_t>(p / k);
        } else {
            where[p] = 0xffffffffu;
        }
    }
    // the expert of every tile: the number of experts whose tiles end at or before it (upper bound search)
    for (int64_t t = int64_t(c) * kTsChunk + threadIdx.x; t < most; t += int64_t(chunks) * kTsChunk) {
        int lo = 0, hi = experts;  // first expert with tile_end > t
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (tile_end[mid] <= t) lo = mid + 1; else hi = mid;
        }
        tile_expert[t] = static_cast<uint32_t>(lo);
    }
}

}  // namespace smoe

using namespace smoe;

extern "C" size_t smoe_tiles_of_workspace_size(int64_t pairs, int64_t experts) {
    const int64_t chunks = (pairs + kTsChunk - 1) / kTsChunk;
    return static_cast<size_t>((chunks * experts + pairs) * 4 + 256);
}

extern "C" int smoe_tiles_of(const int32_t* indices, int64_t pairs, int64_t k, int64_t experts, uint32_t* tile_expert,
                             uint32_t* token, uint32_t* where, void* workspace, size_t workspace_bytes, void* stream) {
    if (pairs == 0) return SMOE_OK;
    SMOE_REQUIRE(indices && tile_expert && token && where && pairs > 0 && k > 0, SMOE_EARG, "null pointer or no pairs");
    SMOE_REQUIRE(experts > 0 && experts <= kTsMaxExperts, SMOE_ESHAPE, "tiles_of takes 1 to 1024 experts");
    SMOE_REQUIRE(pairs % k == 0, SMOE_EARG, "pairs must be a multiple of k");
    SMOE_REQUIRE(workspace && workspace_bytes >= smoe_tiles_of_workspace_size(pairs, experts), SMOE_EWORKSPACE,
                 "tiles_of workspace too small");
    const int64_t chunks = (pairs + kTsChunk - 1) / kTsChunk;
    SMOE_REQUIRE(chunks <= 65535, SMOE_ESHAPE, "too many pairs for one tiles_of call");
    const int64_t most = pairs / kTile + std::min(experts, pairs);
    int32_t* hist = static_cast<int32_t*>(workspace);
    int32_t* rank = hist + chunks * experts;
    cudaStream_t st = as_stream(stream);
    const size_t smem = size_t(kTsWarps) * experts * 4;
    if (int s = max_smem(tiles_rank_kernel, static_cast<int>(smem))) return fail(s, "tiles_of: shared memory limit");
    tiles_rank_kernel<<<static_cast<unsigned>(chunks), kTsChunk, smem, st>>>(indices, pairs, static_cast<int>(experts),
                                                                             hist, rank, token, most * kTile);
    if (int s = launch_status("tiles_of rank")) return s;
    tiles_place_kernel<<<static_cast<unsigned>(chunks), kTsChunk, 0, st>>>(indices, pairs, static_cast<int>(k),
                                                                           static_cast<int>(experts), hist, rank, most,
                                                                           tile_expert, token, where);
    return launch_status("tiles_of place");
}

// ---------------------------------------------------------------- the same permutation without a workspace
//
// Some callers cannot allocate device memory where they call this library: a host framework that owns every
// device allocation and hands a plugin only its input and output buffers, or a serving loop that must not call
// cudaMalloc because it can synchronize the whole device. For them smoe_tiles_of_noalloc runs the two kernels
// above with their scratch (per-chunk histograms and per-pair ranks) in this fixed array instead of a caller's
// workspace. The array is part of the library's device image: every GPU that loads the library holds its
// 1 MiB (+ 256 bytes) until the process exits. All calls share it and it keeps what the last call left; nothing in it needs
// to start at zero (each call writes every histogram entry and rank it later reads), but calls that overlap
// on the GPU (on different streams, or from different host threads) race on it.

namespace smoe {

constexpr size_t kNoAllocScratchBytes = (size_t(1) << 20) + 256;  // 1 MiB of ranks and histograms, + alignment
static __device__ __align__(256) uint8_t g_tiles_scratch[kNoAllocScratchBytes];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

// The device address of g_tiles_scratch on the current device. In host code the array's name is only a
// host-side handle, not a device address, so it is looked up once per device with cudaGetSymbolAddress and kept
// for the life of the process: a device reset (cudaDeviceReset, or the primary context torn down and made again)
// leaves the kept address stale, so a process that resets a device must not call smoe_tiles_of_noalloc on it
// afterwards.
int scratch_on_current_device(void** addr) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(-static_cast<int>(e), std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return fail(SMOE_EARG, "device index beyond the no-alloc table");
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (g_scratch_addr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_tiles_scratch);
        if (e != cudaSuccess)
            return fail(-static_cast<int>(e), std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
        g_scratch_addr[dev] = p;
    }
    *addr = g_scratch_addr[dev];
    return SMOE_OK;
}

}  // namespace

}  // namespace smoe

extern "C" int smoe_tiles_of_noalloc(const int32_t* indices, int64_t pairs, int64_t k, int64_t experts,
                                     uint32_t* tile_expert, uint32_t* token, uint32_t* where, void* stream) {
    using namespace smoe;
    if (pairs == 0) return SMOE_OK;
    SMOE_REQUIRE(indices && tile_expert && token && where && pairs > 0 && k > 0, SMOE_EARG, "null pointer or no pairs");
    SMOE_REQUIRE(experts > 0 && experts <= kTsMaxExperts, SMOE_ESHAPE, "tiles_of takes 1 to 1024 experts");
    SMOE_REQUIRE(pairs % k == 0, SMOE_EARG, "pairs must be a multiple of k");
    const size_t need = smoe_tiles_of_workspace_size(pairs, experts);
    SMOE_REQUIRE(need <= kNoAllocScratchBytes, SMOE_ESHAPE,
                 std::to_string(pairs) + " pairs over " + std::to_string(experts) + " experts need " +
                     std::to_string(need) + " bytes of scratch, more than the " +
                     std::to_string(kNoAllocScratchBytes) + " bytes of smoe_tiles_of_noalloc's fixed array; "
                     "split the pairs or call smoe_tiles_of with a workspace");
    void* scratch = nullptr;
    if (int s = scratch_on_current_device(&scratch)) return s;
    const int64_t chunks = (pairs + kTsChunk - 1) / kTsChunk;
    const int64_t most = pairs / kTile + std::min(experts, pairs);
    int32_t* hist = static_cast<int32_t*>(scratch);
    int32_t* rank = hist + chunks * experts;
    cudaStream_t st = as_stream(stream);
    const size_t smem = size_t(kTsWarps) * experts * 4;
    if (int s = max_smem(tiles_rank_kernel, static_cast<int>(smem))) return fail(s, "tiles_of: shared memory limit");
    tiles_rank_kernel<<<static_cast<unsigned>(chunks), kTsChunk, smem, st>>>(indices, pairs, static_cast<int>(experts),
                                                                             hist, rank, token, most * kTile);
    if (int s = launch_status("tiles_of_noalloc rank")) return s;
    tiles_place_kernel<<<static_cast<unsigned>(chunks), kTsChunk, 0, st>>>(indices, pairs, static_cast<int>(k),
                                                                           static_cast<int>(experts), hist, rank, most,
                                                                           tile_expert, token, where);
    return launch_status("tiles_of_noalloc place");
}
