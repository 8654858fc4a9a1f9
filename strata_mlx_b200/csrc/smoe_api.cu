// Library-wide entry points: error messages, version, block table.
#include <map>
#include <mutex>
#include <string>
#include <utility>

#include "blocks.cuh"

namespace smoe {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int set_max_smem(const void* kernel, int bytes) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, int> done;  // (kernel, device) -> bytes already allowed
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    int& cur = done[{kernel, dev}];
    if (bytes <= cur) return 0;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return -static_cast<int>(e);
    cur = bytes;
    return 0;
}

namespace {
struct PdlRecord {
    Writes w;
};
std::mutex g_pdl_mu;
std::map<cudaStream_t, PdlRecord> g_pdl;  // stream -> what its last launch_pdl launch writes
}  // namespace

void pdl_note(cudaStream_t st, const Writes& w) {
    std::lock_guard<std::mutex> lock(g_pdl_mu);
    g_pdl[st].w = w;
}

bool pdl_early(cudaStream_t st, const void* p, size_t n) {
    if (p == nullptr || n == 0) return true;
    std::lock_guard<std::mutex> lock(g_pdl_mu);
    auto it = g_pdl.find(st);
    if (it == g_pdl.end()) return true;
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(p), a1 = a0 + n;
    const Writes& w = it->second.w;
    if (w.all) return false;
    for (int i = 0; i < w.count; ++i) {
        const uintptr_t b0 = reinterpret_cast<uintptr_t>(w.p[i]), b1 = b0 + w.n[i];
        if (a0 < b1 && b0 < a1) return false;
    }
    return true;
}

}  // namespace smoe

using namespace smoe;

extern "C" const char* smoe_last_error(void) { return g_last_error.c_str(); }

extern "C" int smoe_version(void) { return 1; }

extern "C" int smoe_built_arch(void) {
#ifdef SMOE_ARCH
    return SMOE_ARCH;
#else
    return 0;
#endif
}

extern "C" int smoe_block_info(int kind, int* per_block, int* block_bytes) {
    int per = 0, bytes = 0;
    if (!block_info(kind, per, bytes)) return fail(SMOE_EKIND, "block type " + std::to_string(kind) + " has no decoder");
    if (per_block) *per_block = per;
    if (block_bytes) *block_bytes = bytes;
    return SMOE_OK;
}
