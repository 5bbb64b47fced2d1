// noalloc.cu -- f16acc_gemm_noalloc: the chunked GEMM for callers that cannot
// allocate device memory.
//
// f16acc_gemm needs a caller-provided workspace for its per-tile overflow
// flags.  Some callers have no way to provide one: a plain C or FFI host
// program that links only this library and holds raw pointers but no device
// allocator, or a latency-critical loop that must not call cudaMalloc at all
// (cudaMalloc can synchronise the whole device and can fail when memory is
// tight).  This entry point keeps the flags in a fixed array compiled into
// the library instead, so it allocates nothing.
//
// The array lives in device memory on every GPU that loads the library, until
// the process exits.  All calls on a device share it and it keeps the last
// call's contents; that is harmless here because the main pass writes every
// flag byte of every tile it covers before the redo pass reads it, so nothing
// has to start at zero.  Two calls whose work overlaps on the GPU (different
// streams, or different host threads) race on the array: serialise them, e.g.
// issue them on one stream.
#include <cuda_runtime.h>

#include <cstdint>
#include <atomic>
#include <mutex>

#include "../../include/f16acc.h"

namespace f16acc {
namespace {

// Room for F16ACC_NOALLOC_MAX_TILES output tiles of 128 x 128 at 16 flag
// bytes each (1 MiB per device).
constexpr size_t kNoAllocFlagBytes = size_t(F16ACC_NOALLOC_MAX_TILES) * 16;

// The scratch array.  In host code this name is only a host-side stand-in:
// its device address comes from cudaGetSymbolAddress below, never from
// taking the address of the symbol on the host.
static __device__ __align__(256) uint8_t g_noalloc_flags[kNoAllocFlagBytes];

constexpr int kMaxDevices = 64;

// Device address of g_noalloc_flags, per device; nullptr until resolved.
std::atomic<void*> g_scratch[kMaxDevices];
std::mutex g_scratch_lock;

// The array's device address on `device`, resolved with that device current
// (the caller's device is restored).  A failed lookup is not remembered: the
// next call tries again.
void* scratch_for(int device) {
    void* p = g_scratch[device].load(std::memory_order_acquire);
    if (p != nullptr) return p;
    std::lock_guard<std::mutex> hold(g_scratch_lock);
    p = g_scratch[device].load(std::memory_order_relaxed);
    if (p != nullptr) return p;
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) return nullptr;
    if (prev != device && cudaSetDevice(device) != cudaSuccess) return nullptr;
    void* addr = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&addr, g_noalloc_flags);
    if (prev != device && cudaSetDevice(prev) != cudaSuccess) return nullptr;
    if (err != cudaSuccess) return nullptr;
    g_scratch[device].store(addr, std::memory_order_release);
    return addr;
}

}  // namespace
}  // namespace f16acc

extern "C" int f16acc_gemm_noalloc(const void* A, int64_t sAm, int64_t sAk, const void* B, int64_t sBk, int64_t sBn,
                                   void* C, int64_t sCm, int64_t sCn, int c_dtype, int64_t M, int64_t N, int64_t K,
                                   int chunked, int device, void* stream) {
    int count = 0;
    if (device < 0 || device >= f16acc::kMaxDevices) return F16ACC_ERR_INVALID_ARGUMENT;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device >= count) return F16ACC_ERR_INVALID_ARGUMENT;
    if (M < 0 || N < 0 || K < 0) return F16ACC_ERR_INVALID_ARGUMENT;
    // The flags are only read and written by a chunked product with work to do;
    // every other call is f16acc_gemm without a workspace.
    if (!chunked || M == 0 || N == 0 || K == 0)
        return f16acc_gemm(A, sAm, sAk, B, sBk, sBn, C, sCm, sCn, c_dtype, M, N, K, chunked, nullptr, 0, device,
                           stream);
    // The flags of every 128 x 128 output tile, and no more: handed a workspace
    // that holds only the flags, f16acc_gemm runs without the tail split.
    const size_t need = size_t((M + 127) / 128) * size_t((N + 127) / 128) * 16;
    if (need > f16acc::kNoAllocFlagBytes) return F16ACC_ERR_TOO_LARGE;
    void* flags = f16acc::scratch_for(device);
    if (flags == nullptr) return F16ACC_ERR_CUDA;
    return f16acc_gemm(A, sAm, sAk, B, sBk, sBn, C, sCm, sCn, c_dtype, M, N, K, chunked, flags, need, device,
                       stream);
}
