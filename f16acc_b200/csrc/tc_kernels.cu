// tc_kernels.cu -- instantiations and launchers of the tcgen05 GEMM kernel.
#include <mutex>
#include <set>
#include <utility>

#include "launch.h"
#include "tc_gemm.cuh"

namespace f16acc {

namespace {
std::mutex g_attr_mu;
std::set<std::pair<const void*, int>> g_attr_done;
}  // namespace

cudaError_t ensure_smem_attr_raw(const void* kernel, int smem) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(g_attr_mu);
    if (g_attr_done.count({kernel, dev})) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess) g_attr_done.insert({kernel, dev});
    return e;
}

namespace {

template <int BN, int EPI, bool CHUNKED, bool B_MN, int OUT, bool REDO>
cudaError_t launch_one(const TcParams& p, int grid, cudaStream_t stream) {
    using Cfg = TcConfig<BN, EPI, OUT, CHUNKED>;
    auto kernel = tc_gemm_kernel<BN, EPI, CHUNKED, B_MN, OUT, REDO>;
    cudaError_t e = ensure_smem_attr(kernel, Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    return launch_ex(kernel, p, grid, Cfg::THREADS, Cfg::SMEM_BYTES, stream);
}

template <int BN, int EPI, bool B_MN, int OUT>
cudaError_t launch_mode(const TcParams& p, bool chunked, bool redo, int grid, cudaStream_t stream) {
    if (redo) return launch_one<BN, EPI, false, B_MN, OUT, true>(p, grid, stream);
    if (chunked) return launch_one<BN, EPI, true, B_MN, OUT, false>(p, grid, stream);
    return launch_one<BN, EPI, false, B_MN, OUT, false>(p, grid, stream);
}

template <int BN, int EPI>
cudaError_t launch_shape(const TcParams& p, bool chunked, bool b_mn, int out, bool redo, int grid, cudaStream_t stream) {
    if (b_mn) {
        switch (out) {
            case kOutF16: return launch_mode<BN, EPI, true, kOutF16>(p, chunked, redo, grid, stream);
            case kOutF32: return launch_mode<BN, EPI, true, kOutF32>(p, chunked, redo, grid, stream);
            case kOutBF16: return launch_mode<BN, EPI, true, kOutBF16>(p, chunked, redo, grid, stream);
        }
    } else {
        switch (out) {
            case kOutF16: return launch_mode<BN, EPI, false, kOutF16>(p, chunked, redo, grid, stream);
            case kOutF32: return launch_mode<BN, EPI, false, kOutF32>(p, chunked, redo, grid, stream);
            case kOutBF16: return launch_mode<BN, EPI, false, kOutBF16>(p, chunked, redo, grid, stream);
        }
    }
    return cudaErrorInvalidValue;
}

// 128x256 tiles: FP32 mode (no flags, no redo).
cudaError_t launch_wide_fp32(const TcParams& p, bool b_mn, int out, int grid, cudaStream_t stream) {
    if (b_mn) {
        if (out == kOutF16) return launch_one<256, 4, false, true, kOutF16, false>(p, grid, stream);
        if (out == kOutBF16) return launch_one<256, 4, false, true, kOutBF16, false>(p, grid, stream);
        if (out == kOutF32) return launch_one<256, 4, false, true, kOutF32, false>(p, grid, stream);
    } else {
        if (out == kOutF16) return launch_one<256, 4, false, false, kOutF16, false>(p, grid, stream);
        if (out == kOutBF16) return launch_one<256, 4, false, false, kOutBF16, false>(p, grid, stream);
        if (out == kOutF32) return launch_one<256, 4, false, false, kOutF32, false>(p, grid, stream);
    }
    return cudaErrorInvalidValue;
}

// Zero the tail split's per-tile counters ahead of the GEMM, as a programmatic
// dependent launch on both sides: it may start while the previous kernel on
// the stream drains and writes only after that kernel has completed (the
// memory may be that kernel's recycled workspace); the GEMM behind it may
// start its prologue at once and reads the counters only after this kernel
// has completed.  Unlike a memset, it keeps the overlap between products.
__global__ void __launch_bounds__(256) zero_split_counters_kernel(int* cnt, int n) {
    grid_dep_launch();
    grid_dep_wait();
    for (int i = threadIdx.x; i < n; i += blockDim.x) cnt[i] = 0;
}

}  // namespace

cudaError_t launch_zero_split_counters(int* cnt, int n, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, zero_split_counters_kernel, cnt, n);
}

bool tc_shape_supported(TcShape s) { return s.bn == 128 && (s.epi_split == 2 || s.epi_split == 4); }

cudaError_t launch_tc(const TcParams& p, TcShape shape, bool chunked, bool b_mn, int out, bool redo, int grid,
                      cudaStream_t stream) {
    if (shape.bn == 256) {
        if (chunked || redo || shape.epi_split != 4) return cudaErrorInvalidValue;
        return launch_wide_fp32(p, b_mn, out, grid, stream);
    }
    if (shape.bn == 128 && shape.epi_split == 2)
        return launch_shape<128, 2>(p, chunked, b_mn, out, redo, grid, stream);
    if (shape.bn == 128 && shape.epi_split == 4)
        return launch_shape<128, 4>(p, chunked, b_mn, out, redo, grid, stream);
    return cudaErrorInvalidValue;
}

}  // namespace f16acc
