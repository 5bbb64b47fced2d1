// skinny_kernels.cu -- instantiations and launches of skinny_gemm_kernel
// (its own translation unit so the template instances build in parallel).
#include <cuda_runtime.h>

#include "launch.h"
#include "skinny_gemm.cuh"

namespace f16acc {
namespace {

template <int MT, bool CHUNKED, bool B_KN, int OUT, bool REDO, bool SHALLOW>
cudaError_t launch_one(const SkinnyParams& p, int tiles_n, int splits, cudaStream_t stream) {
    auto kernel = skinny_gemm_kernel<MT, CHUNKED, B_KN, OUT, REDO, SHALLOW>;
    constexpr int smem = SkinnyCfg::smem_bytes<MT, B_KN, SHALLOW>();
    cudaError_t e = ensure_smem_attr(kernel, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(tiles_n), static_cast<unsigned>(splits), 1);
    cfg.blockDim = dim3(SkinnyCfg::THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = static_cast<unsigned>(splits);
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // the kernel waits before global access
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kernel, p);
}

template <int MT, bool B_KN, int OUT, bool SHALLOW>
cudaError_t launch_depth(const SkinnyParams& p, bool chunked, bool redo, int tiles_n, int splits, cudaStream_t s) {
    if (redo) return launch_one<MT, false, B_KN, OUT, true, SHALLOW>(p, tiles_n, splits, s);
    if (chunked) return launch_one<MT, true, B_KN, OUT, false, SHALLOW>(p, tiles_n, splits, s);
    return launch_one<MT, false, B_KN, OUT, false, SHALLOW>(p, tiles_n, splits, s);
}

// The shallow ring for up to 32 rows and more single-CTA tiles than one wave
// of two CTAs per SM holds (SkinnyCfg::stages; at 64 rows it measured 4.6 %
// slower on the lm_head shape).
template <int MT, bool B_KN, int OUT>
cudaError_t launch_mode(const SkinnyParams& p, bool chunked, bool redo, int tiles_n, int splits, cudaStream_t s) {
    return MT <= 2 && splits == 1 && tiles_n > SkinnyCfg::TARGET_CTAS
               ? launch_depth<MT, B_KN, OUT, true>(p, chunked, redo, tiles_n, splits, s)
               : launch_depth<MT, B_KN, OUT, false>(p, chunked, redo, tiles_n, splits, s);
}

template <int MT, bool B_KN>
cudaError_t launch_out(const SkinnyParams& p, bool chunked, int out, bool redo, int tiles_n, int splits,
                       cudaStream_t s) {
    switch (out) {
        case kOutF16: return launch_mode<MT, B_KN, kOutF16>(p, chunked, redo, tiles_n, splits, s);
        case kOutF32: return launch_mode<MT, B_KN, kOutF32>(p, chunked, redo, tiles_n, splits, s);
        case kOutBF16: return launch_mode<MT, B_KN, kOutBF16>(p, chunked, redo, tiles_n, splits, s);
        default: return cudaErrorInvalidValue;
    }
}

template <int MT>
cudaError_t launch_mt(const SkinnyParams& p, bool chunked, bool b_kn, int out, bool redo, int tiles_n, int splits,
                      cudaStream_t s) {
    return b_kn ? launch_out<MT, true>(p, chunked, out, redo, tiles_n, splits, s)
                : launch_out<MT, false>(p, chunked, out, redo, tiles_n, splits, s);
}

}  // namespace

int skinny_rows(int64_t M) { return M <= 16 ? 16 : (M <= 32 ? 32 : 64); }

void skinny_split(int64_t N, int64_t K, int* splits, int* kper) {
    const int64_t tiles_n = (N + SkinnyCfg::BN - 1) / SkinnyCfg::BN;
    int64_t s = SkinnyCfg::TARGET_CTAS / tiles_n;  // at most one wave of resident CTAs
    s = s < 1 ? 1 : (s > SkinnyCfg::MAX_S ? SkinnyCfg::MAX_S : s);
    const int64_t s_k = K / 128 > 0 ? K / 128 : 1;  // at least 128 of K per CTA
    if (s > s_k) s = s_k;
    int64_t kp = (K + s - 1) / s;
    kp = (kp + SkinnyCfg::BK - 1) / SkinnyCfg::BK * SkinnyCfg::BK;
    *kper = static_cast<int>(kp);
    *splits = static_cast<int>((K + kp - 1) / kp);
}

cudaError_t launch_skinny(const SkinnyParams& p, bool chunked, bool b_kn, int out, bool redo, int splits,
                          cudaStream_t stream) {
    const int tiles_n = (p.N + SkinnyCfg::BN - 1) / SkinnyCfg::BN;
    if (splits < 1 || splits > SkinnyCfg::MAX_S) return cudaErrorInvalidValue;
    switch (skinny_rows(p.M)) {
        case 16: return launch_mt<1>(p, chunked, b_kn, out, redo, tiles_n, splits, stream);
        case 32: return launch_mt<2>(p, chunked, b_kn, out, redo, tiles_n, splits, stream);
        default: return launch_mt<4>(p, chunked, b_kn, out, redo, tiles_n, splits, stream);
    }
}

}  // namespace f16acc
