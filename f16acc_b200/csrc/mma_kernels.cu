// mma_kernels.cu -- instantiations and launchers of the mma.sync GEMM kernel
// and the K == 0 zero fill.
#include "launch.h"
#include "mma_gemm.cuh"

namespace f16acc {

namespace {

template <bool CHUNKED, int A_MODE, int B_MODE, int OUT, bool REDO>
cudaError_t launch_one(const MmaParams& p, int grid, cudaStream_t stream) {
    return launch_ex(mma_gemm_kernel<CHUNKED, A_MODE, B_MODE, OUT, REDO>, p, grid, MmaCfg::THREADS, 0, stream);
}

template <int A_MODE, int B_MODE, int OUT>
cudaError_t launch_mode(const MmaParams& p, bool chunked, bool redo, int grid, cudaStream_t stream) {
    if (redo) return launch_one<false, A_MODE, B_MODE, OUT, true>(p, grid, stream);
    if (chunked) return launch_one<true, A_MODE, B_MODE, OUT, false>(p, grid, stream);
    return launch_one<false, A_MODE, B_MODE, OUT, false>(p, grid, stream);
}

template <int A_MODE, int B_MODE>
cudaError_t launch_out(const MmaParams& p, bool chunked, int out, bool redo, int grid, cudaStream_t stream) {
    switch (out) {
        case kOutF16: return launch_mode<A_MODE, B_MODE, kOutF16>(p, chunked, redo, grid, stream);
        case kOutF32: return launch_mode<A_MODE, B_MODE, kOutF32>(p, chunked, redo, grid, stream);
        case kOutBF16: return launch_mode<A_MODE, B_MODE, kOutBF16>(p, chunked, redo, grid, stream);
    }
    return cudaErrorInvalidValue;
}

template <int A_MODE>
cudaError_t launch_b(const MmaParams& p, bool chunked, int b_mode, int out, bool redo, int grid, cudaStream_t stream) {
    switch (b_mode) {
        case kLoadGeneric: return launch_out<A_MODE, kLoadGeneric>(p, chunked, out, redo, grid, stream);
        case kLoadKVec: return launch_out<A_MODE, kLoadKVec>(p, chunked, out, redo, grid, stream);
        case kLoadNVec: return launch_out<A_MODE, kLoadNVec>(p, chunked, out, redo, grid, stream);
    }
    return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t launch_mma(const MmaParams& p, bool chunked, int a_mode, int b_mode, int out, bool redo, int grid,
                       cudaStream_t stream) {
    if (a_mode == kLoadKVec) return launch_b<kLoadKVec>(p, chunked, b_mode, out, redo, grid, stream);
    if (a_mode == kLoadGeneric) return launch_b<kLoadGeneric>(p, chunked, b_mode, out, redo, grid, stream);
    return cudaErrorInvalidValue;
}

cudaError_t launch_fill_zero(void* C, int64_t sCm, int64_t sCn, int M, int N, int out, cudaStream_t stream,
                             const __half* bias, int64_t sbias) {
    const int64_t total = int64_t(M) * N;
    const int threads = 256;
    const int grid = static_cast<int>(total / threads + 1 < 4096 ? total / threads + 1 : 4096);
    switch (out) {
        case kOutF16: fill_zero_kernel<kOutF16><<<grid, threads, 0, stream>>>(C, sCm, sCn, M, N, bias, sbias); break;
        case kOutF32: fill_zero_kernel<kOutF32><<<grid, threads, 0, stream>>>(C, sCm, sCn, M, N, bias, sbias); break;
        case kOutBF16:
            fill_zero_kernel<kOutBF16><<<grid, threads, 0, stream>>>(C, sCm, sCn, M, N, bias, sbias);
            break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace f16acc
