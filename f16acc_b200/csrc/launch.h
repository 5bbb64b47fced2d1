// launch.h -- host-side launch entry points of the kernel translation units
// (one nvcc process per unit so the template instantiations build in parallel).
#pragma once

#include <cuda_runtime.h>

#include "common.cuh"

namespace f16acc {

struct TcParams;
struct MmaParams;

// tcgen05 kernel: BN output columns per tile (128 or 256), EPI_SPLIT column
// slices per TMEM lane quarter.  `redo` selects the FP32 pass over flagged
// tiles (requires chunked == false) launched with programmatic stream
// serialisation.
struct TcShape {
    int bn;
    int epi_split;
};
bool tc_shape_supported(TcShape shape);
cudaError_t launch_tc(const TcParams& p, TcShape shape, bool chunked, bool b_mn, int out, bool redo, int grid,
                      cudaStream_t stream);

// mma.sync kernel: a_mode / b_mode from LoadMode.
cudaError_t launch_mma(const MmaParams& p, bool chunked, int a_mode, int b_mode, int out, bool redo, int grid,
                       cudaStream_t stream);
// Few-row kernel (M <= 64): grid (ceil(N / 128), splits) in clusters of
// `splits` CTAs along K.  skinny_rows: the padded row count (16, 32 or 64)
// for M; skinny_split: the K split of a shape (a function of N and K only, so
// every pass over the same shape adds its partial sums in the same order).
struct SkinnyParams;
int skinny_rows(int64_t M);
void skinny_split(int64_t N, int64_t K, int* splits, int* kper);
cudaError_t launch_skinny(const SkinnyParams& p, bool chunked, bool b_kn, int out, bool redo, int splits,
                          cudaStream_t stream);

// K = 0: C = 0, or C[r][c] = bias[c] when a bias is given.
cudaError_t launch_fill_zero(void* C, int64_t sCm, int64_t sCn, int M, int N, int out, cudaStream_t stream,
                             const __half* bias = nullptr, int64_t sbias = 0);

// Zero the first n tail-split counters ahead of a chunked tcgen05 launch
// (tc_kernels.cu; programmatic dependent launch on both sides).
cudaError_t launch_zero_split_counters(int* cnt, int n, cudaStream_t stream);

// Raw-rate probes (rate_probes.cu): mode 0/1 tcgen05 MMA only with an FP16 /
// FP32 accumulator, mode 2 the chunk-pair pipeline, 30-32 warp-level mma.sync;
// `out` holds grid * (96 + 128 * epi_split) floats (grid * 256 for 30-32).
cudaError_t launch_chunk_rate(int mode, int epi_split, int chunks, int grid, float* out, int* status,
                              cudaStream_t stream);
// Bounded-wait self-test (rate_probes.cu): one CTA whose waits run out after
// limit_ns; out holds 3 values.
cudaError_t launch_wait_selftest(uint64_t limit_ns, unsigned long long* out, int* status, cudaStream_t stream);

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per kernel and device.
cudaError_t ensure_smem_attr_raw(const void* kernel, int smem);
template <typename Kernel>
cudaError_t ensure_smem_attr(Kernel kernel, int smem) {
    return ensure_smem_attr_raw(reinterpret_cast<const void*>(kernel), smem);
}

// Launch helper: cudaLaunchKernelEx with programmatic stream serialisation.
// Every GEMM kernel is launched this way: its CTAs may start their prologue
// while the previous kernel on the stream drains (once that kernel's CTAs have
// all run griddepcontrol.launch_dependents, or exited), and each calls
// griddepcontrol.wait before its first global-memory access, which returns
// when the previous kernel has completed and its writes are visible.  Behind
// a kernel that never triggers, the launch waits for its completion as usual.
template <typename Kernel, typename Params>
cudaError_t launch_ex(Kernel kernel, const Params& p, int grid, int threads, int smem, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
    cfg.blockDim = dim3(static_cast<unsigned>(threads), 1, 1);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, p);
}

}  // namespace f16acc
