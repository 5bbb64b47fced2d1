// probes.cu -- B200 raw-rate probes, the sm_100a analogue of the reference's
// bench/rate.py (raw tensor rate, FP32 vs FP16 accumulate) and
// bench/chunkrate.py (the ceiling once every 32-long chunk is converted and
// added in FP32), steppergg/f16acc bench/rate.py:7-43, bench/chunkrate.py:7-43.
//
// One CTA per SM, operands a fixed shared-memory tile (no global traffic):
//   mode 0  tcgen05.mma kind::f16 128x128x16 back to back, FP16 accumulator
//   mode 1  the same with an FP32 accumulator
//   mode 2  the chunk pipeline of the GEMM kernel: two MMAs per 32-long chunk
//           into a 4-deep TMEM ring, epilogue warps running the kernel's own
//           consume_chunks() (TMEM load + one mixed-precision add per element)
#include <cuda_runtime.h>

#include "../../include/f16acc.h"
#include "launch.h"
#include "tc_epilogue.cuh"

namespace f16acc {

template <int MODE, int EPI_SPLIT>
__global__ void __launch_bounds__(64 + 128 * EPI_SPLIT, 1) chunk_rate_kernel(int chunks, float* out, int* status) {
    constexpr int BM = 128, BN = 128, NBUF = 4, CW = BN / EPI_SPLIT;
    constexpr int TILE_BYTES = BM * 64 * 2;  // one 128 x 64 f16 tile, 128-byte swizzle rows
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + TILE_BYTES;
    uint64_t* tfull = reinterpret_cast<uint64_t*>(smem + 2 * TILE_BYTES);
    uint64_t* tempty = tfull + NBUF;
    uint64_t* done = tempty + NBUF;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // operands: halves 1.0 / 0.0 alternating, so chunk sums stay small and finite
    for (int i = threadIdx.x; i < 2 * TILE_BYTES / 4; i += blockDim.x)
        reinterpret_cast<uint32_t*>(smem)[i] = 0x00003c00u;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic-proxy writes -> tensor-core reads
    if (threadIdx.x == 0) {
        for (int b = 0; b < NBUF; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4 * EPI_SPLIT);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);

    if (warp == 1 && lane == 0) {
        if constexpr (MODE == 0 || MODE == 1) {
            constexpr uint32_t idesc = idesc_f16(MODE == 1, false, BM, BN);
            for (int c = 0; c < chunks; ++c) {
#pragma unroll
                for (int h = 0; h < 2; ++h)
                    umma_f16(tmem, sdesc_sw128(a0 + h * 32, 16, 1024), sdesc_sw128(b0 + h * 32, 16, 1024), idesc,
                             (c | h) != 0);
            }
        } else {
            constexpr uint32_t idesc = idesc_f16(false, false, BM, BN);
            uint32_t b = 0, ph = 0;
            for (int c = 0; c < chunks; ++c) {
                if (!mbar_wait(&tempty[b], ph ^ 1u, abort_flag, status, kStatusTimeoutProbe)) break;
                tc_fence_after();
#pragma unroll
                for (int h = 0; h < 2; ++h)
                    umma_f16(tmem + b * BN, sdesc_sw128(a0 + h * 32, 16, 1024), sdesc_sw128(b0 + h * 32, 16, 1024),
                             idesc, h);
                umma_commit(&tfull[b]);
                if (++b == NBUF) { b = 0; ph ^= 1u; }
            }
        }
        umma_commit(done);
        mbar_wait_drain(done, 0);
    } else if (MODE == 2 && warp >= 2) {
        const int e = warp - 2, q = warp & 3, colg = e >> 2;
        ChunkRing<NBUF> ring{tfull, tempty, tmem + (static_cast<uint32_t>(q * 32) << 16) + colg * CW, BN};
        float acc[CW];
#pragma unroll
        for (int j = 0; j < CW; ++j) acc[j] = 0.0f;
        consume_chunks<CW, NBUF>(acc, chunks, ring, lane, abort_flag, status);
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < CW; ++j) s += acc[j];
        out[blockIdx.x * blockDim.x + threadIdx.x] = s;  // keeps the adds live
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 512);
}

namespace {
template <int MODE, int EPI>
cudaError_t launch_probe(int chunks, int grid, float* out, int* status, cudaStream_t stream) {
    constexpr int smem = 2 * 128 * 64 * 2 + 1024 + 256;
    auto kernel = chunk_rate_kernel<MODE, EPI>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    // 200 KB requested so only one CTA fits per SM (the TMEM ring takes all 512 columns)
    (void)smem;
    kernel<<<grid, 64 + 128 * EPI, 200 * 1024, stream>>>(chunks, out, status);
    return cudaGetLastError();
}
}  // namespace

cudaError_t launch_chunk_rate(int mode, int epi_split, int chunks, int grid, float* out, int* status,
                              cudaStream_t stream) {
    if (mode == 0) return launch_probe<0, 2>(chunks, grid, out, status, stream);
    if (mode == 1) return launch_probe<1, 2>(chunks, grid, out, status, stream);
    if (mode == 2 && epi_split == 2) return launch_probe<2, 2>(chunks, grid, out, status, stream);
    if (mode == 2 && epi_split == 4) return launch_probe<2, 4>(chunks, grid, out, status, stream);
    return cudaErrorInvalidValue;
}

}  // namespace f16acc
