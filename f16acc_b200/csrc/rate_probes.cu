// rate_probes.cu -- B200 raw-rate probes, the sm_100a counterparts of the
// reference's bench/rate.py (tensor-core rate with an FP32 against an FP16
// accumulator) and bench/chunkrate.py (the rate once every 32-long chunk is
// converted and added in FP32): steppergg/f16acc bench/rate.py:7-43 and
// bench/chunkrate.py:7-43.  Also the bounded-wait self-test.
//
// tcgen05 probes: one CTA per SM (200 KB of shared memory requested, so a
// second CTA never shares the SM's TMEM), operands a fixed 128 x 64 tile of A
// and of B in shared memory, no global traffic:
//   mode 0  128x128x16 kind::f16 MMAs back to back, FP16 accumulator
//   mode 1  the same with an FP32 accumulator
//   mode 2  the chunked GEMM's pipeline without operand loads: two MMA warps
//           hand chunk pairs over through two TMEM pairs (4 chunk buffers),
//           the epilogue warps consume them with the GEMM's own
//           consume_chunk_pairs (TMEM load, named-barrier release, one mixed
//           FP32 add per element)
// Work per CTA: `chunks` x 2 x 128 x 128 x 32 flops.
//
// Warp-level mma.sync probes (`grid` blocks of 8 warps, `chunks` iterations
// of 8 independent m16n8k16 products per warp, operands held in registers):
//   mode 30  FP16 accumulate          8 x 4096 flops per warp iteration
//   mode 31  FP32 accumulate          8 x 4096
//   mode 32  two K16 steps into FP16, the chunk added into FP32 registers
//                                     8 x 8192
#include <cuda_runtime.h>

#include <cstdint>

#include "launch.h"
#include "tc_epilogue.cuh"

namespace f16acc {
namespace {

constexpr int kProbeTileBytes = 128 * 64 * 2;  // one 128 x 64 FP16 tile, 128-byte swizzled rows
constexpr int kProbeSmem = 200 * 1024;

struct ProbeCtrl {
    uint64_t tfull[2];
    uint64_t done[2];  // one per MMA-issuing warp: its MMAs have completed
    uint32_t tmem_slot;
    int abort_flag;
};

template <int MODE, int EPI_SPLIT>
__global__ void __launch_bounds__(96 + 128 * EPI_SPLIT, 1) tc_rate_kernel(int chunks, float* out, int* status) {
    constexpr int BN = 128, CW = BN / EPI_SPLIT, EPI_WARPS = 4 * EPI_SPLIT, FIRST_EPI = 3;
    constexpr int NB = 32 * (1 + EPI_WARPS);  // one MMA warp + the epilogue warps per release round
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    auto* ctrl = reinterpret_cast<ProbeCtrl*>(smem + 2 * kProbeTileBytes);
    volatile int* abort_flag = &ctrl->abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // Operands: every FP16 element 0.125 or 0, so products and FP16 chunk sums
    // stay small and finite.
    for (int i = threadIdx.x; i < 2 * kProbeTileBytes / 4; i += blockDim.x)
        reinterpret_cast<uint32_t*>(smem)[i] = (i % 3 == 0) ? 0x30003000u : 0x00003000u;
    fence_proxy_async_smem();  // generic-proxy writes, read by the tensor core
    if (threadIdx.x == 0) {
        mbar_init(&ctrl->tfull[0], 1);
        mbar_init(&ctrl->tfull[1], 1);
        mbar_init(&ctrl->done[0], 1);
        mbar_init(&ctrl->done[1], 1);
        ctrl->abort_flag = 0;
        fence_mbarrier_init();
    }
    if (warp == 0) {
        tmem_alloc(&ctrl->tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctrl->tmem_slot;
    const uint32_t a0 = smem_u32(smem), b0 = a0 + kProbeTileBytes;
    auto adesc = [&](int ks) { return sdesc_sw128(a0 + ks * 32, 16, 1024); };
    auto bdesc = [&](int ks) { return sdesc_sw128(b0 + ks * 32, 16, 1024); };

    if constexpr (MODE == 0 || MODE == 1) {
        if (warp == 1 && lane == 0) {
            constexpr uint32_t idesc = idesc_f16(MODE == 1, false, 128, BN);
            for (int c = 0; c < chunks; ++c) {
                const uint32_t d = tmem + (c & 3) * BN;
#pragma unroll
                for (int h = 0; h < 2; ++h) umma_f16(d, adesc(2 * (c & 1) + h), bdesc(2 * (c & 1) + h), idesc, h);
            }
            umma_commit(&ctrl->done[0]);
            mbar_wait_drain(&ctrl->done[0], 0);
        }
    } else if (warp == 1 || warp == 2) {
        // MMA warp 1 + b issues hand-offs b, b + 2, ... into pair b and reclaims the
        // pair with bar.sync before issuing into it again (the GEMM's protocol).
        const uint32_t mine = uint32_t(warp - 1);
        constexpr uint32_t idesc = idesc_f16(false, false, 128, BN);
        auto aborted = [&]() { return __any_sync(0xffffffffu, *abort_flag != 0); };
        bool pending = false, stopped = false;
        for (int c = 2 * int(mine); c < chunks; c += 4) {
            if (aborted()) { stopped = true; break; }
            if (pending) {
                named_bar_sync(kPairBarrier + int(mine), NB);
                pending = false;
                if (aborted()) { stopped = true; break; }
            }
            tc_fence_after();
            if (lane == 0) {
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
                    if (c + cc >= chunks) break;
#pragma unroll
                    for (int h = 0; h < 2; ++h)
                        umma_f16(tmem + (2 * mine + cc) * BN, adesc(2 * cc + h), bdesc(2 * cc + h), idesc, h);
                }
                umma_commit(&ctrl->tfull[mine]);
            }
            __syncwarp();
            pending = true;
        }
        if (pending && !stopped && !aborted()) named_bar_sync(kPairBarrier + int(mine), NB);
        if (lane == 0) {
            umma_commit(&ctrl->done[mine]);
            mbar_wait_drain(&ctrl->done[mine], 0);
        }
        __syncwarp();
    } else if (warp >= FIRST_EPI && warp < FIRST_EPI + EPI_WARPS) {
        const int e = warp - FIRST_EPI, q = warp & 3, colg = e >> 2;
        PairRing<CW> pairs{ctrl->tfull, NB, tmem + (uint32_t(q * 32) << 16) + colg * CW, BN};
        float acc[CW];
#pragma unroll
        for (int j = 0; j < CW; ++j) acc[j] = 0.0f;
        if (!consume_chunk_pairs<CW>(acc, chunks, pairs, abort_flag, status)) {
            *abort_flag = 1;
            __threadfence_block();
            __syncwarp();
            pairs.release_issued_on_exit(lane);
        }
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < CW; ++j) s += acc[j];
        out[blockIdx.x * blockDim.x + threadIdx.x] = s;  // keeps the adds live
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, 512);
}

__device__ __forceinline__ void mma16816_f16(uint32_t (&d)[2], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f16.f16.f16.f16 {%0,%1}, {%2,%3,%4,%5}, {%6,%7}, {%0,%1};"
                 : "+r"(d[0]), "+r"(d[1])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
__device__ __forceinline__ void mma16816_f32(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
__device__ __forceinline__ float sum_f16x2(uint32_t v) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&v));
    return f.x + f.y;
}

template <int MODE>
__global__ void __launch_bounds__(256) mma_sync_rate_kernel(int iters, float* out) {
    constexpr int CHAINS = 8;
    // Fragments: lane-dependent powers of two (0.25 or 0 in A, 0.5 or 0 in B),
    // so every product is exact and FP16 sums never overflow however long the
    // run: an FP16 accumulator stops growing once the increment is below half
    // an ulp.
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t ah = (lane % 5u == 0u) ? 0x34003400u : 0x00003400u;  // {0.25, 0.25} / {0.25, 0}
    const uint32_t bh = (lane % 3u == 0u) ? 0x38000000u : 0x00003800u;  // {0, 0.5} / {0.5, 0}
    const uint32_t a[4] = {ah, 0u, 0u, ah};
    const uint32_t b[2] = {bh, 0u};
    float s = 0.0f;
    if constexpr (MODE == 31) {
        float d[CHAINS][4] = {};
        for (int i = 0; i < iters; ++i)
#pragma unroll
            for (int j = 0; j < CHAINS; ++j) mma16816_f32(d[j], a, b);
#pragma unroll
        for (int j = 0; j < CHAINS; ++j) s += (d[j][0] + d[j][1]) + (d[j][2] + d[j][3]);
    } else if constexpr (MODE == 30) {
        uint32_t d[CHAINS][2] = {};
        for (int i = 0; i < iters; ++i)
#pragma unroll
            for (int j = 0; j < CHAINS; ++j) mma16816_f16(d[j], a, b);
#pragma unroll
        for (int j = 0; j < CHAINS; ++j) s += sum_f16x2(d[j][0]) + sum_f16x2(d[j][1]);
    } else {
        float t[CHAINS][4] = {};
        for (int i = 0; i < iters; ++i) {
#pragma unroll
            for (int j = 0; j < CHAINS; ++j) {
                uint32_t h[2] = {0u, 0u};  // a fresh FP16 accumulator for each 32-long chunk
                mma16816_f16(h, a, b);
                mma16816_f16(h, a, b);
                add_f16x2_to_f32(t[j][0], t[j][1], h[0]);
                add_f16x2_to_f32(t[j][2], t[j][3], h[1]);
            }
        }
#pragma unroll
        for (int j = 0; j < CHAINS; ++j) s += (t[j][0] + t[j][1]) + (t[j][2] + t[j][3]);
    }
    out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}

template <int MODE, int EPI>
cudaError_t launch_tc_probe(int chunks, int grid, float* out, int* status, cudaStream_t stream) {
    auto kernel = tc_rate_kernel<MODE, EPI>;
    const cudaError_t e = ensure_smem_attr(kernel, kProbeSmem);
    if (e != cudaSuccess) return e;
    kernel<<<grid, 96 + 128 * EPI, kProbeSmem, stream>>>(chunks, out, status);
    return cudaGetLastError();
}

// Bounded-wait self-test: the give-up path of the product kernels' waits
// (mbar_wait), made to run out on purpose.  One CTA of 3 warps and an
// mbarrier that nothing ever arrives on.  Thread 0 waits with a limit of
// limit_ns; when it gives up it records kStatusTimeoutProbe in the status
// word and raises the CTA's abort flag.  Warps 1 and 2 wait with the products'
// limit and must leave as soon as they see the flag.  out[0] = nanoseconds
// thread 0 waited, out[1] = threads of warps 1-2 that left without the
// barrier completing, out[2] = 1 if thread 0's wait reported success.  No
// thread ever waits past kWaitLimitNs, so the kernel always ends.
__global__ void __launch_bounds__(96) wait_selftest_kernel(uint64_t limit_ns, unsigned long long* out, int* status) {
    __shared__ uint64_t never;
    __shared__ int abort_flag;
    __shared__ int left;
    if (threadIdx.x == 0) {
        mbar_init(&never, 1);
        abort_flag = 0;
        left = 0;
        fence_mbarrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint64_t t0 = globaltimer_ns();
        const bool ok = mbar_wait(&never, 0, &abort_flag, status, kStatusTimeoutProbe, limit_ns);
        out[0] = globaltimer_ns() - t0;
        out[2] = ok ? 1ull : 0ull;
    } else if (threadIdx.x >= 32) {
        if (!mbar_wait(&never, 0, &abort_flag, status, kStatusTimeoutProbe)) atomicAdd(&left, 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) out[1] = static_cast<unsigned long long>(left);
}

}  // namespace

cudaError_t launch_chunk_rate(int mode, int epi_split, int chunks, int grid, float* out, int* status,
                              cudaStream_t stream) {
    switch (mode) {
        case 0: return launch_tc_probe<0, 2>(chunks, grid, out, status, stream);
        case 1: return launch_tc_probe<1, 2>(chunks, grid, out, status, stream);
        case 2:
            return epi_split == 4 ? launch_tc_probe<2, 4>(chunks, grid, out, status, stream)
                                  : launch_tc_probe<2, 2>(chunks, grid, out, status, stream);
        case 30: mma_sync_rate_kernel<30><<<grid, 256, 0, stream>>>(chunks, out); break;
        case 31: mma_sync_rate_kernel<31><<<grid, 256, 0, stream>>>(chunks, out); break;
        case 32: mma_sync_rate_kernel<32><<<grid, 256, 0, stream>>>(chunks, out); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_wait_selftest(uint64_t limit_ns, unsigned long long* out, int* status, cudaStream_t stream) {
    wait_selftest_kernel<<<1, 96, 0, stream>>>(limit_ns, out, status);
    return cudaGetLastError();
}

}  // namespace f16acc
