// trace_probe.cu -- where the time of the chunk-pair hand-off goes.  The pair
// pipeline of the chunked kernel (MMA warp -> 2 pairs of TMEM chunk buffers ->
// epilogue warps), without global operands, with SM-clock timestamps of each
// step recorded by CTA 0 for every pair.  A measurement tool only.
//
// Variants: 0 = the product's hand-off (wait, TMEM load, release, mixed adds);
// 1 = the same without the adds; 2 = the MMA warp alone, issuing pairs
// without waiting for releases (the tensor core's own issue rate); 3 = as 0
// with two MMA threads on different sub-partitions, one per chunk of a pair;
// 4 = as 3, and the epilogue warps of the two issuing sub-partitions start
// their adds only once their sub-partition's MMA thread has issued into the
// buffers they just released (the other two sub-partitions add at once).
#include <cuda_runtime.h>

#include "launch.h"
#include "ptx.cuh"
#include "tc_epilogue.cuh"

namespace f16acc {
namespace {

__device__ __forceinline__ long long sm_clock() {
    long long t;
    asm volatile("mov.u64 %0, %%clock64;" : "=l"(t));
    return t;
}

template <int EPI_SPLIT>
__global__ void __launch_bounds__(64 + 128 * EPI_SPLIT, 1)
    pair_trace_kernel(int npairs, int variant, long long* ev, float* out, int* status) {
    constexpr int BM = 128, BN = 128, CW = BN / EPI_SPLIT, EW = 4 * EPI_SPLIT;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + BM * 64 * 2;
    uint64_t* tfull = reinterpret_cast<uint64_t*>(sB + BN * 64 * 2);
    uint64_t* tempty = tfull + 2;
    uint64_t* done = tempty + 2;
    uint64_t* issued = done + 1;  // [sub-partition 0..1][buffer pair 0..1], variant 4
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(issued + 4);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < (BM + BN) * 64; i += blockDim.x)
        reinterpret_cast<__half*>(smem)[i] = __float2half(0.001f * (i & 63));
    const bool two = variant == 3 || variant == 4;  // one MMA thread per chunk of a pair
    const int issuers = two ? 2 : 1;
    if (threadIdx.x == 0) {
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], issuers);
            mbar_init(&tempty[b], EW);
        }
        mbar_init(done, issuers);
        for (int i = 0; i < 4; ++i) mbar_init(&issued[i], 1);
        *abort_flag = 0;
        fence_mbarrier_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the operand writes, for the tensor core
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const bool rec = blockIdx.x == 0;
    // ev row per pair: [0] MMA warp woke  [1] after fence  [2] first MMA issued  [3] 4th MMA issued
    //                  [4] commit issued  [5] epilogue warp 0 woke  [6] epilogue warp 0 released
    //                  [7] last epilogue warp woke  [8] last epilogue warp released
    if ((warp == 1 || (warp == 0 && two)) && lane == 0) {
        // variant 3: warp 1 issues chunk 0 of every pair, warp 0 chunk 1 (each buffer's two
        // K16 MMAs from one thread, which keeps them in order); otherwise warp 1 issues both.
        constexpr uint32_t idesc = idesc_f16(false, false, BM, BN);
        const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
        const int k_lo = (two && warp == 0) ? 1 : 0;
        const int k_hi = (two && warp == 1) ? 1 : 2;
        const bool stamps = rec && warp == 1;
        uint32_t p = 0, ph = 0;
        for (int c2 = 0; c2 < npairs; ++c2, p ^= 1u) {
            if (variant != 2 && !mbar_wait(&tempty[p], ph ^ 1u, abort_flag, status, kStatusTimeoutProbe)) break;
            long long t[5];
            t[0] = sm_clock();
            tc_fence_after();
            t[1] = sm_clock();
            for (int k = k_lo; k < k_hi; ++k)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    umma_f16(tmem + (2 * p + k) * BN, sdesc_sw128(a0 + h * 32, 16, 1024),
                             sdesc_sw128(b0 + h * 32, 16, 1024), idesc, h);
                    if (k == k_lo && h == 0) t[2] = sm_clock();
                }
            t[3] = sm_clock();
            if (variant == 4) mbar_arrive(&issued[warp * 2 + p]);
            umma_commit(&tfull[p]);
            t[4] = sm_clock();
            if (stamps)
#pragma unroll
                for (int i = 0; i < 5; ++i) ev[int64_t(c2) * 9 + i] = t[i];
            if (p == 1) ph ^= 1u;
        }
        umma_commit(done);
        mbar_wait_drain(done, 0);
    } else if (warp >= 2 && variant != 2) {
        const int e = warp - 2, q = warp & 3, colg = e >> 2;
        const uint32_t base = tmem + (static_cast<uint32_t>(q * 32) << 16) + colg * CW;
        const bool mark = rec && lane == 0 && (e == 0 || e == EW - 1);
        const int col = e == 0 ? 5 : 7;
        float acc[CW];
#pragma unroll
        for (int j = 0; j < CW; ++j) acc[j] = 0.0f;
        uint32_t p = 0, ph = 0;
        for (int c2 = 0; c2 < npairs; ++c2, p ^= 1u) {
            const bool ok = mbar_wait(&tfull[p], ph, abort_flag, status, kStatusTimeoutProbe);
            if (!__all_sync(0xffffffffu, ok)) break;
            if (mark) ev[int64_t(c2) * 9 + col] = sm_clock();
            tc_fence_after();
            uint32_t r0[CW / 2], r1[CW / 2];
            tmem_ld_chunk<CW>(base + (2 * p) * BN, r0);
            tmem_ld_chunk<CW>(base + (2 * p + 1) * BN, r1);
            tmem_wait_ld();
            reg_fence(r0);
            reg_fence(r1);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&tempty[p]);
                if (mark) ev[int64_t(c2) * 9 + col + 1] = sm_clock();
            }
            // variant 4: the issuing sub-partitions wait for the issue of pair
            // c2 + 2 into the buffers just released (issue number c2/2 + 1 there)
            if (variant == 4 && q < 2 && c2 + 2 < npairs) {
                const bool ok2 = mbar_wait(&issued[q * 2 + p], uint32_t((c2 >> 1) + 1) & 1u, abort_flag, status,
                                           kStatusTimeoutProbe);
                if (!__all_sync(0xffffffffu, ok2)) break;
            }
            if (variant == 0 || variant == 3 || variant == 4) {
                add_chunk<CW>(acc, r0);
                add_chunk<CW>(acc, r1);
            }
            if (p == 1) ph ^= 1u;
        }
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < CW; ++j) s += acc[j];
        out[blockIdx.x * blockDim.x + threadIdx.x] = s;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, 512);
}

}  // namespace

cudaError_t launch_pair_trace(int variant, int epi_split, int npairs, int grid, long long* ev, float* out,
                              int* status, cudaStream_t stream) {
    // 200 KB of dynamic smem so one CTA fits per SM (the pipeline takes all 512 TMEM columns)
    constexpr int smem = 200 * 1024;
    if (epi_split == 2) {
        cudaError_t e = cudaFuncSetAttribute(pair_trace_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        pair_trace_kernel<2><<<grid, 64 + 256, smem, stream>>>(npairs, variant, ev, out, status);
    } else {
        cudaError_t e = cudaFuncSetAttribute(pair_trace_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        pair_trace_kernel<4><<<grid, 64 + 512, smem, stream>>>(npairs, variant, ev, out, status);
    }
    return cudaGetLastError();
}

}  // namespace f16acc
