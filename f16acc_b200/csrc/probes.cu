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

// Probe modes 12-15 re-run modes 2, 4 and a barrier ping-pong with spinning
// (non-suspending) waits: BASE is the behaviour, SPIN the wait style.
// 24-26: ping-pong without tcgen05 fences / with per-thread arrives / both;
// 27: the MMA hand-off (mode 4) with per-thread arrives; 28: MMA issue + one
// commit per chunk with nobody waiting (issue/commit throughput).
template <int MODE>
struct ProbeMode {
    static constexpr int BASE = MODE == 12 ? 2
                                : MODE == 13 || MODE == 27 ? 4
                                : (MODE == 14 || MODE == 15 || MODE == 20 || (MODE >= 24 && MODE <= 26)) ? 14
                                                                                                          : MODE;
    static constexpr bool SPIN = MODE == 12 || MODE == 13 || MODE == 15;
    static constexpr bool NO_FENCE = MODE == 24 || MODE == 26;
    static constexpr bool PER_THREAD = MODE == 25 || MODE == 26 || MODE == 27;
    static constexpr int NBUF = MODE == 20 ? 8 : 4;  // 20: ping-pong with 8 slots (no TMEM involved)
};

template <int MODE, int EPI_SPLIT>
__global__ void __launch_bounds__(64 + 128 * EPI_SPLIT, 1) chunk_rate_kernel(int chunks, float* out, int* status) {
    constexpr int BM = 128, BN = 128, NBUF = ProbeMode<MODE>::NBUF, CW = BN / EPI_SPLIT;
    constexpr int BASE = ProbeMode<MODE>::BASE;
    constexpr bool SPIN = ProbeMode<MODE>::SPIN;
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
            mbar_init(&tempty[b], (ProbeMode<MODE>::PER_THREAD ? 32 : 1) * 4 * EPI_SPLIT);
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

    if (warp == 1 && lane == 0 && MODE >= 8 && MODE <= 11) {
        // latency: one thread issues a dependent group of MMAs, commits and waits, `chunks` times.
        // 8: 2 MMAs N=128 per group; 9: 1 MMA N=128; 10: 2 MMAs N=64; 11: 8 MMAs N=128
        constexpr int NM = MODE == 9 ? 1 : (MODE == 11 ? 8 : 2);
        constexpr int NN = MODE == 10 ? 64 : 128;
        constexpr uint32_t idesc = idesc_f16(false, false, BM, NN);
        uint32_t ph = 0;
        for (int c = 0; c < chunks; ++c) {
#pragma unroll
            for (int h = 0; h < NM; ++h)
                umma_f16(tmem, sdesc_sw128(a0 + (h & 3) * 32, 16, 1024), sdesc_sw128(b0 + (h & 3) * 32, 16, 1024),
                         idesc, h);
            umma_commit(done);
            if (!mbar_wait_drain(done, ph)) break;
            ph ^= 1u;
        }
    } else if (MODE == 23 && warp >= 2) {
        // merged issuer: no MMA warp.  The epilogue warps read chunk c, meet at a
        // named barrier, and one of them issues chunk c+NBUF into the freed buffer.
        const int e = warp - 2, q = warp & 3, colg = e >> 2;
        (void)e;
        constexpr uint32_t idesc = idesc_f16(false, false, BM, BN);
        const bool issuer = warp == 2 && lane == 0;
        auto issue = [&](int b) {
#pragma unroll
            for (int h = 0; h < 2; ++h)
                umma_f16(tmem + b * BN, sdesc_sw128(a0 + h * 32, 16, 1024), sdesc_sw128(b0 + h * 32, 16, 1024), idesc,
                         h);
            umma_commit(&tfull[b]);
        };
        if (issuer)
            for (int b = 0; b < NBUF && b < chunks; ++b) issue(b);
        ChunkRing<NBUF> ring{tfull, tempty, tmem + (static_cast<uint32_t>(q * 32) << 16) + colg * CW, BN};
        float acc[CW];
#pragma unroll
        for (int j = 0; j < CW; ++j) acc[j] = 0.0f;
        for (int c = 0; c < chunks; ++c) {
            if (!ring.wait_full(abort_flag, status)) break;  // every epilogue warp waits on the same phase
            uint32_t r[CW / 2];
            tmem_ld_chunk<CW>(ring.addr(), r);
            tmem_wait_ld();
            reg_fence(r);
            tc_fence_before();
            asm volatile("bar.sync 1, %0;" ::"r"(32 * 4 * EPI_SPLIT) : "memory");
            if (issuer && c + NBUF < chunks) {
                tc_fence_after();
                issue(ring.b);
            }
            add_chunk<CW>(acc, r);
            if (++ring.b == NBUF) { ring.b = 0; ring.phase ^= 1u; }
        }
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < CW; ++j) s += acc[j];
        out[blockIdx.x * blockDim.x + threadIdx.x] = s;
        if (issuer) {
            umma_commit(done);
            mbar_wait_drain(done, 0);
        }
    } else if (warp == 1 && lane == 0 && BASE != 6 && BASE != 7 && MODE != 23) {
        if constexpr (MODE == 28) {
            constexpr uint32_t idesc = idesc_f16(false, false, BM, BN);
            for (int c = 0; c < chunks; ++c) {
#pragma unroll
                for (int h = 0; h < 2; ++h)
                    umma_f16(tmem + (c & 3) * BN, sdesc_sw128(a0 + h * 32, 16, 1024),
                             sdesc_sw128(b0 + h * 32, 16, 1024), idesc, h);
                umma_commit(&tfull[c & 3]);  // nobody waits on these
            }
        } else if constexpr (MODE == 21 || MODE == 22) {
            // MMA only, FP16 accumulator, same flops per chunk as mode 0 with N=64 (4 MMAs) or N=256 (1 MMA)
            constexpr int NN = MODE == 21 ? 64 : 256, NM = MODE == 21 ? 4 : 1;
            constexpr uint32_t idesc = idesc_f16(false, false, BM, NN);
            for (int c = 0; c < chunks; ++c) {
#pragma unroll
                for (int h = 0; h < NM; ++h)
                    umma_f16(tmem, sdesc_sw128(a0 + (h & 1) * 32, 16, 1024), sdesc_sw128(b0 + (h & 1) * 32, 16, 1024),
                             idesc, (c | h) != 0);
            }
        } else if constexpr (BASE == 0 || BASE == 1) {
            constexpr uint32_t idesc = idesc_f16(BASE == 1, false, BM, BN);
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
                const bool ok = SPIN ? mbar_wait_spin(&tempty[b], ph ^ 1u, abort_flag, status, kStatusTimeoutProbe)
                                     : mbar_wait(&tempty[b], ph ^ 1u, abort_flag, status, kStatusTimeoutProbe);
                if (!ok) break;
                if constexpr (BASE == 14) {
                    mbar_arrive(&tfull[b]);  // barrier ping-pong without the tensor core
                } else {
                    tc_fence_after();
#pragma unroll
                    for (int h = 0; h < 2; ++h)
                        umma_f16(tmem + b * BN, sdesc_sw128(a0 + h * 32, 16, 1024),
                                 sdesc_sw128(b0 + h * 32, 16, 1024), idesc, h);
                    umma_commit(&tfull[b]);
                }
                if (++b == NBUF) { b = 0; ph ^= 1u; }
            }
        }
        umma_commit(done);
        mbar_wait_drain(done, 0);
    } else if (BASE >= 2 && warp >= 2) {
        const int e = warp - 2, q = warp & 3, colg = e >> 2;
        ChunkRing<NBUF, SPIN, ProbeMode<MODE>::PER_THREAD, ProbeMode<MODE>::NO_FENCE> ring{
            tfull, tempty, tmem + (static_cast<uint32_t>(q * 32) << 16) + colg * CW, BN};
        float acc[CW];
#pragma unroll
        for (int j = 0; j < CW; ++j) acc[j] = 0.0f;
        if constexpr (BASE == 2) {
            consume_chunks<CW>(acc, chunks, ring, lane, abort_flag, status);
        } else if constexpr (BASE == 3) {
            // TMEM loads and ring hand-off only, no adds
            uint32_t x = 0;
            for (int c = 0; c < chunks; ++c) {
                if (!ring.wait_full(abort_flag, status)) break;
                uint32_t r[CW / 2];
                tmem_ld_chunk<CW>(ring.addr(), r);
                tmem_wait_ld();
                reg_fence(r);
                ring.release(lane);
#pragma unroll
                for (int i = 0; i < CW / 2; ++i) x ^= r[i];
            }
            acc[0] = __uint_as_float(x);
        } else if constexpr (BASE == 4 || BASE == 14) {
            // ring hand-off only: no TMEM loads, no adds
            for (int c = 0; c < chunks; ++c) {
                if (!ring.wait_full(abort_flag, status)) break;
                ring.release(lane);
            }
        } else if constexpr (BASE == 6 || BASE == 7) {
            // no MMA and no hand-off: back-to-back TMEM loads (6), plus the adds (7)
            uint32_t x = 0;
            for (int c = 0; c < chunks; ++c) {
                uint32_t r[CW / 2];
                tmem_ld_chunk<CW>(ring.col_base + (c & (NBUF - 1)) * BN, r);
                tmem_wait_ld();
                reg_fence(r);
                if constexpr (BASE == 7) {
                    add_chunk<CW>(acc, r);
                } else {
#pragma unroll
                    for (int i = 0; i < CW / 2; ++i) x ^= r[i];
                }
            }
            acc[0] += __uint_as_float(x);
        }
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

// Warp-level mma.sync rate (the reference's bench/rate.py and bench/chunkrate.py
// loops on sm_100a): 8 independent m16n8k16 chains per warp on register
// operands (1.0 / 0.0 halves).  30: FP16 accumulate, 31: FP32 accumulate,
// 32: FP16 accumulate converted and added into FP32 every 2 steps (one
// 32-long chunk).  One warp iteration = 8 x 4096 flops.
template <int MODE>
__global__ void __launch_bounds__(256) mma_sync_rate_kernel(int iters, float* out) {
    const uint32_t a = 0x3c00u * (threadIdx.x & 1u);
    float s = 0.0f;
    if constexpr (MODE == 31) {
        float c[8][4] = {};
        for (int i = 0; i < iters; ++i) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
                asm volatile(
                    "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                    "{%0,%1,%2,%3};"
                    : "+f"(c[j][0]), "+f"(c[j][1]), "+f"(c[j][2]), "+f"(c[j][3])
                    : "r"(a), "r"(a), "r"(a), "r"(a), "r"(a), "r"(a));
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) s += c[j][0] + c[j][1] + c[j][2] + c[j][3];
    } else {
        uint32_t h[8][2] = {};
        float t[8][4] = {};
        for (int i = 0; i < iters; ++i) {
            if constexpr (MODE == 32) {
#pragma unroll
                for (int j = 0; j < 8; ++j) h[j][0] = h[j][1] = 0u;
            }
#pragma unroll
            for (int step = 0; step < (MODE == 32 ? 2 : 1); ++step) {
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    asm volatile(
                        "mma.sync.aligned.m16n8k16.row.col.f16.f16.f16.f16 {%0,%1}, {%2,%3,%4,%5}, {%6,%7}, {%0,%1};"
                        : "+r"(h[j][0]), "+r"(h[j][1])
                        : "r"(a), "r"(a), "r"(a), "r"(a), "r"(a), "r"(a));
            }
            if constexpr (MODE == 32) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    add_f16x2_to_f32(t[j][0], t[j][1], h[j][0]);
                    add_f16x2_to_f32(t[j][2], t[j][3], h[j][1]);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) s += t[j][0] + t[j][1] + t[j][2] + t[j][3] + __uint_as_float(h[j][0] ^ h[j][1]);
    }
    out[blockIdx.x * blockDim.x + threadIdx.x] = s;
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
    if (mode >= 30 && mode <= 32) {  // `grid` blocks of 8 warps; out holds grid * 256 floats
        switch (mode) {
            case 30: mma_sync_rate_kernel<30><<<grid, 256, 0, stream>>>(chunks, out); break;
            case 31: mma_sync_rate_kernel<31><<<grid, 256, 0, stream>>>(chunks, out); break;
            case 32: mma_sync_rate_kernel<32><<<grid, 256, 0, stream>>>(chunks, out); break;
        }
        return cudaGetLastError();
    }
    if (mode == 0) return launch_probe<0, 2>(chunks, grid, out, status, stream);
    if (mode == 1) return launch_probe<1, 2>(chunks, grid, out, status, stream);
    if (epi_split == 2) {
        switch (mode) {
            case 2: return launch_probe<2, 2>(chunks, grid, out, status, stream);
            case 3: return launch_probe<3, 2>(chunks, grid, out, status, stream);
            case 4: return launch_probe<4, 2>(chunks, grid, out, status, stream);
            case 6: return launch_probe<6, 2>(chunks, grid, out, status, stream);
            case 7: return launch_probe<7, 2>(chunks, grid, out, status, stream);
            case 8: return launch_probe<8, 2>(chunks, grid, out, status, stream);
            case 9: return launch_probe<9, 2>(chunks, grid, out, status, stream);
            case 10: return launch_probe<10, 2>(chunks, grid, out, status, stream);
            case 11: return launch_probe<11, 2>(chunks, grid, out, status, stream);
            case 12: return launch_probe<12, 2>(chunks, grid, out, status, stream);
            case 13: return launch_probe<13, 2>(chunks, grid, out, status, stream);
            case 14: return launch_probe<14, 2>(chunks, grid, out, status, stream);
            case 15: return launch_probe<15, 2>(chunks, grid, out, status, stream);
            case 20: return launch_probe<20, 2>(chunks, grid, out, status, stream);
            case 21: return launch_probe<21, 2>(chunks, grid, out, status, stream);
            case 22: return launch_probe<22, 2>(chunks, grid, out, status, stream);
            case 23: return launch_probe<23, 2>(chunks, grid, out, status, stream);
            case 24: return launch_probe<24, 2>(chunks, grid, out, status, stream);
            case 25: return launch_probe<25, 2>(chunks, grid, out, status, stream);
            case 26: return launch_probe<26, 2>(chunks, grid, out, status, stream);
            case 27: return launch_probe<27, 2>(chunks, grid, out, status, stream);
            case 28: return launch_probe<28, 2>(chunks, grid, out, status, stream);
        }
    }
    if (epi_split == 4) {
        switch (mode) {
            case 2: return launch_probe<2, 4>(chunks, grid, out, status, stream);
            case 3: return launch_probe<3, 4>(chunks, grid, out, status, stream);
            case 6: return launch_probe<6, 4>(chunks, grid, out, status, stream);
            case 7: return launch_probe<7, 4>(chunks, grid, out, status, stream);
        }
    }
    return cudaErrorInvalidValue;
}

}  // namespace f16acc
