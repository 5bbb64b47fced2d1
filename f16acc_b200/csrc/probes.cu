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

// Shared-memory flag signalling for probe modes 54 (release/acquire at CTA scope).
__device__ __forceinline__ uint32_t ld_acquire_smem(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_smem(uint32_t* p, uint32_t v) {
    asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_add_smem(uint32_t* p, uint32_t v) {
    asm volatile("red.release.cta.shared::cta.add.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}
// Spin until *p >= target; bounded by kWaitLimitNs (clock read every 1024 polls).
__device__ __forceinline__ bool spin_ge(const uint32_t* p, uint32_t target, int* status) {
    uint64_t t0 = 0;
    for (uint32_t i = 1;; ++i) {
        if (ld_acquire_smem(p) >= target) return true;
        if ((i & 1023u) == 0u) {
            const uint64_t now = globaltimer_ns();
            if (t0 == 0) {
                t0 = now;
            } else if (now - t0 > kWaitLimitNs) {
                atomicCAS(status, 0, kStatusTimeoutProbe);
                return false;
            }
        }
    }
}
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
    uint32_t* flag_go = tmem_slot + 4;    // mode 54: issuer -> epilogue warps
    uint32_t* flag_back = tmem_slot + 8;  // mode 54: epilogue warps -> issuer (a count)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // operands: halves 1.0 / 0.0 alternating, so chunk sums stay small and finite
    for (int i = threadIdx.x; i < 2 * TILE_BYTES / 4; i += blockDim.x)
        reinterpret_cast<uint32_t*>(smem)[i] = 0x00003c00u;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic-proxy writes -> tensor-core reads
    if (threadIdx.x == 0) {
        for (int b = 0; b < NBUF; ++b) {
            mbar_init(&tfull[b], 1);
            // mode 41: only the 8 warps that own a chunk (2 column slices x 4 quarters) release it
            mbar_init(&tempty[b], (MODE == 41 || MODE == 46) ? 8
                                  : (MODE == 51 || MODE == 52) ? 1
                                                               : (ProbeMode<MODE>::PER_THREAD ? 32 : 1) * 4 * EPI_SPLIT);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        *flag_go = 0;
        *flag_back = 0;
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
    } else if (warp == 1 && lane == 0 && MODE >= 47 && MODE <= 50) {
        // latency detail, one thread per SM: 47 = 1 MMA + commit with a spinning wait;
        // 48 = a commit alone (nothing in flight) with a suspending wait; 49 = the
        // same with a spinning wait; 50 = 2 MMAs + commit with a spinning wait
        constexpr int NM = MODE == 47 ? 1 : (MODE == 50 ? 2 : 0);
        constexpr bool SPINW = MODE != 48;
        constexpr uint32_t idesc = idesc_f16(false, false, BM, BN);
        uint32_t ph = 0;
        for (int c = 0; c < chunks; ++c) {
#pragma unroll
            for (int h = 0; h < NM; ++h)
                umma_f16(tmem, sdesc_sw128(a0 + h * 32, 16, 1024), sdesc_sw128(b0 + h * 32, 16, 1024), idesc, h);
            umma_commit(done);
            const bool ok = SPINW ? mbar_wait_spin(done, ph, abort_flag, status, kStatusTimeoutProbe)
                                  : mbar_wait(done, ph, abort_flag, status, kStatusTimeoutProbe);
            if (!ok) break;
            ph ^= 1u;
        }
    } else if ((MODE == 51 || MODE == 52) && (warp == 1 || warp == 2) && lane == 0) {
        // mbarrier ping-pong between one thread of warp 1 and one of warp 2 (two
        // sub-partitions), two hops per iteration: 51 suspending waits, 52 spinning
        const bool ping = warp == 1;
        uint32_t ph = 0;
        for (int c = 0; c < chunks; ++c) {
            if (ping) mbar_arrive(&tfull[0]);
            uint64_t* w = ping ? &tempty[0] : &tfull[0];
            const bool ok = MODE == 52 ? mbar_wait_spin(w, ph, abort_flag, status, kStatusTimeoutProbe)
                                       : mbar_wait(w, ph, abort_flag, status, kStatusTimeoutProbe);
            if (!ok) break;
            if (!ping) mbar_arrive(&tempty[0]);
            ph ^= 1u;
        }
    } else if (MODE >= 53 && MODE <= 56 && warp >= 1) {
        // Release round trip between one issuing thread (warp 1) and the 16 epilogue
        // warps, no MMAs: the issuer signals "go", every epilogue warp answers, the
        // issuer waits for all 16 answers.  53: mbarriers both ways (the product's
        // tfull/tempty); 54: shared-memory flags (a go word, an answer count);
        // 55: named barriers both ways (bar.arrive / bar.sync, 17 warps);
        // 56: an mbarrier out (as a commit would be) and a named barrier back.
        // Every warp runs exactly `chunks` iterations with no early exit, so the
        // named-barrier counts always match.
        constexpr int NB = 32 * (1 + 4 * EPI_SPLIT);
        const bool issuer = warp == 1;
        uint32_t ph = 0;
        for (int c = 0; c < chunks; ++c) {
            if (issuer) {
                if (MODE == 53 || MODE == 56) {
                    if (lane == 0) mbar_arrive(&tfull[0]);
                } else if (MODE == 54) {
                    if (lane == 0) st_release_smem(flag_go, uint32_t(c + 1));
                } else {
                    named_bar_arrive(1, NB);
                }
                if (MODE == 53) {
                    if (lane == 0) mbar_wait(&tempty[0], ph, abort_flag, status, kStatusTimeoutProbe);
                } else if (MODE == 54) {
                    if (lane == 0) spin_ge(flag_back, uint32_t(4 * EPI_SPLIT * (c + 1)), status);
                } else {
                    named_bar_sync(2, NB);
                }
                __syncwarp();
            } else {
                if (MODE == 53 || MODE == 56) {
                    mbar_wait(&tfull[0], ph, abort_flag, status, kStatusTimeoutProbe);
                } else if (MODE == 54) {
                    if (lane == 0) spin_ge(flag_go, uint32_t(c + 1), status);
                } else {
                    named_bar_sync(1, NB);
                }
                __syncwarp();
                if (MODE == 53) {
                    if (lane == 0) mbar_arrive(&tempty[0]);
                } else if (MODE == 54) {
                    if (lane == 0) red_release_add_smem(flag_back, 1u);
                } else {
                    named_bar_arrive(2, NB);
                }
            }
            ph ^= 1u;
        }
    } else if (MODE == 46 && warp == 1 && lane == 0) {
        // pairs split by N-halves: per pair and half, 4 MMAs N=64 (2 chunks) + one commit;
        // tfull/tempty index = half * 2 + pair
        constexpr uint32_t idesc = idesc_f16(false, false, BM, 64);
        uint32_t p = 0, ph = 0;
        for (int c = 0; c < chunks; c += 2) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                if (!mbar_wait(&tempty[h * 2 + p], ph ^ 1u, abort_flag, status, kStatusTimeoutProbe)) goto probe46_done;
                tc_fence_after();
#pragma unroll
                for (int k = 0; k < 2; ++k)
#pragma unroll
                    for (int s = 0; s < 2; ++s)
                        umma_f16(tmem + (2 * p + k) * BN + h * 64, sdesc_sw128(a0 + s * 32, 16, 1024),
                                 sdesc_sw128(b0 + h * 64 * 128 + s * 32, 16, 1024), idesc, s);
                umma_commit(&tfull[h * 2 + p]);
            }
            p ^= 1u;
            if (p == 0) ph ^= 1u;
        }
    probe46_done:
        umma_commit(done);
        mbar_wait_drain(done, 0);
    } else if (MODE == 46 && warp >= 2) {
        const int e = warp - 2, q = warp & 3, colg = e >> 2, half = colg >> 1;  // 16 warps, 32 columns each
        const uint32_t base = tmem + (static_cast<uint32_t>(q * 32) << 16) + colg * 32;
        float acc[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] = 0.0f;
        uint32_t p = 0, ph = 0;
        for (int c = 0; c < chunks; c += 2) {
            const bool ok = mbar_wait(&tfull[half * 2 + p], ph, abort_flag, status, kStatusTimeoutProbe);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            uint32_t r0[16], r1[16];
            tmem_ld_chunk<32>(base + (2 * p) * BN, r0);
            tmem_ld_chunk<32>(base + (2 * p + 1) * BN, r1);
            tmem_wait_ld();
            reg_fence(r0);
            reg_fence(r1);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[half * 2 + p]);
            add_chunk<32>(acc, r0);
            add_chunk<32>(acc, r1);
            p ^= 1u;
            if (p == 0) ph ^= 1u;
        }
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j) s += acc[j];
        out[blockIdx.x * blockDim.x + threadIdx.x] = s;
    } else if (MODE == 45 && warp == 1 && lane == 0) {
        // wide chunks: 2 MMAs N=256 per chunk into 2 buffers of 256 columns
        constexpr uint32_t idesc = idesc_f16(false, false, BM, 256);
        uint32_t b = 0, ph = 0;
        for (int c = 0; c < chunks; c += 2) {  // `chunks` counts 128-column chunks, 2 per wide chunk
            if (!mbar_wait(&tempty[b], ph ^ 1u, abort_flag, status, kStatusTimeoutProbe)) break;
            tc_fence_after();
#pragma unroll
            for (int h = 0; h < 2; ++h)
                umma_f16(tmem + b * 256, sdesc_sw128(a0 + h * 32, 16, 1024), sdesc_sw128(b0 + h * 32, 16, 1024),
                         idesc, h);
            umma_commit(&tfull[b]);
            if (++b == 2) { b = 0; ph ^= 1u; }
        }
        umma_commit(done);
        mbar_wait_drain(done, 0);
    } else if (MODE == 45 && warp >= 2) {
        const int e = warp - 2, q = warp & 3, colg = e >> 2;  // 16 warps: 4 slices of 64 over 256 columns
        ChunkRing<2> ring{tfull, tempty, tmem + (static_cast<uint32_t>(q * 32) << 16) + colg * 64, 256};
        float acc[64];
#pragma unroll
        for (int j = 0; j < 64; ++j) acc[j] = 0.0f;
        consume_chunks<64>(acc, chunks / 2, ring, lane, abort_flag, status);
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < 64; ++j) s += acc[j];
        out[blockIdx.x * blockDim.x + threadIdx.x] = s;
    } else if ((MODE == 40 || MODE == 42 || MODE == 43) && warp == 1 && lane == 0) {
        // pairs: one tempty wait, 4 MMAs into 2 chunk buffers, one commit per 2 chunks
        constexpr uint32_t idesc = idesc_f16(false, false, BM, BN);
        uint32_t p = 0, ph = 0;
        for (int c = 0; c < chunks; c += 2, p ^= 1u) {
            if (!mbar_wait(&tempty[p], ph ^ 1u, abort_flag, status, kStatusTimeoutProbe)) break;
            tc_fence_after();
#pragma unroll
            for (int k = 0; k < 2; ++k)
#pragma unroll
                for (int h = 0; h < 2; ++h)
                    umma_f16(tmem + (2 * p + k) * BN, sdesc_sw128(a0 + h * 32, 16, 1024),
                             sdesc_sw128(b0 + h * 32, 16, 1024), idesc, h);
            umma_commit(&tfull[p]);
            if (p == 1) ph ^= 1u;
        }
        umma_commit(done);
        mbar_wait_drain(done, 0);
    } else if ((MODE == 40 || MODE == 42) && warp >= 2) {
        const int e = warp - 2, q = warp & 3, colg = e >> 2;
        const uint32_t base = tmem + (static_cast<uint32_t>(q * 32) << 16) + colg * CW;
        float acc[CW];
#pragma unroll
        for (int j = 0; j < CW; ++j) acc[j] = 0.0f;
        uint32_t p = 0, ph = 0;
        for (int c = 0; c < chunks; c += 2, p ^= 1u) {
            const bool ok = mbar_wait(&tfull[p], ph, abort_flag, status, kStatusTimeoutProbe);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            uint32_t r0[CW / 2], r1[CW / 2];
            tmem_ld_chunk<CW>(base + (2 * p) * BN, r0);
            tmem_ld_chunk<CW>(base + (2 * p + 1) * BN, r1);
            tmem_wait_ld();
            reg_fence(r0);
            reg_fence(r1);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[p]);
            add_chunk<CW>(acc, r0);
            add_chunk<CW>(acc, r1);
            if (p == 1) ph ^= 1u;
        }
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < CW; ++j) s += acc[j];
        out[blockIdx.x * blockDim.x + threadIdx.x] = s;
    } else if (MODE == 43 && warp >= 2) {
        // pairs, software pipelined: the next pair's loads are in flight while this pair is added
        const int e = warp - 2, q = warp & 3, colg = e >> 2;
        const uint32_t base = tmem + (static_cast<uint32_t>(q * 32) << 16) + colg * CW;
        float acc[CW];
#pragma unroll
        for (int j = 0; j < CW; ++j) acc[j] = 0.0f;
        uint32_t ra0[CW / 2], ra1[CW / 2], rb0[CW / 2], rb1[CW / 2];
        uint32_t p = 0, ph = 0;
        auto wait_pair = [&]() {
            const bool ok = mbar_wait(&tfull[p], ph, abort_flag, status, kStatusTimeoutProbe);
            if (!__all_sync(0xffffffffu, ok)) return false;
            tc_fence_after();
            return true;
        };
        auto release_pair = [&]() {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[p]);
            if (p == 1) ph ^= 1u;
            p ^= 1u;
        };
        const int pairs = chunks / 2;
        if (pairs > 0 && wait_pair()) {
            tmem_ld_chunk<CW>(base + (2 * p) * BN, ra0);
            tmem_ld_chunk<CW>(base + (2 * p + 1) * BN, ra1);
            for (int i = 0; i < pairs; i += 2) {
                tmem_wait_ld();
                reg_fence(ra0);
                reg_fence(ra1);
                release_pair();
                const bool more = i + 1 < pairs;
                if (more) {
                    if (!wait_pair()) break;
                    tmem_ld_chunk<CW>(base + (2 * p) * BN, rb0);
                    tmem_ld_chunk<CW>(base + (2 * p + 1) * BN, rb1);
                }
                add_chunk<CW>(acc, ra0);
                add_chunk<CW>(acc, ra1);
                if (!more) break;
                tmem_wait_ld();
                reg_fence(rb0);
                reg_fence(rb1);
                release_pair();
                const bool more2 = i + 2 < pairs;
                if (more2) {
                    if (!wait_pair()) break;
                    tmem_ld_chunk<CW>(base + (2 * p) * BN, ra0);
                    tmem_ld_chunk<CW>(base + (2 * p + 1) * BN, ra1);
                }
                add_chunk<CW>(acc, rb0);
                add_chunk<CW>(acc, rb1);
                if (!more2) break;
            }
        }
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < CW; ++j) s += acc[j];
        out[blockIdx.x * blockDim.x + threadIdx.x] = s;
    } else if (MODE == 41 && warp >= 2) {
        // turn groups: two warps per (lane quarter, column slice) take alternate chunks
        const int e = warp - 2, q = warp & 3, turn = (e >> 2) & 1, colg = e >> 3;
        constexpr int CW41 = 64;
        const uint32_t base = tmem + (static_cast<uint32_t>(q * 32) << 16) + colg * CW41;
        float acc[CW41];
#pragma unroll
        for (int j = 0; j < CW41; ++j) acc[j] = 0.0f;
        for (int c = turn; c < chunks; c += 2) {
            const uint32_t b = c & (NBUF - 1), ph = (c / NBUF) & 1;
            const bool ok = mbar_wait(&tfull[b], ph, abort_flag, status, kStatusTimeoutProbe);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            uint32_t r[CW41 / 2];
            tmem_ld_chunk<CW41>(base + b * BN, r);
            tmem_wait_ld();
            reg_fence(r);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[b]);
            add_chunk<CW41>(acc, r);
        }
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < CW41; ++j) s += acc[j];
        out[blockIdx.x * blockDim.x + threadIdx.x] = s;
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

// mma.sync fed from shared memory, the shape a register-accumulator GEMM would
// use: 8 warps, each a 64 x 64 output tile (32 m16n8 tiles), per 32-long chunk
// 16 ldmatrix.x4 (A 4 m-tiles x 2 k-halves, B 8 n-tiles x 2 k-halves), 64
// mma.sync with an FP16 accumulator, 128 mixed adds into FP32 registers.
// Operands are a fixed smem tile (A 128 x 32, B 256 x 32 K-contiguous,
// padded rows).  33: as described; 34: the same without the FP32 adds (the
// FP16 chunk results XOR-folded instead) to separate issue from smem costs.
template <int MODE>
__global__ void __launch_bounds__(256, 1) mma_sync_smem_kernel(int chunks, float* out) {
    constexpr int LDK = 40;  // halves per smem row: 32 + 8 padding, conflict-free ldmatrix
    __shared__ __align__(128) __half sA[128 * LDK];
    __shared__ __align__(128) __half sB[256 * LDK];
    for (int i = threadIdx.x; i < 128 * LDK; i += 256) sA[i] = __float2half((i & 3) == 0 ? 1.0f : 0.0f);
    for (int i = threadIdx.x; i < 256 * LDK; i += 256) sB[i] = __float2half((i & 5) == 0 ? 1.0f : 0.0f);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wm = warp >> 2, wn = warp & 3;  // 2 x 4 warps: rows wm*64, cols wn*64
    float acc[4][8][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int v = 0; v < 4; ++v) acc[i][j][v] = 0.0f;
    uint32_t fold = 0;
    for (int c = 0; c < chunks; ++c) {
        uint32_t af[2][4][4], bf[2][8][2];
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const __half* src = &sA[(wm * 64 + i * 16 + (lane & 15)) * LDK + ks * 16 + (lane >> 4) * 8];
                asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                             : "=r"(af[ks][i][0]), "=r"(af[ks][i][1]), "=r"(af[ks][i][2]), "=r"(af[ks][i][3])
                             : "r"(smem_u32(src)));
            }
#pragma unroll
            for (int jp = 0; jp < 4; ++jp) {
                const __half* src = &sB[(wn * 64 + jp * 16 + (lane >> 4) * 8 + (lane & 7)) * LDK + ks * 16 +
                                        ((lane >> 3) & 1) * 8];
                asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                             : "=r"(bf[ks][2 * jp][0]), "=r"(bf[ks][2 * jp][1]), "=r"(bf[ks][2 * jp + 1][0]),
                               "=r"(bf[ks][2 * jp + 1][1])
                             : "r"(smem_u32(src)));
            }
        }
        if constexpr (MODE == 33 || MODE == 34) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    uint32_t h0 = 0, h1 = 0;
#pragma unroll
                    for (int ks = 0; ks < 2; ++ks)
                        asm volatile(
                            "mma.sync.aligned.m16n8k16.row.col.f16.f16.f16.f16 {%0,%1}, {%2,%3,%4,%5}, {%6,%7}, "
                            "{%0,%1};"
                            : "+r"(h0), "+r"(h1)
                            : "r"(af[ks][i][0]), "r"(af[ks][i][1]), "r"(af[ks][i][2]), "r"(af[ks][i][3]),
                              "r"(bf[ks][j][0]), "r"(bf[ks][j][1]));
                    if constexpr (MODE == 33) {
                        add_f16x2_to_f32(acc[i][j][0], acc[i][j][1], h0);
                        add_f16x2_to_f32(acc[i][j][2], acc[i][j][3], h1);
                    } else {
                        fold ^= h0 ^ h1;
                    }
                }
        } else {
            // 35 / 36: groups of G tiles -- every tile's first K16 MMA, then every
            // second one, then the adds -- so no MMA waits on the one just issued
            constexpr int G = MODE == 35 ? 8 : 16;
#pragma unroll
            for (int g0 = 0; g0 < 32; g0 += G) {
                uint32_t h[G][2];
#pragma unroll
                for (int ks = 0; ks < 2; ++ks)
#pragma unroll
                    for (int t = 0; t < G; ++t) {
                        const int i = (g0 + t) >> 3, j = (g0 + t) & 7;
                        if (ks == 0) h[t][0] = h[t][1] = 0u;
                        asm("mma.sync.aligned.m16n8k16.row.col.f16.f16.f16.f16 {%0,%1}, {%2,%3,%4,%5}, {%6,%7}, "
                            "{%0,%1};"
                            : "+r"(h[t][0]), "+r"(h[t][1])
                            : "r"(af[ks][i][0]), "r"(af[ks][i][1]), "r"(af[ks][i][2]), "r"(af[ks][i][3]),
                              "r"(bf[ks][j][0]), "r"(bf[ks][j][1]));
                    }
#pragma unroll
                for (int t = 0; t < G; ++t) {
                    const int i = (g0 + t) >> 3, j = (g0 + t) & 7;
                    add_f16x2_to_f32(acc[i][j][0], acc[i][j][1], h[t][0]);
                    add_f16x2_to_f32(acc[i][j][2], acc[i][j][3], h[t][1]);
                }
            }
        }
    }
    float s = __uint_as_float(fold);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) s += acc[i][j][0] + acc[i][j][1] + acc[i][j][2] + acc[i][j][3];
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
    if (mode >= 30 && mode <= 36) {  // `grid` blocks of 8 warps; out holds grid * 256 floats
        switch (mode) {
            case 30: mma_sync_rate_kernel<30><<<grid, 256, 0, stream>>>(chunks, out); break;
            case 31: mma_sync_rate_kernel<31><<<grid, 256, 0, stream>>>(chunks, out); break;
            case 32: mma_sync_rate_kernel<32><<<grid, 256, 0, stream>>>(chunks, out); break;
            case 33: mma_sync_smem_kernel<33><<<grid, 256, 0, stream>>>(chunks, out); break;
            case 34: mma_sync_smem_kernel<34><<<grid, 256, 0, stream>>>(chunks, out); break;
            case 35: mma_sync_smem_kernel<35><<<grid, 256, 0, stream>>>(chunks, out); break;
            case 36: mma_sync_smem_kernel<36><<<grid, 256, 0, stream>>>(chunks, out); break;
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
            case 40: return launch_probe<40, 2>(chunks, grid, out, status, stream);
            case 47: return launch_probe<47, 2>(chunks, grid, out, status, stream);
            case 48: return launch_probe<48, 2>(chunks, grid, out, status, stream);
            case 49: return launch_probe<49, 2>(chunks, grid, out, status, stream);
            case 50: return launch_probe<50, 2>(chunks, grid, out, status, stream);
            case 51: return launch_probe<51, 2>(chunks, grid, out, status, stream);
            case 52: return launch_probe<52, 2>(chunks, grid, out, status, stream);
        }
    }
    if (epi_split == 4) {
        switch (mode) {
            case 2: return launch_probe<2, 4>(chunks, grid, out, status, stream);
            case 3: return launch_probe<3, 4>(chunks, grid, out, status, stream);
            case 6: return launch_probe<6, 4>(chunks, grid, out, status, stream);
            case 7: return launch_probe<7, 4>(chunks, grid, out, status, stream);
            case 41: return launch_probe<41, 4>(chunks, grid, out, status, stream);
            case 42: return launch_probe<42, 4>(chunks, grid, out, status, stream);
            case 43: return launch_probe<43, 4>(chunks, grid, out, status, stream);
            case 45: return launch_probe<45, 4>(chunks, grid, out, status, stream);
            case 46: return launch_probe<46, 4>(chunks, grid, out, status, stream);
            case 53: return launch_probe<53, 4>(chunks, grid, out, status, stream);
            case 54: return launch_probe<54, 4>(chunks, grid, out, status, stream);
            case 55: return launch_probe<55, 4>(chunks, grid, out, status, stream);
            case 56: return launch_probe<56, 4>(chunks, grid, out, status, stream);
        }
    }
    return cudaErrorInvalidValue;
}

}  // namespace f16acc
