// tc_epilogue.cuh -- the per-chunk epilogue of the chunked tcgen05 kernel:
// TMEM -> registers (FP16 pairs packed) and one mixed-precision FP32 add per
// element, software pipelined so the TMEM load of chunk c+1 is in flight while
// chunk c is being added.  Shared by the GEMM kernel and the chunk-rate probe
// so the probe measures exactly the product's code.
#pragma once

#include "ptx.cuh"

namespace f16acc {

// Keep the compiler from moving uses of TMEM-loaded registers above the
// tcgen05.wait::ld that makes them valid: each register is "redefined" by an
// empty volatile asm placed after the wait.
template <int N>
__device__ __forceinline__ void reg_fence(uint32_t (&r)[N]) {
#pragma unroll
    for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

// Load CW consecutive 16-bit accumulator columns of this warp's 32 TMEM lanes,
// two columns per register (low half = lower column).
template <int CW>
__device__ __forceinline__ void tmem_ld_chunk(uint32_t taddr, uint32_t (&r)[CW / 2]) {
    static_assert(CW == 32 || CW % 64 == 0, "column slice");
    if constexpr (CW == 32) {
        tmem_ld_32x32b_x16_pack16(taddr, r);
    } else {
#pragma unroll
        for (int j = 0; j < CW / 64; ++j)
            tmem_ld_32x32b_x32_pack16(taddr + j * 64, *reinterpret_cast<uint32_t(*)[32]>(&r[j * 32]));
    }
}

template <int CW>
__device__ __forceinline__ void add_chunk(float (&acc)[CW], const uint32_t (&r)[CW / 2]) {
#pragma unroll
    for (int i = 0; i < CW / 2; ++i) add_f16x2_to_f32(acc[2 * i], acc[2 * i + 1], r[i]);
}

// Ring of NBUF chunk accumulators in TMEM shared with the MMA warp:
// tfull[b] completes when chunk b's MMAs are done, tempty[b] gets one arrival
// per epilogue warp once that warp has its values in registers.
// PER_THREAD: every thread arrives on tempty (barrier count = 32 x epilogue
// warps) instead of one elected lane after a __syncwarp.  NO_FENCE drops the
// tcgen05 fences (only valid where no tcgen05 op is ordered by the hand-off).
template <int NBUF, bool SPIN = false, bool PER_THREAD = false, bool NO_FENCE = false>
struct ChunkRing {
    uint64_t* tfull;
    uint64_t* tempty;
    uint32_t col_base;  // TMEM address of buffer 0 for this warp's lanes and column slice
    uint32_t stride;    // TMEM columns between buffers
    uint32_t b = 0, phase = 0;

    __device__ __forceinline__ uint32_t addr() const { return col_base + b * stride; }
    __device__ __forceinline__ bool wait_full(volatile int* abort, int* status) {
        const bool ok = SPIN ? mbar_wait_spin(&tfull[b], phase, abort, status, kStatusTimeoutEpilogue)
                             : mbar_wait(&tfull[b], phase, abort, status, kStatusTimeoutEpilogue);
        if (!__all_sync(0xffffffffu, ok)) return false;
        if (!NO_FENCE) tc_fence_after();
        return true;
    }
    __device__ __forceinline__ void release(int lane) {
        if (!NO_FENCE) tc_fence_before();
        if (PER_THREAD) {
            mbar_arrive(&tempty[b]);
        } else {
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[b]);
        }
        if (++b == NBUF) { b = 0; phase ^= 1u; }
    }
};

// Sum `nchunks` chunk accumulators into acc (FP32), consuming them from the
// ring in order.  Returns false when a wait gave up (nothing in flight then).
template <int CW, typename Ring>
__device__ __forceinline__ bool consume_chunks(float (&acc)[CW], int nchunks, Ring& ring, int lane,
                                               volatile int* abort, int* status) {
    uint32_t ra[CW / 2], rb[CW / 2];
    if (nchunks <= 0) return true;
    if (!ring.wait_full(abort, status)) return false;
    tmem_ld_chunk<CW>(ring.addr(), ra);
    for (int c = 0;; c += 2) {
        // chunk c: loaded into ra
        tmem_wait_ld();
        reg_fence(ra);
        ring.release(lane);
        if (c + 1 >= nchunks) {
            add_chunk<CW>(acc, ra);
            return true;
        }
        if (!ring.wait_full(abort, status)) return false;
        tmem_ld_chunk<CW>(ring.addr(), rb);  // chunk c+1 in flight while chunk c is added
        add_chunk<CW>(acc, ra);
        // chunk c+1: loaded into rb
        tmem_wait_ld();
        reg_fence(rb);
        ring.release(lane);
        if (c + 2 >= nchunks) {
            add_chunk<CW>(acc, rb);
            return true;
        }
        if (!ring.wait_full(abort, status)) return false;
        tmem_ld_chunk<CW>(ring.addr(), ra);
        add_chunk<CW>(acc, rb);
    }
}

}  // namespace f16acc
