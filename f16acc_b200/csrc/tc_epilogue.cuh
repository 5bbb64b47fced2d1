// tc_epilogue.cuh -- the per-chunk epilogue of the chunked tcgen05 kernel:
// TMEM -> registers (FP16 pairs packed) and one mixed-precision FP32 add per
// element.  Shared by the GEMM kernel and the chunk-rate probe so the probe
// measures exactly the product's code.
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
template <int CW>
__device__ __forceinline__ void init_chunk(float (&acc)[CW], const uint32_t (&r)[CW / 2]) {
#pragma unroll
    for (int i = 0; i < CW / 2; ++i) init_f16x2_to_f32(acc[2 * i], acc[2 * i + 1], r[i]);
}

// Ring of NBUF accumulators in TMEM shared with the MMA warp (FP32 mode):
// tfull[b] completes when buffer b's MMAs are done, tempty[b] gets one arrival
// per epilogue warp once that warp has its values in registers.
template <int NBUF>
struct ChunkRing {
    uint64_t* tfull;
    uint64_t* tempty;
    uint32_t col_base;  // TMEM address of buffer 0 for this warp's lanes and column slice
    uint32_t stride;    // TMEM columns between buffers
    uint32_t b = 0, phase = 0;

    __device__ __forceinline__ uint32_t addr() const { return col_base + b * stride; }
    __device__ __forceinline__ bool wait_full(volatile int* abort, int* status) {
        const bool ok = mbar_wait(&tfull[b], phase, abort, status, kStatusTimeoutEpilogue);
        if (!__all_sync(0xffffffffu, ok)) return false;
        tc_fence_after();
        return true;
    }
    __device__ __forceinline__ void release(int lane) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[b]);
        if (++b == NBUF) { b = 0; phase ^= 1u; }
    }
};

// Chunk pairs: an MMA thread fills the two chunk buffers (2p, 2p+1) of pair p
// from one 64-wide smem stage and signals them with one commit on tfull[p];
// the epilogue reads both and releases the pair with one arrival on named
// barrier kPairBarrier + p, on which the pair's MMA warp bar.syncs before
// reusing it.  Two pairs in flight (4 buffers).  Handing chunks over in pairs
// halves the hand-offs: each costs a commit and a barrier hop of latency, and
// only 4 chunk buffers fit in TMEM.  The release is a named barrier rather
// than an mbarrier because its round trip is about half as long (bar.arrive
// wakes a bar.sync sooner than an mbarrier arrive wakes a try_wait).
constexpr int kPairBarrier = 1;  // named barrier IDs 1 and 2, one per pair

template <int CW>
struct PairRing {
    uint64_t* tfull;   // [2], one per pair
    int bar_threads;   // threads of one MMA warp + the epilogue warps
    uint32_t col_base; // TMEM address of buffer 0 for this warp's lanes and column slice
    uint32_t stride;   // TMEM columns between chunk buffers
    uint32_t p = 0, phase = 0;  // pair of the next hand-off and its tfull phase parity

    // Wait for pair p's next hand-off (whole warp; false when the wait gave up).
    __device__ __forceinline__ bool wait(volatile int* abort, int* status) {
        const bool ok = mbar_wait(&tfull[p], phase, abort, status, kStatusTimeoutEpilogue);
        return __all_sync(0xffffffffu, ok);
    }
    // Whole warp, after its TMEM loads of pair p have completed.
    __device__ __forceinline__ void release() {
        tc_fence_before();
        __syncwarp();
        named_bar_arrive(kPairBarrier + int(p), bar_threads);
        p ^= 1u;
        if (p == 0) phase ^= 1u;
    }

    // Whole warp, when leaving before the end (after raising the abort flag):
    // arrive once for every hand-off that was issued and not yet released by
    // this warp, so that an MMA warp in bar.sync on it wakes.  That is at most
    // the next hand-off of each pair (a pair's MMA warp issues into it again
    // only after every epilogue warp released it), and it was issued exactly
    // when its tfull completes, which the MMAs do within microseconds (waited
    // for up to 20 ms).  Arriving only for issued hand-offs never puts a second
    // arrival of this warp into a round.
    __device__ __forceinline__ void release_issued_on_exit(int lane) {
        uint32_t pp = p, ph = phase;
        for (int k = 0; k < 2; ++k) {
            bool issued = false;
            if (lane == 0) issued = mbar_wait_for(&tfull[pp], ph, 20000000ull);
            issued = __shfl_sync(0xffffffffu, issued, 0);
            if (issued) named_bar_arrive(kPairBarrier + int(pp), bar_threads);
            pp ^= 1u;
            if (pp == 0) ph ^= 1u;
        }
    }
};

// Sum `nchunks` (>= 1) chunks, delivered in pairs, into acc (FP32); the first
// chunk initialises acc (the value an add into zeros gives), so acc needs no
// zeroing at the start of a tile.  The last pair of a tile holds one chunk
// when nchunks is odd.  Returns false when a wait gave
// up (no TMEM load is left in flight then).
template <int CW>
__device__ __forceinline__ bool consume_chunk_pairs(float (&acc)[CW], int nchunks, PairRing<CW>& ring,
                                                    volatile int* abort, int* status) {
    for (int c = 0; c < nchunks; c += 2) {
        if (!ring.wait(abort, status)) return false;
        tc_fence_after();
        const bool two = c + 1 < nchunks;
        const uint32_t a0 = ring.col_base + (2 * ring.p) * ring.stride;
        uint32_t r0[CW / 2], r1[CW / 2];
        tmem_ld_chunk<CW>(a0, r0);
        if (two) tmem_ld_chunk<CW>(a0 + ring.stride, r1);
        tmem_wait_ld();
        reg_fence(r0);
        if (two) reg_fence(r1);
        ring.release();
        if (c == 0)
            init_chunk<CW>(acc, r0);
        else
            add_chunk<CW>(acc, r0);
        if (two) add_chunk<CW>(acc, r1);
    }
    return true;
}

// One FP32 accumulator (a whole redo tile) handed over through the pair ring:
// it sits in the pair's first chunk buffer.  Returns false when the wait gave up.
template <int CW>
__device__ __forceinline__ bool consume_fp32_pair(float (&acc)[CW], PairRing<CW>& ring, volatile int* abort,
                                                  int* status) {
    if (!ring.wait(abort, status)) return false;
    tc_fence_after();
    const uint32_t a0 = ring.col_base + (2 * ring.p) * ring.stride;
#pragma unroll
    for (int j = 0; j < CW / 32; ++j) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(a0 + j * 32, r);
        tmem_wait_ld();
        reg_fence(r);
#pragma unroll
        for (int k = 0; k < 32; ++k) acc[j * 32 + k] = __uint_as_float(r[k]);
    }
    ring.release();
    return true;
}

}  // namespace f16acc
