// skinny_gemm.cuh -- the chunked GEMM for few rows (M <= 64: decode-shaped
// products).  A 128-row tensor-core tile would waste most of its MMA work
// there, and the time goes to streaming B (the weight) from HBM once, so this
// kernel is built for memory-level parallelism instead.
//
// Reference semantics (steppergg/f16acc f16acc/kernel.py:37-81): 32-long K
// chunks from absolute offset 0, each accumulated in FP16 (two m16n8k16 MMAs
// with FP16 C/D, rounding after each K=16 step as on every path here), the
// chunk values added in FP32; a tile with a non-finite sum is flagged and
// recomputed with FP32 accumulation.
//
// Design.  Output tile 16*MT x 128 (MT m16 row blocks cover M), 4 warps of 32
// columns.  The K range is split over a thread-block cluster of S <= 8 CTAs
// along y: CTA s sums the chunks of its own K range, a multiple of 64 long, in
// FP32.  Operands move global -> shared memory with cp.async in a 4-5 stage ring
// (rows padded for conflict-free ldmatrix).  The partial tiles are then added
// in the fixed order s = 0, 1, ..., S-1, each CTA taking a share of the tile
// and reading the others' shared memory (distributed shared memory); the
// cluster ORs its non-finite checks, rank 0 writes the tile's flag, and with
// the in-kernel redo a flagged tile is recomputed in FP32 mode by the same
// cluster in the same launch.  S is a function of the shape only, so FP32
// mode, the in-kernel redo and the separate redo launch add the same partials
// in the same order: bit-identical results.
//
// The FP32 sum over chunks is associated per K range here (partials added
// after), where the other kernels add chunk by chunk: an FP32 rounding
// difference, inside the parity bound.
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"
#include "mma_gemm.cuh"
#include "ptx.cuh"

namespace f16acc {

struct SkinnyParams {
    const __half* A;  // [M, K], K contiguous, 16-byte aligned rows
    const __half* B;  // [K, N]: K-contiguous columns (sBk == 1) or N-contiguous rows (sBn == 1), 16-byte aligned
    void* C;
    int64_t sAm, sBk, sBn, sCm, sCn;
    int M, N, K;
    int kper;         // K range of one CTA of a cluster, a multiple of 64
    int c_vec;        // C has unit column stride, rows aligned for 4-element vector stores
    uint8_t* flags;   // 16 bytes per 128-column tile
    const __half* bias;
    int64_t sbias;
    int inline_redo;  // chunked mode: redo a flagged tile in this launch
};

struct SkinnyCfg {
    static constexpr int BN = 128, BK = 64, THREADS = 128;
    static constexpr int LDK = BK + 8;   // [row][k] pitch (halves)
    static constexpr int LDN = BN + 8;   // [k][n] pitch (halves)
    static constexpr int MAX_S = 8;      // portable cluster size
    static constexpr int TARGET_CTAS = 296;  // the split aims at one wave of two CTAs per SM of a B200
    // Ring depth: as many stages as keep two CTAs resident per SM (the bytes in
    // flight per SM are what the streaming of B needs).  SHALLOW, for launches
    // of more single-CTA tiles than one wave holds (lm_head-sized N): 3 stages,
    // so three CTAs fit per SM and one's pipeline fill and tile end overlap the
    // others' streaming (measured on the lm_head shape at M = 1 / 16 / 32:
    // 96.6 -> 88.5, 100.8 -> 94.7, 117 -> 104 us; with a K split, or at 64
    // rows, the deeper ring is faster).
    template <int MT, bool SHALLOW = false>
    static constexpr int stages() { return SHALLOW ? 3 : (MT == 1 ? 5 : 4); }
    template <int MT>
    static constexpr int a_elems() { return 16 * MT * LDK; }
    template <bool B_KN>
    static constexpr int b_elems() { return B_KN ? BK * LDN : BN * LDK; }
    template <int MT, bool B_KN, bool SHALLOW = false>
    static constexpr int smem_bytes() { return stages<MT, SHALLOW>() * (a_elems<MT>() + b_elems<B_KN>()) * 2; }
    static constexpr int RED_LD = BN + 4;  // FP32 partial tile pitch (floats)
};

// 16-byte global -> shared copy; bytes past `src_bytes` (0..16) are zero-filled.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(gsrc), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Sum this CTA's K range [k_begin, k_end) into acc (FP32): chunk by chunk in FP16
// (CHUNKED) or straight FP32 accumulation.  Leaves every cp.async drained and
// the ring free (it ends with a __syncthreads).
template <int MT, bool CHUNKED, bool B_KN, bool SHALLOW>
__device__ __forceinline__ void skinny_mainloop(const SkinnyParams& p, __half* sA, __half* sB, int n0, int k_begin,
                                                int k_end, float (&acc)[MT][4][4]) {
    using Cfg = SkinnyCfg;
    constexpr int BK = Cfg::BK, STAGES = Cfg::stages<MT, SHALLOW>(), LDK = Cfg::LDK, LDN = Cfg::LDN;
    constexpr int A_EL = Cfg::a_elems<MT>(), B_EL = Cfg::b_elems<B_KN>();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int v = 0; v < 4; ++v) acc[i][j][v] = 0.0f;
    const int nst = (k_end - k_begin + BK - 1) / BK;

    auto load_stage = [&](int st) {
        const int buf = st % STAGES;
        const int k0 = k_begin + st * BK;
        // A: 16*MT rows x 8 vectors of 8 halves
#pragma unroll
        for (int v = 0; v < MT; ++v) {
            const int idx = tid + v * Cfg::THREADS;
            const int r = idx >> 3, kv = (idx & 7) * 8;
            const int k = k0 + kv;
            const int bytes = (r < p.M && k < k_end) ? min(16, (k_end - k) * 2) : 0;
            const __half* src = p.A + (bytes ? int64_t(r) * p.sAm + k : 0);
            cp_async16(&sA[buf * A_EL + r * LDK + kv], src, bytes);
        }
        if constexpr (B_KN) {
            // B rows k (64) x 16 vectors of 8 columns
#pragma unroll
            for (int v = 0; v < 8; ++v) {
                const int idx = tid + v * Cfg::THREADS;
                const int kr = idx >> 4, nv = (idx & 15) * 8;
                const int k = k0 + kr, n = n0 + nv;
                const int bytes = (k < k_end && n < p.N) ? min(16, (p.N - n) * 2) : 0;
                const __half* src = p.B + (bytes ? int64_t(k) * p.sBk + n : 0);
                cp_async16(&sB[buf * B_EL + kr * LDN + nv], src, bytes);
            }
        } else {
            // B columns n (128) x 8 vectors of 8 k
#pragma unroll
            for (int v = 0; v < 8; ++v) {
                const int idx = tid + v * Cfg::THREADS;
                const int nr = idx >> 3, kv = (idx & 7) * 8;
                const int k = k0 + kv, n = n0 + nr;
                const int bytes = (n < p.N && k < k_end) ? min(16, (k_end - k) * 2) : 0;
                const __half* src = p.B + (bytes ? int64_t(n) * p.sBn + k : 0);
                cp_async16(&sB[buf * B_EL + nr * LDK + kv], src, bytes);
            }
        }
    };

#pragma unroll
    for (int st = 0; st < STAGES - 1; ++st) {
        if (st < nst) load_stage(st);
        cp_async_commit();
    }
    for (int kb = 0; kb < nst; ++kb) {
        cp_async_wait<STAGES - 2>();
        __syncthreads();  // stage kb landed for everyone; stage kb-1's buffer is free
        if (kb + STAGES - 1 < nst) load_stage(kb + STAGES - 1);
        cp_async_commit();
        const int buf = kb % STAGES;
        const __half* a_s = sA + buf * A_EL;
        const __half* b_s = sB + buf * B_EL;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            const int ck = k_begin + kb * BK + c * 32;  // absolute K offset of this chunk
            if (ck >= k_end) break;
            uint32_t hacc[MT][4][2];
            if constexpr (CHUNKED) {
#pragma unroll
                for (int i = 0; i < MT; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) hacc[i][j][0] = hacc[i][j][1] = 0u;
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                if (ck + h * 16 >= k_end) break;  // a K16 step wholly past the range adds nothing
                const int kk = c * 32 + h * 16;   // within the stage
                uint32_t af[MT][4], bf[4][2];
#pragma unroll
                for (int i = 0; i < MT; ++i) {
                    const __half* src = a_s + (i * 16 + (lane & 15)) * LDK + kk + (lane >> 4) * 8;
                    ldsm_x4(smem_u32(src), af[i][0], af[i][1], af[i][2], af[i][3]);
                }
#pragma unroll
                for (int jp = 0; jp < 2; ++jp) {
                    if constexpr (B_KN) {
                        const __half* src =
                            b_s + (kk + ((lane >> 3) & 1) * 8 + (lane & 7)) * LDN + warp * 32 + jp * 16 + (lane >> 4) * 8;
                        ldsm_x4_t(smem_u32(src), bf[2 * jp][0], bf[2 * jp][1], bf[2 * jp + 1][0], bf[2 * jp + 1][1]);
                    } else {
                        const __half* src =
                            b_s + (warp * 32 + jp * 16 + (lane >> 4) * 8 + (lane & 7)) * LDK + kk + ((lane >> 3) & 1) * 8;
                        ldsm_x4(smem_u32(src), bf[2 * jp][0], bf[2 * jp][1], bf[2 * jp + 1][0], bf[2 * jp + 1][1]);
                    }
                }
#pragma unroll
                for (int i = 0; i < MT; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        if constexpr (CHUNKED) mma_f16acc(hacc[i][j], af[i], bf[j][0], bf[j][1]);
                        else mma_f32acc(acc[i][j], af[i], bf[j][0], bf[j][1]);
                    }
            }
            if constexpr (CHUNKED) {
#pragma unroll
                for (int i = 0; i < MT; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        add_f16x2_to_f32(acc[i][j][0], acc[i][j][1], hacc[i][j][0]);
                        add_f16x2_to_f32(acc[i][j][2], acc[i][j][3], hacc[i][j][1]);
                    }
            }
        }
    }
    cp_async_wait<0>();
    __syncthreads();
}

// acc[i][j][v] holds row i*16 + g (+8 for v >= 2), column warp*32 + j*8 + 2*tq (+1 for odd v).
template <int MT>
__device__ __forceinline__ void skinny_store_partial(float* red, const float (&acc)[MT][4][4]) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3;
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int hr = 0; hr < 2; ++hr) {
                const int r = i * 16 + g + hr * 8, c = warp * 32 + j * 8 + 2 * tq;
                *reinterpret_cast<float2*>(&red[r * SkinnyCfg::RED_LD + c]) =
                    make_float2(acc[i][j][2 * hr], acc[i][j][2 * hr + 1]);
            }
}

// Every CTA of the cluster reduces its share of the tile, four columns at a
// time: sum = partial 0 + partial 1 + ... in that order (all S loads issued
// before the adds), then stores it to C with the optional bias.  Returns
// whether this CTA saw a non-finite sum.
template <int MT, int OUT>
__device__ __forceinline__ bool skinny_reduce_store(cooperative_groups::cluster_group& cluster, const float* red,
                                                    int S, int rank, const SkinnyParams& p, int n0) {
    using Cfg = SkinnyCfg;
    using Tr = OutTraits<OUT>;
    using T = typename Tr::T;
    constexpr int NV = 16 * MT * (Cfg::BN / 4);  // float4s in the tile
    const float* parts[Cfg::MAX_S];
#pragma unroll
    for (int q = 0; q < Cfg::MAX_S; ++q) parts[q] = cluster.map_shared_rank(red, q < S ? q : 0);
    T* C = reinterpret_cast<T*>(p.C);
    float z = 0.0f;
    for (int v = rank * Cfg::THREADS + int(threadIdx.x); v < NV; v += S * Cfg::THREADS) {
        const int r = v / (Cfg::BN / 4), c = (v % (Cfg::BN / 4)) * 4;
        float4 x[Cfg::MAX_S];
#pragma unroll
        for (int q = 0; q < Cfg::MAX_S; ++q)
            if (q < S) x[q] = *reinterpret_cast<const float4*>(parts[q] + r * Cfg::RED_LD + c);
        float4 s = x[0];
#pragma unroll
        for (int q = 1; q < Cfg::MAX_S; ++q)
            if (q < S) {
                s.x += x[q].x;
                s.y += x[q].y;
                s.z += x[q].z;
                s.w += x[q].w;
            }
        z = nonfinite_probe(nonfinite_probe(nonfinite_probe(nonfinite_probe(z, s.x), s.y), s.z), s.w);
        if (r >= p.M) continue;
        float o[4] = {s.x, s.y, s.z, s.w};
        const int col = n0 + c;
        T* crow = C + int64_t(r) * p.sCm;
#pragma unroll
        for (int e = 0; e < 4; ++e)
            if (p.bias != nullptr && col + e < p.N)  // the reference adds the bias after the product (and its flag)
                o[e] = add_bias<OUT>(o[e], p.bias, p.sbias, col + e);
        if (p.c_vec && col + 4 <= p.N) {
            if constexpr (OUT == kOutF32) {
                *reinterpret_cast<float4*>(crow + col) = make_float4(o[0], o[1], o[2], o[3]);
            } else if constexpr (OUT == kOutF16) {
                const __half2 h0 = __floats2half2_rn(o[0], o[1]), h1 = __floats2half2_rn(o[2], o[3]);
                *reinterpret_cast<uint2*>(crow + col) =
                    make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
            } else {
                const __nv_bfloat162 h0 = __floats2bfloat162_rn(o[0], o[1]), h1 = __floats2bfloat162_rn(o[2], o[3]);
                *reinterpret_cast<uint2*>(crow + col) =
                    make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
            }
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (col + e < p.N) crow[int64_t(col + e) * p.sCn] = Tr::cvt(o[e]);
        }
    }
    return z != z;
}

// grid (ceil(N / 128), S), cluster (1, S, 1).  REDO: the separate FP32 pass
// over flagged tiles (launched behind the chunked pass).
template <int MT, bool CHUNKED, bool B_KN, int OUT, bool REDO, bool SHALLOW>
__global__ void __launch_bounds__(SkinnyCfg::THREADS) skinny_gemm_kernel(const __grid_constant__ SkinnyParams p) {
    namespace cg = cooperative_groups;
    using Cfg = SkinnyCfg;
    static_assert(!(CHUNKED && REDO), "the redo pass runs in FP32 mode");
    extern __shared__ __align__(128) uint8_t skinny_smem[];
    __half* sA = reinterpret_cast<__half*>(skinny_smem);
    __half* sB = sA + Cfg::stages<MT, SHALLOW>() * Cfg::a_elems<MT>();
    float* red = reinterpret_cast<float*>(skinny_smem);  // the ring, reused once the main loop is done
    __shared__ int tile_bad;                            // OR over the cluster of "saw a non-finite sum"

    cg::cluster_group cluster = cg::this_cluster();
    const int S = int(cluster.dim_blocks().y);
    const int rank = int(cluster.block_rank());
    const int tile = blockIdx.x;
    const int n0 = tile * Cfg::BN;
    const int k_begin = rank * p.kper;
    const int k_end = min(p.K, k_begin + p.kper);

    // Programmatic dependent launch (as every GEMM kernel here): nothing above
    // touches global memory; the wait returns once the previous kernel on the
    // stream (for the redo pass: the chunked pass, its flags and C) is complete.
    grid_dep_wait();
    if constexpr (REDO) {
        if (!tile_flagged(p.flags, tile)) return;  // every CTA of the cluster reads the same flag
    } else {
        grid_dep_launch();
    }
    if (threadIdx.x == 0) tile_bad = 0;  // before the first cluster barrier: peers OR into it after

    float acc[MT][4][4];
    skinny_mainloop<MT, CHUNKED, B_KN, SHALLOW>(p, sA, sB, n0, k_begin, k_end, acc);
    skinny_store_partial<MT>(red, acc);
    cluster.sync();  // every partial tile is in its CTA's shared memory
    const bool bad = skinny_reduce_store<MT, OUT>(cluster, red, S, rank, p, n0);
    if constexpr (CHUNKED) {
        if (__syncthreads_or(bad) && threadIdx.x == 0)
            for (int q = 0; q < S; ++q) atomicOr(cluster.map_shared_rank(&tile_bad, q), 1);
    }
    cluster.sync();  // every read of a peer's partials is done; tile_bad is the cluster's OR
    if constexpr (CHUNKED) {
        if (rank == 0 && threadIdx.x == 0)
            *reinterpret_cast<uint4*>(p.flags + int64_t(tile) * kFlagBytesPerTile) =
                make_uint4(tile_bad ? 1u : 0u, 0u, 0u, 0u);
        if (!(p.inline_redo && tile_bad)) return;
        // The flagged tile again in FP32 mode: the FP32 kernel's loop and summation order.
        skinny_mainloop<MT, false, B_KN, SHALLOW>(p, sA, sB, n0, k_begin, k_end, acc);
        skinny_store_partial<MT>(red, acc);
        cluster.sync();
        skinny_reduce_store<MT, OUT>(cluster, red, S, rank, p, n0);
        cluster.sync();
    }
}

}  // namespace f16acc
