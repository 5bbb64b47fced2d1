// mma_gemm.cuh -- warp-level mma.sync variant of the chunked GEMM: register
// accumulators, any operand strides.  It is the path for operands the TMA
// kernel cannot take (unaligned rows, non-unit inner strides, odd K such as
// 777) and the warp-level variant measured against the tcgen05 kernel.
//
// Reference semantics (steppergg/f16acc f16acc/kernel.py:37-81): 32-long K
// chunks from absolute offset 0, each accumulated in FP16 by two m16n8k16
// MMAs (FP16 C/D), converted and added into FP32 registers; FP32 mode runs
// the same loop with FP32 C/D; per-tile non-finite flag; redo in FP32 mode.
//
// CTA tile 128 x 128, one 32-long chunk per K step, 8 warps as 2 (M) x 4 (N),
// warp tile 64 x 32.  Operands are staged global -> registers -> shared memory
// (double buffered), so the same loop serves every stride pattern; only the
// global load differs (16-byte vectors when the inner stride is 1 and rows
// are aligned, element loads otherwise).
#pragma once

#include "common.cuh"
#include "ptx.cuh"

namespace f16acc {

struct MmaParams {
    const __half* A;
    const __half* B;
    void* C;
    int64_t sAm, sAk, sBk, sBn, sCm, sCn;
    int M, N, K;
    int tiles_m, tiles_n;
    int group_m;
    int c_vec;  // C has unit column stride and 4-byte aligned pairs
    uint8_t* flags;
    const __half* bias;  // optional per-column bias (element stride sbias), added before the cast
    int64_t sbias;
};

// Operand load modes.
enum LoadMode : int {
    kLoadGeneric = 0,  // element loads, any strides
    kLoadKVec = 1,     // K-contiguous, 16-byte vectors along K
    kLoadNVec = 2,     // (B only) N-contiguous, 16-byte vectors along N
};

struct MmaCfg {
    static constexpr int BM = 128, BN = 128, BK = 32;
    static constexpr int THREADS = 256;
    static constexpr int LDK = BK + 8;   // [row][k] smem row pitch (halves): conflict-free ldmatrix
    static constexpr int LDN = BN + 8;   // [k][n] smem row pitch (halves)
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void mma_f16acc(uint32_t (&d)[2], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f16.f16.f16.f16 {%0,%1}, {%2,%3,%4,%5}, {%6,%7}, {%0,%1};"
                 : "+r"(d[0]), "+r"(d[1])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_f32acc(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 8 consecutive f16 of a K-contiguous (or N-contiguous) row, masked past `lim`.
// `vec` = the 8 elements are 16-byte aligned in global memory.
__device__ __forceinline__ uint4 load8(const __half* base, int64_t stride, int first, int lim, bool vec) {
    if (vec && first + 8 <= lim) return __ldg(reinterpret_cast<const uint4*>(base + first));
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int e0 = first + 2 * i, e1 = e0 + 1;
        const unsigned short lo = e0 < lim ? __ldg(reinterpret_cast<const unsigned short*>(base + int64_t(e0) * stride)) : 0;
        const unsigned short hi = e1 < lim ? __ldg(reinterpret_cast<const unsigned short*>(base + int64_t(e1) * stride)) : 0;
        w[i] = uint32_t(lo) | (uint32_t(hi) << 16);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

template <bool CHUNKED, int A_MODE, int B_MODE, int OUT, bool REDO>
__global__ void __launch_bounds__(MmaCfg::THREADS) mma_gemm_kernel(const __grid_constant__ MmaParams p) {
    using Cfg = MmaCfg;
    constexpr int BM = Cfg::BM, BN = Cfg::BN, BK = Cfg::BK, LDK = Cfg::LDK, LDN = Cfg::LDN;
    constexpr bool B_KN = (B_MODE == kLoadNVec);  // B staged as [k][n] and read with ldmatrix.trans
    constexpr int B_ELEMS = B_KN ? BK * LDN : BN * LDK;
    static_assert(!(CHUNKED && REDO), "the redo pass runs in FP32 mode");

    __shared__ __align__(128) __half sA[2][BM * LDK];
    __shared__ __align__(128) __half sB[2][B_ELEMS];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wm = warp >> 2, wn = warp & 3;  // warp tile origin: rows wm*64, cols wn*32
    const int g = lane >> 2, tq = lane & 3;   // mma fragment coordinates

    // programmatic dependent launch: nothing above touches global memory
    grid_dep_wait();
    if constexpr (!REDO) grid_dep_launch();

    const int tiles = p.tiles_m * p.tiles_n;
    const int nkt = (p.K + BK - 1) / BK;  // one chunk per K step

    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
        int tm, tn;
        raster(t, p.tiles_m, p.tiles_n, p.group_m, tm, tn);
        const int64_t tile_id = int64_t(tm) * p.tiles_n + tn;
        if (REDO && !tile_flagged(p.flags, tile_id)) continue;

        // Per-thread share of one K step: A row ar, k [ak0, ak0+16); B either
        // column bn / k [bk0, bk0+16) ([n][k] staging) or k row bkr / n [bn0, bn0+16).
        const int ar = tid >> 1, ak0 = (tid & 1) * 16;
        const int a_row = tm * BM + ar;
        const bool a_in = a_row < p.M;
        const __half* a_ptr = p.A + int64_t(a_in ? a_row : 0) * p.sAm;
        const int bcol = tid >> 1, bk0 = (tid & 1) * 16;   // [n][k] staging
        const int bkr = tid >> 3, bn0 = (tid & 7) * 16;    // [k][n] staging
        const int b_col = tn * BN + bcol;
        const bool b_in = b_col < p.N;
        const __half* b_ptr_n = p.B + int64_t(b_in ? b_col : 0) * p.sBn;

        uint4 ra[2], rb[2];
        auto gload = [&](int kt) {
            const int k0 = kt * BK;
            if (a_in) {
#pragma unroll
                for (int v = 0; v < 2; ++v)
                    ra[v] = load8(a_ptr, p.sAk, k0 + ak0 + 8 * v, p.K, A_MODE == kLoadKVec);
            } else {
                ra[0] = ra[1] = make_uint4(0, 0, 0, 0);
            }
            if constexpr (B_KN) {
                const int k = k0 + bkr;
                if (k < p.K) {
                    const __half* row = p.B + int64_t(k) * p.sBk;
#pragma unroll
                    for (int v = 0; v < 2; ++v) rb[v] = load8(row, p.sBn, tn * BN + bn0 + 8 * v, p.N, true);
                } else {
                    rb[0] = rb[1] = make_uint4(0, 0, 0, 0);
                }
            } else {
                if (b_in) {
#pragma unroll
                    for (int v = 0; v < 2; ++v) rb[v] = load8(b_ptr_n, p.sBk, k0 + bk0 + 8 * v, p.K, B_MODE == kLoadKVec);
                } else {
                    rb[0] = rb[1] = make_uint4(0, 0, 0, 0);
                }
            }
        };
        auto sstore = [&](int buf) {
            *reinterpret_cast<uint4*>(&sA[buf][ar * LDK + ak0]) = ra[0];
            *reinterpret_cast<uint4*>(&sA[buf][ar * LDK + ak0 + 8]) = ra[1];
            if constexpr (B_KN) {
                *reinterpret_cast<uint4*>(&sB[buf][bkr * LDN + bn0]) = rb[0];
                *reinterpret_cast<uint4*>(&sB[buf][bkr * LDN + bn0 + 8]) = rb[1];
            } else {
                *reinterpret_cast<uint4*>(&sB[buf][bcol * LDK + bk0]) = rb[0];
                *reinterpret_cast<uint4*>(&sB[buf][bcol * LDK + bk0 + 8]) = rb[1];
            }
        };

        float acc[4][4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int v = 0; v < 4; ++v) acc[i][j][v] = 0.0f;

        __syncthreads();  // previous tile's readers are done with both buffers
        if (nkt > 0) {
            gload(0);
            sstore(0);
        }
        __syncthreads();
        for (int kt = 0; kt < nkt; ++kt) {
            const int cur = kt & 1;
            if (kt + 1 < nkt) gload(kt + 1);
            uint32_t hacc[4][4][2];
            if constexpr (CHUNKED) {
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) hacc[i][j][0] = hacc[i][j][1] = 0u;
            }
#pragma unroll
            for (int ks = 0; ks < 2; ++ks) {
                if (kt * BK + ks * 16 >= p.K) break;  // a K16 step wholly past the end adds nothing
                uint32_t af[4][4], bf[4][2];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const __half* src = &sA[cur][(wm * 64 + i * 16 + (lane & 15)) * LDK + ks * 16 + (lane >> 4) * 8];
                    ldsm_x4(smem_u32(src), af[i][0], af[i][1], af[i][2], af[i][3]);
                }
#pragma unroll
                for (int jp = 0; jp < 2; ++jp) {
                    if constexpr (B_KN) {
                        const __half* src = &sB[cur][(ks * 16 + ((lane >> 3) & 1) * 8 + (lane & 7)) * LDN + wn * 32 +
                                                     jp * 16 + (lane >> 4) * 8];
                        ldsm_x4_t(smem_u32(src), bf[2 * jp][0], bf[2 * jp][1], bf[2 * jp + 1][0], bf[2 * jp + 1][1]);
                    } else {
                        const __half* src = &sB[cur][(wn * 32 + jp * 16 + (lane >> 4) * 8 + (lane & 7)) * LDK + ks * 16 +
                                                     ((lane >> 3) & 1) * 8];
                        ldsm_x4(smem_u32(src), bf[2 * jp][0], bf[2 * jp][1], bf[2 * jp + 1][0], bf[2 * jp + 1][1]);
                    }
                }
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        if constexpr (CHUNKED) mma_f16acc(hacc[i][j], af[i], bf[j][0], bf[j][1]);
                        else mma_f32acc(acc[i][j], af[i], bf[j][0], bf[j][1]);
                    }
            }
            if constexpr (CHUNKED) {
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        add_f16x2_to_f32(acc[i][j][0], acc[i][j][1], hacc[i][j][0]);
                        add_f16x2_to_f32(acc[i][j][2], acc[i][j][3], hacc[i][j][1]);
                    }
            }
            if (kt + 1 < nkt) sstore(cur ^ 1);
            __syncthreads();
        }

        if constexpr (CHUNKED) {
            float z = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j)
#pragma unroll
                    for (int v = 0; v < 4; ++v) z = nonfinite_probe(z, acc[i][j][v]);
            const bool bad = __any_sync(0xffffffffu, z != z);
            if (lane == 0) *reinterpret_cast<uint16_t*>(p.flags + tile_id * kFlagBytesPerTile + 2 * warp) = bad ? 1 : 0;
        }

        if (p.bias != nullptr) {  // after the flag, as the reference adds it outside the kernel
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int col = tn * BN + wn * 32 + j * 8 + 2 * tq;
                if (col < p.N) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        acc[i][j][0] = add_bias<OUT>(acc[i][j][0], p.bias, p.sbias, col);
                        acc[i][j][2] = add_bias<OUT>(acc[i][j][2], p.bias, p.sbias, col);
                    }
                }
                if (col + 1 < p.N) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        acc[i][j][1] = add_bias<OUT>(acc[i][j][1], p.bias, p.sbias, col + 1);
                        acc[i][j][3] = add_bias<OUT>(acc[i][j][3], p.bias, p.sbias, col + 1);
                    }
                }
            }
        }
        // Store: acc[i][j] = rows r0 (v 0,1) and r0+8 (v 2,3), columns c, c+1.
        using Tr = OutTraits<OUT>;
        using T = typename Tr::T;
        T* C = reinterpret_cast<T*>(p.C);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
            for (int hrow = 0; hrow < 2; ++hrow) {
                const int row = tm * BM + wm * 64 + i * 16 + g + hrow * 8;
                if (row >= p.M) continue;
                T* crow = C + int64_t(row) * p.sCm;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int col = tn * BN + wn * 32 + j * 8 + 2 * tq;
                    const float v0 = acc[i][j][2 * hrow], v1 = acc[i][j][2 * hrow + 1];
                    if (p.c_vec && col + 1 < p.N) {
                        if constexpr (OUT == kOutF32) {
                            *reinterpret_cast<float2*>(crow + col) = make_float2(v0, v1);
                        } else if constexpr (OUT == kOutF16) {
                            *reinterpret_cast<__half2*>(crow + col) = __floats2half2_rn(v0, v1);
                        } else {
                            *reinterpret_cast<__nv_bfloat162*>(crow + col) = __floats2bfloat162_rn(v0, v1);
                        }
                    } else {
                        if (col < p.N) crow[int64_t(col) * p.sCn] = Tr::cvt(v0);
                        if (col + 1 < p.N) crow[int64_t(col + 1) * p.sCn] = Tr::cvt(v1);
                    }
                }
            }
        }
    }
}

// C = 0 (or the bias broadcast over rows) for K == 0, an empty sum; any strides.
template <int OUT>
__global__ void fill_zero_kernel(void* C, int64_t sCm, int64_t sCn, int M, int N, const __half* bias, int64_t sbias) {
    using T = typename OutTraits<OUT>::T;
    T* c = reinterpret_cast<T*>(C);
    const int64_t total = int64_t(M) * N;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = i / N, col = i - r * N;
        const float v = bias != nullptr ? __half2float(bias[col * sbias]) : 0.0f;  // K = 0: empty sum, plus the bias
        c[r * sCm + col * sCn] = OutTraits<OUT>::cvt(v);
    }
}

}  // namespace f16acc
