// common.cuh -- pieces shared by the tcgen05 and mma.sync GEMM kernels:
// tile raster, output-row stores, flag layout.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace f16acc {

// Output element types (the C-ABI's c_dtype).
enum OutType : int { kOutF16 = 0, kOutF32 = 1, kOutBF16 = 2 };

// Every tile owns kFlagBytesPerTile bytes of the flag area: one slot per
// epilogue warp, each written on every chunked pass whether or not the tile
// overflowed, so the area never needs clearing.  The tile is flagged when any
// byte of its slot is non-zero.  Tiles are numbered row-major over the tile
// grid (tile_m * tiles_n + tile_n), independent of the raster order.
constexpr int kFlagBytesPerTile = 16;

// Most peer outputs a fused GEMM + all-gather call stores to (8 GPUs per node).
constexpr int kMaxPeers = 7;

// Grouped raster: `group_m` consecutive tile rows are walked column by column,
// so the CTAs that run at the same time share A row-panels and B column-panels
// in L2.  Maps the linear schedule index t to (tile_m, tile_n).
__device__ __forceinline__ void raster(int t, int tiles_m, int tiles_n, int group_m, int& tm, int& tn) {
    const int per_group = group_m * tiles_n;
    const int g = t / per_group;
    const int first = g * group_m;
    const int rows = min(tiles_m - first, group_m);
    const int r = t - g * per_group;
    tm = first + r % rows;
    tn = r / rows;
}

__device__ __forceinline__ bool tile_flagged(const uint8_t* flags, int64_t tile) {
    // .cg: read at L2, where the previous kernel on the stream left the flags.
    const uint4 v = __ldcg(reinterpret_cast<const uint4*>(flags + tile * kFlagBytesPerTile));
    return (v.x | v.y | v.z | v.w) != 0u;
}

template <int OUT>
struct OutTraits;
template <>
struct OutTraits<kOutF16> {
    using T = __half;
    static constexpr int kVec = 8;  // elements per 16-byte store
    __device__ static T cvt(float x) { return __float2half_rn(x); }
};
template <>
struct OutTraits<kOutBF16> {
    using T = __nv_bfloat16;
    static constexpr int kVec = 8;
    __device__ static T cvt(float x) { return __float2bfloat16_rn(x); }
};
template <>
struct OutTraits<kOutF32> {
    using T = float;
    static constexpr int kVec = 4;
    __device__ static T cvt(float x) { return x; }
};

// 16 bytes of output built from kVec consecutive accumulators.
template <int OUT>
__device__ __forceinline__ uint4 pack16(const float* v) {
    uint4 u;
    if constexpr (OUT == kOutF32) {
        u.x = __float_as_uint(v[0]);
        u.y = __float_as_uint(v[1]);
        u.z = __float_as_uint(v[2]);
        u.w = __float_as_uint(v[3]);
    } else if constexpr (OUT == kOutF16) {
        __half2 h0 = __floats2half2_rn(v[0], v[1]), h1 = __floats2half2_rn(v[2], v[3]);
        __half2 h2 = __floats2half2_rn(v[4], v[5]), h3 = __floats2half2_rn(v[6], v[7]);
        u.x = *reinterpret_cast<uint32_t*>(&h0);
        u.y = *reinterpret_cast<uint32_t*>(&h1);
        u.z = *reinterpret_cast<uint32_t*>(&h2);
        u.w = *reinterpret_cast<uint32_t*>(&h3);
    } else {
        __nv_bfloat162 h0 = __floats2bfloat162_rn(v[0], v[1]), h1 = __floats2bfloat162_rn(v[2], v[3]);
        __nv_bfloat162 h2 = __floats2bfloat162_rn(v[4], v[5]), h3 = __floats2bfloat162_rn(v[6], v[7]);
        u.x = *reinterpret_cast<uint32_t*>(&h0);
        u.y = *reinterpret_cast<uint32_t*>(&h1);
        u.z = *reinterpret_cast<uint32_t*>(&h2);
        u.w = *reinterpret_cast<uint32_t*>(&h3);
    }
    return u;
}

// Store CW consecutive accumulators of one output row, columns [col0, col0+CW).
// `vec` = C has unit column stride and 16-byte aligned rows, so full 16-byte
// groups go out as vector stores; everything else is element by element with
// bounds checks.  64-bit offsets throughout (outputs past 2^31 elements).
template <int OUT, int CW>
__device__ __forceinline__ void store_row(void* C, int64_t sCm, int64_t sCn, int row, int col0, int M, int N,
                                          const float (&acc)[CW], bool vec) {
    using Tr = OutTraits<OUT>;
    using T = typename Tr::T;
    if (row >= M) return;
    T* crow = reinterpret_cast<T*>(C) + static_cast<int64_t>(row) * sCm;
    if (vec && col0 + CW <= N) {
#pragma unroll
        for (int j = 0; j < CW; j += Tr::kVec) {
            *reinterpret_cast<uint4*>(crow + col0 + j) = pack16<OUT>(&acc[j]);
        }
        return;
    }
#pragma unroll
    for (int j = 0; j < CW; ++j) {
        const int col = col0 + j;
        if (col < N) crow[static_cast<int64_t>(col) * sCn] = Tr::cvt(acc[j]);
    }
}

}  // namespace f16acc
