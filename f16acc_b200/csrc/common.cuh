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
    __device__ static float round_trip(float x) { return __half2float(__float2half_rn(x)); }
    __device__ static float to_float(T x) { return __half2float(x); }
};
template <>
struct OutTraits<kOutBF16> {
    using T = __nv_bfloat16;
    static constexpr int kVec = 8;
    __device__ static T cvt(float x) { return __float2bfloat16_rn(x); }
    __device__ static float round_trip(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
    __device__ static float to_float(T x) { return __bfloat162float(x); }
};
template <>
struct OutTraits<kOutF32> {
    using T = float;
    static constexpr int kVec = 4;
    __device__ static T cvt(float x) { return x; }
    __device__ static float round_trip(float x) { return x; }
    __device__ static float to_float(T x) { return x; }
};

// Bias epilogue: the product is rounded to the output type first and the bias
// added to that value, so C = cvt(cvt(A@B) + bias) is bit-identical to the
// reference's unfused `y = mm(x, w.t()); y += b` (patch.py:28-30), whose
// in-place half add computes in FP32 and rounds once.
template <int OUT>
__device__ __forceinline__ float add_bias(float acc, const __half* bias, int64_t sbias, int col) {
    return OutTraits<OUT>::round_trip(acc) + __half2float(bias[int64_t(col) * sbias]);
}

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

// add_bias over 16 bytes of output already rounded to OUT (columns col ..
// col + kVec - 1; the ones at or past N are left as they are).
template <int OUT>
__device__ __forceinline__ uint4 add_bias16(uint4 u, const __half* bias, int64_t sbias, int col, int N) {
    constexpr int kVec = OutTraits<OUT>::kVec;
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    float f[kVec];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if constexpr (OUT == kOutF32) {
            f[i] = __uint_as_float(w[i]);
        } else if constexpr (OUT == kOutF16) {
            const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
            f[2 * i] = t.x;
            f[2 * i + 1] = t.y;
        } else {
            const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
            f[2 * i] = t.x;
            f[2 * i + 1] = t.y;
        }
    }
#pragma unroll
    for (int t = 0; t < kVec; ++t)
        if (col + t < N) f[t] += __half2float(bias[int64_t(col + t) * sbias]);
    return pack16<OUT>(f);
}

}  // namespace f16acc
