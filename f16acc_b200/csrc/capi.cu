// capi.cu -- the C ABI declared in include/f16acc.h: argument checks, kernel
// choice, TMA descriptors, and the main + redo launches on the caller's stream.
//
// Reference host logic (steppergg/f16acc f16acc/kernel.py:84-105): checks
// (:87-90), output and flag buffers (:93-95), 64-bit indexing (:97-98 -- here
// always 64-bit address arithmetic, TMA coordinates are 32-bit per dimension),
// main launch (:99), redo launch on the same stream with no host sync
// (:100-104).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <atomic>
#include <mutex>

#include "../../include/f16acc.h"
#include "launch.h"
#include "mma_gemm.cuh"
#include "skinny_gemm.cuh"
#include "tc_gemm.cuh"

namespace f16acc {

// Device status word: kernels record the first wait they gave up on here.
__device__ int g_status = 0;

namespace {

constexpr int kMaxDevices = 64;

struct DeviceInfo {
    std::once_flag once;
    cudaError_t err = cudaSuccess;
    int sms = 0;
    int* status = nullptr;
};
DeviceInfo g_dev[kMaxDevices];

// Per-device facts, looked up once.  The status word's address is resolved
// with `device` current (cudaGetSymbolAddress answers for the current
// device), whatever device the calling thread had selected; the caller's
// device is restored afterwards.  nullptr for an ordinal that is not a
// device of this process.
DeviceInfo* device_info(int device) {
    if (device < 0 || device >= kMaxDevices) return nullptr;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device >= count) return nullptr;
    DeviceInfo* d = &g_dev[device];
    std::call_once(d->once, [d, device]() {
        d->err = cudaDeviceGetAttribute(&d->sms, cudaDevAttrMultiProcessorCount, device);
        if (d->err != cudaSuccess) return;
        int prev = -1;
        d->err = cudaGetDevice(&prev);
        if (d->err != cudaSuccess) return;
        if (prev != device && (d->err = cudaSetDevice(device)) != cudaSuccess) return;
        d->err = cudaGetSymbolAddress(reinterpret_cast<void**>(&d->status), g_status);
        if (prev != device) {
            const cudaError_t back = cudaSetDevice(prev);
            if (d->err == cudaSuccess) d->err = back;
        }
    });
    return d;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
std::once_flag g_encode_once;
EncodeTiledFn g_encode = nullptr;

EncodeTiledFn encode_fn() {
    std::call_once(g_encode_once, []() {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    });
    return g_encode;
}

// 2-D tensor map (FP16 unless `dtype` says otherwise): inner dimension d0
// (contiguous), outer d1 with byte stride stride1, box {b0, b1}, 128-byte
// swizzle, zero fill out of bounds.
bool make_map(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint64_t stride1_bytes, uint32_t b0,
              uint32_t b1, CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_FLOAT16) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {d0, d1};
    const cuuint64_t strides[1] = {stride1_bytes};
    const cuuint32_t box[2] = {b0, b1};
    const cuuint32_t estr[2] = {1, 1};
    return enc(m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Operand layout facts the kernel choice needs.  Strides of size-1 dimensions
// carry no information and are replaced by the natural ones.
struct Layout {
    int64_t sAm, sAk, sBk, sBn;
    bool a_kcontig, a_tma, b_kcontig, b_ncontig, b_tma_k, b_tma_n;
    bool a_vec, b_kvec, b_nvec;
};

Layout analyse(const void* A, int64_t sAm, int64_t sAk, const void* B, int64_t sBk, int64_t sBn, int64_t M, int64_t N,
               int64_t K) {
    Layout L{};
    if (K == 1) sAk = 1;
    if (M == 1) sAm = K;
    if (K == 1) sBk = N;
    if (N == 1) sBn = 1;
    // N == 1 and K == 1 together: B is one element; either view works.
    L.sAm = sAm; L.sAk = sAk; L.sBk = sBk; L.sBn = sBn;
    const uintptr_t pa = reinterpret_cast<uintptr_t>(A), pb = reinterpret_cast<uintptr_t>(B);
    L.a_kcontig = sAk == 1;
    L.b_kcontig = sBk == 1;
    L.b_ncontig = sBn == 1;
    const bool a16 = pa % 16 == 0, b16 = pb % 16 == 0;
    const uint64_t max_stride = uint64_t(1) << 39;  // TMA byte strides must stay below 2^40
    L.a_tma = L.a_kcontig && a16 && sAm % 8 == 0 && sAm >= K && uint64_t(sAm) < max_stride;
    L.b_tma_k = L.b_kcontig && b16 && sBn % 8 == 0 && sBn >= K && uint64_t(sBn) < max_stride;
    L.b_tma_n = L.b_ncontig && b16 && sBk % 8 == 0 && sBk >= N && uint64_t(sBk) < max_stride;
    L.a_vec = L.a_kcontig && a16 && sAm % 8 == 0;
    L.b_kvec = L.b_kcontig && b16 && sBn % 8 == 0;
    L.b_nvec = L.b_ncontig && b16 && sBk % 8 == 0;
    return L;
}

// tcgen05 tile configuration: output columns per tile and epilogue column
// slices per TMEM lane quarter (0 = by mode: 2 for the chunked kernel, whose
// shorter release rounds with 8 epilogue warps measured faster, 4 for FP32
// accumulation).  Process-wide; f16acc_set_tc_config changes it (tuning and
// measurement), calls already issued keep theirs.
std::atomic<int> g_tc_bn{128}, g_tc_epi{0};

// Upper bound on the SMs a persistent launch may occupy (0 = all).  Leaving a
// few SMs free lets kernels on other streams -- NCCL collectives overlapping a
// sharded product -- run alongside instead of queueing behind the GEMM.
std::atomic<int> g_sm_limit{0};
int usable_sms(int sms) {
    const int lim = g_sm_limit.load(std::memory_order_relaxed);
    return lim > 0 && lim < sms ? lim : sms;
}
TcShape tc_shape(bool chunked) {
    const int epi = g_tc_epi.load(std::memory_order_relaxed);
    return TcShape{g_tc_bn.load(std::memory_order_relaxed), epi != 0 ? epi : (chunked ? 2 : 4)};
}

// Where flagged tiles of a chunked tcgen05 call are redone: 1 = inside the main
// kernel, each CTA after its own main tiles; 0 = a second, dependent launch.
std::atomic<int> g_redo_mode{F16ACC_REDO_INLINE};

// Tile order of the chunked main pass (F16ACC_SCHEDULE_*).
std::atomic<int> g_schedule{F16ACC_SCHEDULE_DYNAMIC};

// Tile width of FP32-mode calls (F16ACC_FP32_TILES_*).
std::atomic<int> g_fp32_tiles{F16ACC_FP32_TILES_AUTO};
constexpr int kGroupM = 8;

// Tail split of the chunked tcgen05 main pass (F16ACC_TAIL_SPLIT_*).  The
// tiles past the last full wave of the SMs (all of them when there are fewer
// tiles than SMs) run as S units over contiguous shares of K: S = the units
// that still fit beside each other on the SMs, at most kSplitMax, each unit at
// least kSplitMinStages 64-wide stages.  A split costs about 6-8 us on the
// critical path (the counter reset, each unit's pipeline fill and partial
// write, the last unit's read-back), measured on shapes from 1024^3 to the
// Qwen projections, against about 0.39 us per 64-wide stage it takes off a
// tile; so it is used only when it takes at least kSplitMinSaved stages off
// (measured break-even: 16-18 stages lose about 1 us, 22-24 gain 2).
std::atomic<int> g_tail_split{F16ACC_TAIL_SPLIT_ON};
constexpr int64_t kSplitMax = 4;
constexpr int64_t kSplitMinStages = 6;
constexpr int64_t kSplitMinSaved = 20;
constexpr int64_t kSplitSlots = 148;  // partial tiles at most: S x split tiles <= SMs
constexpr int64_t kSplitPartialBytes = 128 * 128 * 4;

struct TailSplit {
    int64_t s = 0, first = 0, tiles = 0;  // parts, first split tile, split tiles
};
TailSplit plan_split(int64_t tiles, int64_t K, int64_t sms) {
    TailSplit t;
    const int64_t nkb = cdiv(K, 64);
    const int64_t r = tiles < sms ? tiles : tiles % sms;
    if (r <= 0) return t;
    int64_t S = sms / r;
    if (S > kSplitMax) S = kSplitMax;
    if (S > nkb / kSplitMinStages) S = nkb / kSplitMinStages;
    if (S < 2 || S * r > kSplitSlots || nkb - nkb / S < kSplitMinSaved) return t;
    t.s = S;
    t.first = tiles - r;
    t.tiles = r;
    return t;
}
// Workspace layout: the flags (kFlagBytesPerTile a tile), then, when a tail
// split can happen, one counter per split tile and the partial tiles.
int64_t flag_area(int64_t M, int64_t N) { return cdiv(M, 128) * cdiv(N, 128) * kFlagBytesPerTile; }
int64_t split_counters_at(int64_t M, int64_t N) { return cdiv(flag_area(M, N), 256) * 256; }
int64_t split_partials_at(int64_t M, int64_t N) { return split_counters_at(M, N) + kSplitSlots * 4 + 512; }
bool split_possible(int64_t M, int64_t N, int64_t K) {
    const int64_t nkb = cdiv(K, 64);
    return M > 0 && N > 0 && nkb / kSplitMax >= kSplitMinStages && nkb - nkb / kSplitMax >= kSplitMinSaved;
}

// Rows up to which the few-row kernel is the automatic choice: 64, except
// for very wide products (lm_head-sized N), where at 64 rows the tcgen05
// kernel is faster (measured on the 1536 x 151936 weight: 110 against 148 us);
// there the few-row kernel is chosen up to 32 rows.
constexpr int64_t kSkinnyMaxRows = 64;
constexpr int64_t kSkinnyMaxRowsWide = 32;
constexpr int64_t kSkinnyWideN = 32768;

int choose_variant(const Layout& L, int64_t M, int64_t N, int64_t K, int requested, bool peers = false) {
    const bool dims_ok = M < (int64_t(1) << 31) && N < (int64_t(1) << 31) && K < (int64_t(1) << 31);
    const bool tc_ok = dims_ok && K > 0 && L.a_tma && (L.b_tma_k || L.b_tma_n) && encode_fn() != nullptr;
    // cp.async wants 16-byte aligned rows with unit inner stride; no peer stores
    const bool skinny_ok = dims_ok && K > 0 && M <= kSkinnyMaxRows && L.a_vec && (L.b_kvec || L.b_nvec) && !peers;
    const bool skinny_auto = skinny_ok && (M <= kSkinnyMaxRowsWide || N <= kSkinnyWideN);
    if (requested == F16ACC_VARIANT_TCGEN05) return tc_ok ? F16ACC_VARIANT_TCGEN05 : -1;
    if (requested == F16ACC_VARIANT_MMA_SYNC) return dims_ok ? F16ACC_VARIANT_MMA_SYNC : -1;
    if (requested == F16ACC_VARIANT_SKINNY) return skinny_ok ? F16ACC_VARIANT_SKINNY : -1;
    if (requested != F16ACC_VARIANT_AUTO) return -1;
    if (skinny_auto) return F16ACC_VARIANT_SKINNY;
    if (tc_ok) return F16ACC_VARIANT_TCGEN05;
    if (skinny_ok) return F16ACC_VARIANT_SKINNY;
    return dims_ok ? F16ACC_VARIANT_MMA_SYNC : -1;
}

// Which of the two launches run() makes: the main pass writes C and the
// flags, the redo pass recomputes flagged tiles (kernel.py:99 and :100-104).
constexpr int kPhaseMain = 1, kPhaseRedo = 2, kPhaseBoth = 3;

struct DeviceGuard {
    int prev = -1;
    bool switched = false;
    cudaError_t err = cudaSuccess;
    explicit DeviceGuard(int device) {
        err = cudaGetDevice(&prev);
        if (err == cudaSuccess && prev != device) {
            err = cudaSetDevice(device);
            switched = err == cudaSuccess;
        }
    }
    ~DeviceGuard() {
        if (switched) cudaSetDevice(prev);
    }
};

int run(const void* A, int64_t sAm, int64_t sAk, const void* B, int64_t sBk, int64_t sBn, void* C, int64_t sCm,
        int64_t sCn, int c_dtype, int64_t M, int64_t N, int64_t K, int chunked, void* workspace, size_t ws_bytes,
        int device, void* stream_ptr, int variant, int phases, void* const* peers = nullptr, int n_peers = 0,
        const void* bias = nullptr, int64_t sbias = 0) {
    if (n_peers < 0 || n_peers > kMaxPeers || (n_peers > 0 && peers == nullptr)) return F16ACC_ERR_INVALID_ARGUMENT;
    for (int i = 0; i < n_peers; ++i)
        if (peers[i] == nullptr) return F16ACC_ERR_INVALID_ARGUMENT;
    if (M < 0 || N < 0 || K < 0) return F16ACC_ERR_INVALID_ARGUMENT;
    if (c_dtype != F16ACC_OUT_F16 && c_dtype != F16ACC_OUT_F32 && c_dtype != F16ACC_OUT_BF16)
        return F16ACC_ERR_INVALID_ARGUMENT;
    if (M == 0 || N == 0) return F16ACC_OK;
    if (C == nullptr) return F16ACC_ERR_INVALID_ARGUMENT;
    if (M >= (int64_t(1) << 31) || N >= (int64_t(1) << 31) || K >= (int64_t(1) << 31))
        return F16ACC_ERR_INVALID_ARGUMENT;
    DeviceInfo* info = device_info(device);
    if (!info) return F16ACC_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess || info->err != cudaSuccess) return F16ACC_ERR_CUDA;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);

    if (K == 0) {  // empty sum: C = 0, nothing to flag
        if (!(phases & kPhaseMain)) return F16ACC_OK;
        return launch_fill_zero(C, sCm, sCn, int(M), int(N), c_dtype, stream, static_cast<const __half*>(bias),
                                sbias) == cudaSuccess
                   ? F16ACC_OK
                   : F16ACC_ERR_CUDA;
    }
    if (A == nullptr || B == nullptr) return F16ACC_ERR_INVALID_ARGUMENT;
    const Layout L = analyse(A, sAm, sAk, B, sBk, sBn, M, N, K);
    int v = choose_variant(L, M, N, K, variant, n_peers > 0);
    if (v < 0) return variant == F16ACC_VARIANT_AUTO ? F16ACC_ERR_INVALID_ARGUMENT : F16ACC_ERR_UNSUPPORTED;
    if (chunked) {
        // The flags must fit; the tail split's area is used only when it fits too.
        if (workspace == nullptr || ws_bytes < size_t(flag_area(M, N)) ||
            reinterpret_cast<uintptr_t>(workspace) % 16 != 0)
            return F16ACC_ERR_WORKSPACE;
    }
    const int esize = c_dtype == F16ACC_OUT_F32 ? 4 : 2;
    const uintptr_t pc = reinterpret_cast<uintptr_t>(C);

    if (v == F16ACC_VARIANT_SKINNY) {
        SkinnyParams s;
        std::memset(&s, 0, sizeof(s));
        s.A = static_cast<const __half*>(A);
        s.B = static_cast<const __half*>(B);
        s.C = C;
        s.sAm = L.sAm;
        s.sBk = L.sBk;
        s.sBn = L.sBn;
        s.sCm = sCm;
        s.sCn = sCn;
        s.M = int(M);
        s.N = int(N);
        s.K = int(K);
        int splits = 1, kper = 64;
        skinny_split(N, K, &splits, &kper);
        s.kper = kper;
        s.c_vec = (sCn == 1 && pc % (4 * esize) == 0 && sCm % 4 == 0) ? 1 : 0;
        s.flags = static_cast<uint8_t*>(workspace);
        s.bias = static_cast<const __half*>(bias);
        s.sbias = sbias;
        s.inline_redo = chunked && phases == kPhaseBoth &&
                        g_redo_mode.load(std::memory_order_relaxed) == F16ACC_REDO_INLINE;
        const bool b_kn = !L.b_kvec;  // N-contiguous B
        if ((phases & kPhaseMain) && launch_skinny(s, chunked != 0, b_kn, c_dtype, false, splits, stream) != cudaSuccess)
            return F16ACC_ERR_CUDA;
        if (chunked && (phases & kPhaseRedo) && !s.inline_redo &&
            launch_skinny(s, false, b_kn, c_dtype, true, splits, stream) != cudaSuccess)
            return F16ACC_ERR_CUDA;
        return F16ACC_OK;
    }

    TcParams p;
    std::memset(&p, 0, sizeof(p));
    const bool b_mn = !L.b_tma_k;
    // FP32 mode into C with at least 256 columns: 128x256 tiles, twice
    // the tensor work per MMA instruction and per stage hand-over (the FP32
    // kernel is bound by its issuing thread's per-stage path), when they finish
    // sooner: a wide tile takes about 1.52x a 128-wide one (35.7 against 23.4
    // us at K = 4096), so e.g. 32 narrow tiles on 148 SMs beat 16 wide ones.
    // Flags and redo stay on 128x128 tiles.
    const int64_t sms_all = usable_sms(info->sms);
    const int64_t waves_narrow = cdiv(cdiv(M, 128) * cdiv(N, 128), sms_all);
    const int64_t waves_wide = cdiv(cdiv(M, 128) * cdiv(N, 256), sms_all);
    const int fp32_tiles = g_fp32_tiles.load(std::memory_order_relaxed);
    const bool wide = !chunked && N >= 256 &&
                      (fp32_tiles == F16ACC_FP32_TILES_WIDE ||
                       (fp32_tiles == F16ACC_FP32_TILES_AUTO && double(waves_wide) * 1.52 < double(waves_narrow)));
    const TcShape shape = wide ? TcShape{256, 4} : tc_shape(chunked != 0);
    if (v == F16ACC_VARIANT_TCGEN05) {
        const int bn = shape.bn;
        const bool maps_ok =
            make_map(&p.tmA, A, uint64_t(K), uint64_t(M), uint64_t(L.sAm) * 2, 64, 128) &&
            (b_mn ? make_map(&p.tmB, B, uint64_t(N), uint64_t(K), uint64_t(L.sBk) * 2, 64, 64)
                  : make_map(&p.tmB, B, uint64_t(K), uint64_t(N), uint64_t(L.sBn) * 2, 64, bn));
        if (!maps_ok) {
            if (variant != F16ACC_VARIANT_AUTO) return F16ACC_ERR_UNSUPPORTED;
            v = F16ACC_VARIANT_MMA_SYNC;  // the descriptor encoder refused these operands
        }
    }
    if (v == F16ACC_VARIANT_TCGEN05) {
        const int bn = shape.bn;
        p.C = C;
        p.sCm = sCm;
        p.sCn = sCn;
        p.M = int(M);
        p.N = int(N);
        p.K = int(K);
        p.tiles_m = int(cdiv(M, 128));
        p.tiles_n = int(cdiv(N, bn));
        p.group_m = kGroupM;
        bool aligned = pc % 16 == 0;
        for (int i = 0; i < n_peers; ++i) aligned = aligned && reinterpret_cast<uintptr_t>(peers[i]) % 16 == 0;
        p.c_vec = (sCn == 1 && aligned && (sCm * esize) % 16 == 0) ? 1 : 0;
        p.flags = static_cast<uint8_t*>(workspace);
        p.status = info->status;
        p.n_peers = n_peers;
        for (int i = 0; i < n_peers; ++i) p.peers[i] = peers[i];
        p.bias = static_cast<const __half*>(bias);
        p.sbias = sbias;
        // Finished tiles leave through TMA stores when C allows (row-major, 16-byte
        // aligned rows) and no peer copies have to be written with them.
        if (p.c_vec && n_peers == 0) {
            const CUtensorMapDataType ct = c_dtype == F16ACC_OUT_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                           : c_dtype == F16ACC_OUT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
            p.tma_store = make_map(&p.tmC, C, uint64_t(N), uint64_t(M), uint64_t(sCm) * esize, 128 / uint32_t(esize),
                                   128, ct)
                              ? 1
                              : 0;
        }
        const int64_t tiles = int64_t(p.tiles_m) * p.tiles_n;
        if (tiles >= (int64_t(1) << 31)) return F16ACC_ERR_INVALID_ARGUMENT;
        const int sms = usable_sms(info->sms);
        // Tail split of the chunked main pass, when the caller's workspace holds
        // its counters and partials; the counters start at zero.
        int64_t units = tiles;
        if (chunked && (phases & kPhaseMain) && bn == 128 &&
            g_tail_split.load(std::memory_order_relaxed) == F16ACC_TAIL_SPLIT_ON && split_possible(M, N, K)) {
            const TailSplit t = plan_split(tiles, K, sms);
            const int64_t need = split_partials_at(M, N) + t.s * t.tiles * kSplitPartialBytes;
            if (t.s >= 2 && int64_t(ws_bytes) >= need) {
                uint8_t* ws = static_cast<uint8_t*>(workspace);
                p.split_s = int(t.s);
                p.split_first = int(t.first);
                units = t.first + t.tiles * t.s;
                p.units = int(units);
                p.split_cnt = reinterpret_cast<int*>(ws + split_counters_at(M, N));
                p.split_part = reinterpret_cast<float*>(ws + split_partials_at(M, N));
                if (launch_zero_split_counters(p.split_cnt, int(t.tiles), stream) != cudaSuccess)
                    return F16ACC_ERR_CUDA;
            }
        }
        const int grid = int(units < sms ? units : sms);
        // Both passes in one launch when the caller wants both.
        p.inline_redo = chunked && phases == kPhaseBoth &&
                        g_redo_mode.load(std::memory_order_relaxed) == F16ACC_REDO_INLINE;
        // The chunked main pass takes its tiles dynamically (one CTA launched per
        // tile, running CTAs take over the tiles of CTAs not started yet) unless
        // an SM cap asks for a bounded persistent grid.
        p.dyn_sched = chunked && units > grid && g_sm_limit.load(std::memory_order_relaxed) == 0 &&
                      g_schedule.load(std::memory_order_relaxed) == F16ACC_SCHEDULE_DYNAMIC;
        if ((phases & kPhaseMain) &&
            launch_tc(p, shape, chunked != 0, b_mn, c_dtype, false, p.dyn_sched ? int(units) : grid, stream) !=
                cudaSuccess)
            return F16ACC_ERR_CUDA;
        p.dyn_sched = 0;  // the separate redo pass walks the flags in static order, whole tiles
        p.split_s = 0;
        if (chunked && (phases & kPhaseRedo) && !p.inline_redo &&
            launch_tc(p, tc_shape(false), false, b_mn, c_dtype, true, grid, stream) != cudaSuccess)
            return F16ACC_ERR_CUDA;
        return F16ACC_OK;
    }

    if (n_peers > 0) return F16ACC_ERR_UNSUPPORTED;  // peer stores: tcgen05 path only
    MmaParams q;
    std::memset(&q, 0, sizeof(q));
    q.A = static_cast<const __half*>(A);
    q.B = static_cast<const __half*>(B);
    q.C = C;
    q.sAm = L.sAm;
    q.sAk = L.sAk;
    q.sBk = L.sBk;
    q.sBn = L.sBn;
    q.sCm = sCm;
    q.sCn = sCn;
    q.M = int(M);
    q.N = int(N);
    q.K = int(K);
    q.tiles_m = int(cdiv(M, MmaCfg::BM));
    q.tiles_n = int(cdiv(N, MmaCfg::BN));
    q.group_m = kGroupM;
    q.c_vec = (sCn == 1 && pc % (2 * esize) == 0 && sCm % 2 == 0) ? 1 : 0;
    q.flags = static_cast<uint8_t*>(workspace);
    q.bias = static_cast<const __half*>(bias);
    q.sbias = sbias;
    const int a_mode = L.a_vec ? kLoadKVec : kLoadGeneric;
    const int b_mode = L.b_kvec ? kLoadKVec : (L.b_nvec ? kLoadNVec : kLoadGeneric);
    const int64_t tiles = int64_t(q.tiles_m) * q.tiles_n;
    if (tiles >= (int64_t(1) << 31)) return F16ACC_ERR_INVALID_ARGUMENT;
    if ((phases & kPhaseMain) &&
        launch_mma(q, chunked != 0, a_mode, b_mode, c_dtype, false, int(tiles), stream) != cudaSuccess)
        return F16ACC_ERR_CUDA;
    if (chunked && (phases & kPhaseRedo)) {
        const int64_t sms2 = 2 * int64_t(usable_sms(info->sms));
        const int64_t redo_grid = tiles < sms2 ? tiles : sms2;
        if (launch_mma(q, false, a_mode, b_mode, c_dtype, true, int(redo_grid), stream) != cudaSuccess)
            return F16ACC_ERR_CUDA;
    }
    return F16ACC_OK;
}

}  // namespace
}  // namespace f16acc

using namespace f16acc;

extern "C" {

int f16acc_gemm(const void* A, int64_t sAm, int64_t sAk, const void* B, int64_t sBk, int64_t sBn, void* C,
                int64_t sCm, int64_t sCn, int c_dtype, int64_t M, int64_t N, int64_t K, int chunked, void* workspace,
                size_t ws_bytes, int device, void* stream) {
    return run(A, sAm, sAk, B, sBk, sBn, C, sCm, sCn, c_dtype, M, N, K, chunked, workspace, ws_bytes, device, stream,
               F16ACC_VARIANT_AUTO, kPhaseBoth);
}

int f16acc_gemm_ex(const void* A, int64_t sAm, int64_t sAk, const void* B, int64_t sBk, int64_t sBn, void* C,
                   int64_t sCm, int64_t sCn, int c_dtype, int64_t M, int64_t N, int64_t K, int chunked,
                   void* workspace, size_t ws_bytes, int device, void* stream, int variant) {
    return run(A, sAm, sAk, B, sBk, sBn, C, sCm, sCn, c_dtype, M, N, K, chunked, workspace, ws_bytes, device, stream,
               variant, kPhaseBoth);
}

int f16acc_gemm_main(const void* A, int64_t sAm, int64_t sAk, const void* B, int64_t sBk, int64_t sBn, void* C,
                     int64_t sCm, int64_t sCn, int c_dtype, int64_t M, int64_t N, int64_t K, int chunked,
                     void* workspace, size_t ws_bytes, int device, void* stream, int variant) {
    return run(A, sAm, sAk, B, sBk, sBn, C, sCm, sCn, c_dtype, M, N, K, chunked, workspace, ws_bytes, device, stream,
               variant, kPhaseMain);
}

int f16acc_gemm_redo(const void* A, int64_t sAm, int64_t sAk, const void* B, int64_t sBk, int64_t sBn, void* C,
                     int64_t sCm, int64_t sCn, int c_dtype, int64_t M, int64_t N, int64_t K, int chunked,
                     void* workspace, size_t ws_bytes, int device, void* stream, int variant) {
    return run(A, sAm, sAk, B, sBk, sBn, C, sCm, sCn, c_dtype, M, N, K, chunked, workspace, ws_bytes, device, stream,
               variant, kPhaseRedo);
}

int f16acc_gemm_allgather(const void* A, int64_t sAm, int64_t sAk, const void* B, int64_t sBk, int64_t sBn,
                          void* const* outs, int n_outs, int64_t sCm, int64_t sCn, int c_dtype, int64_t M, int64_t N,
                          int64_t K, int chunked, void* workspace, size_t ws_bytes, int device, void* stream) {
    if (outs == nullptr || n_outs < 1 || n_outs > kMaxPeers + 1) return F16ACC_ERR_INVALID_ARGUMENT;
    return run(A, sAm, sAk, B, sBk, sBn, outs[0], sCm, sCn, c_dtype, M, N, K, chunked, workspace, ws_bytes, device,
               stream, F16ACC_VARIANT_TCGEN05, kPhaseBoth, outs + 1, n_outs - 1);
}

int f16acc_gemm_bias(const void* A, int64_t sAm, int64_t sAk, const void* B, int64_t sBk, int64_t sBn,
                     const void* bias, int64_t sbias, void* C, int64_t sCm, int64_t sCn, int c_dtype, int64_t M,
                     int64_t N, int64_t K, int chunked, void* workspace, size_t ws_bytes, int device, void* stream,
                     int variant) {
    if (bias == nullptr && M > 0 && N > 0) return F16ACC_ERR_INVALID_ARGUMENT;
    return run(A, sAm, sAk, B, sBk, sBn, C, sCm, sCn, c_dtype, M, N, K, chunked, workspace, ws_bytes, device, stream,
               variant, kPhaseBoth, nullptr, 0, bias, sbias);
}

size_t f16acc_workspace_bytes(int64_t M, int64_t N, int64_t K) {
    if (M <= 0 || N <= 0) return 16;
    // Smallest tile any variant uses is 128 x 128: its flags, then room for the
    // tail split (at most kSplitSlots partial tiles, and 4 a tile).
    if (!split_possible(M, N, K)) return size_t(flag_area(M, N));
    const int64_t tiles = cdiv(M, 128) * cdiv(N, 128);
    const int64_t slots = tiles * kSplitMax < kSplitSlots ? tiles * kSplitMax : kSplitSlots;
    return size_t(split_partials_at(M, N) + slots * kSplitPartialBytes);
}

const char* f16acc_strerror(int code) {
    switch (code) {
        case F16ACC_OK: return "ok";
        case F16ACC_ERR_INVALID_ARGUMENT:
            return "mm needs (M, K) @ (K, N) fp16 operands with non-negative sizes below 2**31 and a supported output dtype";
        case F16ACC_ERR_WORKSPACE: return "workspace missing, smaller than f16acc_workspace_bytes(), or not 16-byte aligned";
        case F16ACC_ERR_UNSUPPORTED: return "the requested kernel variant cannot take these operands";
        case F16ACC_ERR_CUDA: return "a CUDA call or kernel launch failed";
        case F16ACC_ERR_DEVICE_TIMEOUT: return "a kernel gave up waiting on the device (see f16acc_device_status)";
        case F16ACC_ERR_TOO_LARGE:
            return "output needs more 128x128 tiles than f16acc_gemm_noalloc's fixed flag array holds "
                   "(F16ACC_NOALLOC_MAX_TILES); use f16acc_gemm with a workspace";
    }
    return "unknown f16acc error code";
}

int f16acc_get_plan(const void* A, int64_t sAm, int64_t sAk, const void* B, int64_t sBk, int64_t sBn, int64_t M,
                    int64_t N, int64_t K, int variant, f16acc_plan* out) {
    if (!out || M < 0 || N < 0 || K < 0) return F16ACC_ERR_INVALID_ARGUMENT;
    const Layout L = analyse(A, sAm, sAk, B, sBk, sBn, M, N, K);
    const int v = choose_variant(L, M, N, K, variant);
    if (v < 0) return variant == F16ACC_VARIANT_AUTO ? F16ACC_ERR_INVALID_ARGUMENT : F16ACC_ERR_UNSUPPORTED;
    out->variant = v;
    out->tile_m = v == F16ACC_VARIANT_SKINNY ? skinny_rows(M) : 128;
    out->tile_n = v == F16ACC_VARIANT_TCGEN05 ? tc_shape(true).bn : (v == F16ACC_VARIANT_SKINNY ? SkinnyCfg::BN : MmaCfg::BN);
    out->tiles_m = cdiv(M, out->tile_m);
    out->tiles_n = cdiv(N, out->tile_n);
    return F16ACC_OK;
}

int f16acc_flag_bytes_per_tile(void) { return kFlagBytesPerTile; }

int f16acc_probe_chunk_rate(int mode, int epi_split, int chunks, int grid, void* out, int device, void* stream) {
    const bool known = mode == 0 || mode == 1 || mode == 2 || mode == 30 || mode == 31 || mode == 32;
    if (!known || chunks < 0 || grid <= 0 || out == nullptr) return F16ACC_ERR_INVALID_ARGUMENT;
    if (mode == 2 && epi_split != 2 && epi_split != 4) return F16ACC_ERR_INVALID_ARGUMENT;
    DeviceInfo* info = device_info(device);
    if (!info) return F16ACC_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess || info->err != cudaSuccess) return F16ACC_ERR_CUDA;
    return launch_chunk_rate(mode, epi_split, chunks, grid, static_cast<float*>(out), info->status,
                             static_cast<cudaStream_t>(stream)) == cudaSuccess
               ? F16ACC_OK
               : F16ACC_ERR_CUDA;
}

int f16acc_selftest_wait_timeout(uint64_t limit_ns, void* out, int device, void* stream) {
    if (limit_ns == 0 || limit_ns > kWaitLimitNs || out == nullptr) return F16ACC_ERR_INVALID_ARGUMENT;
    DeviceInfo* info = device_info(device);
    if (!info) return F16ACC_ERR_INVALID_ARGUMENT;
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess || info->err != cudaSuccess) return F16ACC_ERR_CUDA;
    return launch_wait_selftest(limit_ns, static_cast<unsigned long long*>(out), info->status,
                                static_cast<cudaStream_t>(stream)) == cudaSuccess
               ? F16ACC_OK
               : F16ACC_ERR_CUDA;
}

int f16acc_set_sm_limit(int max_sms) {
    if (max_sms < 0) return F16ACC_ERR_INVALID_ARGUMENT;
    const int prev = g_sm_limit.exchange(max_sms);
    return prev;
}

int f16acc_set_redo_mode(int mode) {
    if (mode != F16ACC_REDO_SEPARATE && mode != F16ACC_REDO_INLINE) return F16ACC_ERR_INVALID_ARGUMENT;
    return g_redo_mode.exchange(mode);
}

int f16acc_set_schedule(int mode) {
    if (mode != F16ACC_SCHEDULE_STATIC && mode != F16ACC_SCHEDULE_DYNAMIC) return F16ACC_ERR_INVALID_ARGUMENT;
    return g_schedule.exchange(mode);
}

int f16acc_set_tail_split(int mode) {
    if (mode != F16ACC_TAIL_SPLIT_ON && mode != F16ACC_TAIL_SPLIT_OFF) return F16ACC_ERR_INVALID_ARGUMENT;
    return g_tail_split.exchange(mode);
}

int f16acc_set_fp32_tiles(int mode) {
    if (mode != F16ACC_FP32_TILES_AUTO && mode != F16ACC_FP32_TILES_WIDE && mode != F16ACC_FP32_TILES_NARROW)
        return F16ACC_ERR_INVALID_ARGUMENT;
    return g_fp32_tiles.exchange(mode);
}

int f16acc_set_tc_config(int tile_n, int epi_split) {
    if (!tc_shape_supported(TcShape{tile_n, epi_split == 0 ? 4 : epi_split})) return F16ACC_ERR_INVALID_ARGUMENT;
    g_tc_bn.store(tile_n);
    g_tc_epi.store(epi_split);
    return F16ACC_OK;
}

int f16acc_device_status(int device, int reset) {
    DeviceInfo* info = device_info(device);
    if (!info || info->err != cudaSuccess) return -1;
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess) return -1;
    if (cudaDeviceSynchronize() != cudaSuccess) return -1;
    int v = 0;
    if (cudaMemcpy(&v, info->status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (reset) {
        const int zero = 0;
        if (cudaMemcpy(info->status, &zero, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) return -1;
    }
    return v;
}

const char* f16acc_version(void) { return "f16acc_b200 0.1 (sm_100a: tcgen05 + mma.sync)"; }

}  // extern "C"
