// tc_gemm.cuh -- warp-specialised tcgen05 GEMM for sm_100a, chunked FP16
// accumulate with FP32 chunk sums, plus its FP32-accumulate twin that serves
// both `chunked=False` and the redo of flagged tiles.
//
// Reference semantics (steppergg/f16acc):
//   f16acc/kernel.py:44-49  K walked in 32-long chunks from absolute offset 0;
//                           each chunk is a dot with an FP16 accumulator,
//                           converted to FP32 and added to an FP32 total.
//   f16acc/kernel.py:50-51  FP32 mode: one FP32 accumulator over all of K.
//   f16acc/kernel.py:70-71  tile flag = any accumulator not finite.
//   f16acc/kernel.py:75-81  redo: flagged tiles recomputed in FP32 mode.
//
// Design (128 x BN output tiles, 1-CTA UMMA, one CTA per SM at a time; BN =
// 128, or 256 in FP32 mode):
//   warp 0      tile scheduler and TMA producer: A [128 x 64] and B [BN x 64]
//               (or [64 x BN] when B is N-contiguous) per stage into a 4-stage
//               (BN = 256: 3-stage) smem ring, 128-byte swizzle, completion
//               counted on full[s].
//   warps 1-2   MMA warps (lane 0 issues; warp 1 owns TMEM).  Chunked mode:
//               per 64-wide stage, the two 32-long chunks go to the two chunk
//               buffers of a TMEM pair as two K=16 tcgen05.mma kind::f16 each
//               (FP16 D, first with accumulate off), then one tcgen05.commit
//               -> tfull[pair].  Hand-offs alternate between the pairs and
//               between the two warps (warp 1 + b issues into pair b), and a
//               pair is reclaimed with bar.sync on its named barrier.  FP32
//               mode: warp 1 alone, the whole K loop into one FP32 buffer.
//   warps 3..   epilogue, 4*EPI_SPLIT warps: warp w reads TMEM lanes
//               32*(w%4).. (its lane quarter) and a CW = BN/EPI_SPLIT column
//               slice.  Chunked mode: per pair tcgen05.ld (FP16 pairs packed),
//               bar.arrive to release the pair, then one mixed-precision FP32
//               add per element into register accumulators; at tile end a
//               non-finite probe sets the tile's flag bytes and the tile is
//               staged in smem (128-byte-swizzled boxes for the TMA store).
//   last warp   store warp: writes each staged tile out (TMA bulk tensor
//               stores, or plain stores to a strided C and to the peers) and
//               makes the in-kernel redo decisions.
// Chunked mode may split the tiles past the last full wave of the SMs over K
// (TcParams::split_s): each unit is an ordinary work item over a share of the
// stages, and the tile's last unit to finish adds the FP32 partials.
// Every TMA load fills this CTA's own shared memory from this GPU's own memory.
#pragma once

#include "common.cuh"
#include "ptx.cuh"
#include "tc_epilogue.cuh"

namespace f16acc {

struct TcParams {
    CUtensorMap tmA;  // A [M, K], K contiguous: dims {K, M}, box {64, 128}
    CUtensorMap tmB;  // B K-contiguous: dims {K, N}, box {64, BN};  N-contiguous: dims {N, K}, box {64, 64}
    CUtensorMap tmC;  // C row-major, when tma_store: dims {N, M}, box {128 bytes of columns, 128 rows}
    // Finished tiles leave through TMA stores (C row-major and 16-byte aligned,
    // no bias, no peers): staged in 128-byte-swizzled boxes, one bulk tensor
    // store per box.  Otherwise the store warps copy them out with plain stores.
    int tma_store;
    void* C;
    int64_t sCm, sCn;
    int M, N, K;
    int tiles_m, tiles_n;
    int group_m;
    int c_vec;        // C rows allow 16-byte vector stores
    uint8_t* flags;   // kFlagBytesPerTile per tile
    int* status;      // device status word (timeouts)
    // Fused all-gather: each finished tile is also stored, at the same element
    // offsets and strides, into these peer buffers (another GPU's memory mapped
    // into this process, written over NVLink by plain stores).  0 peers = a
    // plain GEMM.
    int n_peers;
    void* peers[kMaxPeers];
    // Optional bias, one fp16 value per output column (element stride sbias),
    // added to the FP32 result before the cast (nn.Linear's y = x W^T + b).
    const __half* bias;
    int64_t sbias;
    // Chunked mode: a CTA recomputes the tiles it flagged in FP32 mode within
    // the same launch, between its main tiles (no second kernel, no wait for
    // the whole grid).
    int inline_redo;
    // Tile order.  0: static, the grid is persistent and CTA i takes tiles
    // i, i + grid, ...  1: dynamic, one CTA per tile is launched and a running
    // CTA takes over the tile of a CTA not yet started (cluster launch
    // control), so a CTA slowed by redo work takes fewer main tiles.
    int dyn_sched;
    // Tail split (chunked main pass): the tiles from split_first on (those past
    // the last full wave of the SMs) run as split_s work units each, unit s
    // over the s-th contiguous share of the 64-wide K stages.  Each unit leaves
    // its FP32 partial tile in split_part; the unit that finishes last (counted
    // in split_cnt, zeroed before the launch) adds the tile's partials in part
    // order, then flags and stores the tile like a whole one.  split_s < 2: no
    // split, units = tiles.
    int split_s;
    int split_first;
    int units;
    int* split_cnt;      // one counter per split tile
    float* split_part;   // [split tile][part][epilogue warp][CW / 4][32 lanes] float4
};

// Work unit u: its tile and its part code, -1 for the whole K range, else
// (split tile index << 3) | part.
__device__ __forceinline__ void unit_tile(const TcParams& p, int u, int& tm, int& tn, int& part) {
    int t = u;
    part = -1;
    if (p.split_s > 1 && u >= p.split_first) {
        const int j = u - p.split_first;
        t = p.split_first + j / p.split_s;
        part = ((j / p.split_s) << 3) | (j % p.split_s);
    }
    raster(t, p.tiles_m, p.tiles_n, p.group_m, tm, tn);
}
// The 64-wide K stages [kb0, kb1) of a work unit.
__device__ __forceinline__ void unit_stages(const TcParams& p, int part, int nkb, int& kb0, int& kb1) {
    if (part < 0) {
        kb0 = 0;
        kb1 = nkb;
    } else {
        const int s = part & 7;
        kb0 = s * nkb / p.split_s;
        kb1 = (s + 1) * nkb / p.split_s;
    }
}

// Work items the producer warp hands to the MMA warp and the epilogue.
enum TcWork : int { kWorkMain = 0, kWorkRedo = 1, kWorkEnd = 2 };
constexpr int kSchedDepth = 4;   // work items in flight between the roles
constexpr int kRedoQueue = 32;   // flagged tiles waiting for their FP32 redo (bounded by the pipeline depth)

// Control block at the end of the kernel's shared memory.
template <int STAGES, int NBUF>
struct alignas(16) TcCtrl {
    uint4 clc_resp;                    // cluster launch control response
    int4 sched[kSchedDepth];           // {tm, tn, kind, part code}
    int2 redo_q[kRedoQueue];           // {tm, tn} of flagged tiles
    uint64_t full[STAGES], empty[STAGES];
    uint64_t tfull[NBUF], tempty[NBUF];
    uint64_t sched_full[kSchedDepth], sched_empty[kSchedDepth];
    uint64_t st_full[2], st_empty[2];  // staging tile b: staged by the epilogue / copied out by the store warps
    int4 st_meta[2];                   // {tm, tn, TcStore kind, column half} of the tile in staging b
    uint64_t clc_bar, drain;
    uint32_t tmem_slot;
    int abort_flag;
    int rq_tail;                       // redo items pushed (store warps)
    int rq_head;                       // redo items taken (producer)
    int main_done;                     // main tiles whose flag is decided (store warps)
    int tile_bad[2];                   // OR of the epilogue warps' flags for the tile in staging b
    // Tail split: every epilogue warp has written its slice of the unit's
    // partial (split_written), and epilogue warp 0 has counted the unit in
    // (split_decided; split_last: it was the tile's last unit).
    uint64_t split_written, split_decided;
    int split_last;
};

// What a staged tile asks of the store warps.
enum TcStore : int {
    kStoreTile = 0,     // copy it out
    kStoreDecide = 1,   // copy it out, and decide whether it needs the in-kernel FP32 redo
    kStoreEnd = 2,      // no tile: the epilogue is done
    kStoreNone = 3,     // no tile: a split unit that was not its tile's last (its main item is done)
};

template <int BN_, int EPI_SPLIT_, int OUT_, bool CHUNKED_>
struct TcConfig {
    static constexpr int BM = 128;
    static constexpr int BN = BN_;
    static constexpr int BK = 64;  // one 128-byte swizzle row of f16 = two 32-long chunks
    static constexpr int EPI_SPLIT = EPI_SPLIT_;
    static constexpr int EPI_WARPS = 4 * EPI_SPLIT;
    // MMA-issuing warps: two in the chunked kernel (warps 1 and 2, one per chunk
    // of a pair), one in the FP32 kernels, whose single accumulator takes every
    // MMA in order.  Store warps copy staged tiles out to C (and peers): one in
    // the chunked kernel (a tile's copy-out is a few hundred store instructions
    // against ~40 us of compute), two in the FP32 kernels (a tile every ~20 us).
    // Either way 16 epilogue warps make 20 warps, 96 registers a thread (a 21st
    // warp would cut it to 80); 8 make 12 warps and 168.
    static constexpr int MMA_WARPS = CHUNKED_ ? 2 : 1;
    static constexpr int FIRST_EPI = 1 + MMA_WARPS;
    static constexpr int STORE_WARPS = CHUNKED_ ? 1 : 2;
    static constexpr int CW = BN / EPI_SPLIT;  // columns per epilogue warp
    static constexpr int THREADS = 32 * (FIRST_EPI + EPI_WARPS + STORE_WARPS);
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int OUT_BYTES = OUT_ == kOutF32 ? 4 : 2;
    // Output staging: the finished tile is assembled in smem so rows leave in
    // whole, coalesced 16-byte-per-lane stores (local C and every peer).  Row
    // pitch padded by 16 bytes so the per-thread row writes spread over banks.
    // Two staging tiles let the epilogue stage tile k+1 while the store warps
    // copy tile k out; an fp32 tile is twice the size and gets one, and so does
    // a 128x256 tile, whose 48 KB stages leave room for three in the ring.  An
    // fp32 128x256 tile (128 KB) is staged one 128-column half at a time, a
    // hand-over each.
    static constexpr int STAGE_COLS = (BN == 256 && OUT_BYTES == 4) ? 128 : BN;
    static constexpr int HALVES = BN / STAGE_COLS;
    static constexpr int STAGE_PITCH = STAGE_COLS * OUT_BYTES + 16;
    static constexpr int STAGING_BYTES = BM * STAGE_PITCH;
    static constexpr int SBUF = (OUT_BYTES == 4 || BN == 256) ? 1 : 2;
    static constexpr int STAGES = BN == 256 ? 3 : 4;  // measured at BN = 128: a fifth stage adds about 1 %
    static constexpr int TMEM_COLS = 512;
    static constexpr int ACC_COLS = BN;  // one 32-bit TMEM column per accumulator element, f16 or f32
    static constexpr int NBUF = TMEM_COLS / ACC_COLS;
    using Ctrl = TcCtrl<STAGES, NBUF>;
    static constexpr int SMEM_BYTES =
        STAGES * STAGE_BYTES + SBUF * STAGING_BYTES + 1024 /*alignment slack*/ + int(sizeof(Ctrl));
    static constexpr int FLAG_BYTES_PER_WARP = kFlagBytesPerTile / EPI_WARPS;  // every slot byte gets written
    static_assert(FLAG_BYTES_PER_WARP * EPI_WARPS == kFlagBytesPerTile &&
                      (FLAG_BYTES_PER_WARP == 1 || FLAG_BYTES_PER_WARP == 2),
                  "flag slot split over the epilogue warps");
    static_assert(CW == 32 || CW % 64 == 0, "epilogue column slice");
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
    // Chunked mode keeps 4 FP16 chunk buffers of BN 32-bit TMEM columns.
    static_assert(BN == 128 || (BN == 256 && !CHUNKED_), "tile width");
};

// Write this thread's CW accumulators of one tile row into the smem staging tile.
template <int OUT, int CW, int PITCH>
__device__ __forceinline__ void stage_row(uint8_t* staging, int row_in_tile, int col_in_tile, const float (&acc)[CW]) {
    using Tr = OutTraits<OUT>;
    uint8_t* dst = staging + row_in_tile * PITCH + col_in_tile * int(sizeof(typename Tr::T));
#pragma unroll
    for (int j = 0; j < CW; j += Tr::kVec) *reinterpret_cast<uint4*>(dst + j * int(sizeof(typename Tr::T))) = pack16<OUT>(&acc[j]);
}

// Stage one thread's row segment for the TMA store: the tile is kept as
// BN*sizeof(T)/128 boxes of BM rows x 128 bytes, each with the 128-byte
// swizzle of the C tensor map (16-byte piece w of row r at position w ^ (r % 8)
// of the row), which also spreads a warp's rows over all banks.
// With `bias` (this thread's first column; element stride sbias, `ncols`
// columns inside C) each value becomes add_bias of it, as the store warps'
// copy-out computes it; the bias loads and the staging stores are then ordered
// volatile asm, so only one piece's bias is live at a time.
template <int OUT, int BM, int CW>
__device__ __forceinline__ void stage_row_swizzled(uint8_t* staging, int r, int col_in_tile, const float (&acc)[CW],
                                                   const __half* bias, int64_t sbias, int ncols) {
    using Tr = OutTraits<OUT>;
    constexpr int ES = int(sizeof(typename Tr::T));
#pragma unroll
    for (int j = 0; j < CW; j += Tr::kVec) {
        const int piece = (col_in_tile + j) * ES / 16;  // 16-byte piece of the tile row
        const int box = piece >> 3, w = piece & 7;
        uint8_t* dst = staging + box * (BM * 128) + r * 128 + ((w ^ (r & 7)) << 4);
        if (bias == nullptr) {
            *reinterpret_cast<uint4*>(dst) = pack16<OUT>(&acc[j]);
        } else {
            float v[Tr::kVec];
#pragma unroll
            for (int i = 0; i < Tr::kVec; ++i)
                v[i] = j + i < ncols ? Tr::round_trip(acc[j + i]) + __half2float(ldg_half_ordered(bias + (j + i) * sbias))
                                     : acc[j + i];
            st_shared_v4_ordered(dst, pack16<OUT>(v));
        }
    }
}

// Copy the staged BM x BN tile to `n_dst` outputs with identical row stride:
// lanes run along a row, 16 bytes each, so every store instruction writes
// whole contiguous row segments.  Each lane reads U pieces from shared memory
// before it stores them, so U loads are in flight at once.  Column tails past
// N go element by element.
template <int OUT, int BM, int BN, int PITCH, int NWARPS>
__device__ __forceinline__ void store_staged(const uint8_t* staging, void* const* dst, int n_dst, int64_t sCm,
                                             int row0, int col0, int M, int N, int warp_idx, int lane,
                                             const __half* bias, int64_t sbias) {
    using Tr = OutTraits<OUT>;
    using T = typename Tr::T;
    constexpr int kChunks = BN * int(sizeof(T)) / 16;  // 16-byte pieces per tile row
    constexpr int kStep = NWARPS * 32;
    constexpr int kIters = BM * kChunks / kStep;
    constexpr int U = 4;
    static_assert(BM * kChunks % kStep == 0 && kIters % U == 0, "store split");
    for (int it = 0; it < kIters; it += U) {
        uint4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int idx = (it + u) * kStep + warp_idx * 32 + lane;
            const int r = idx / kChunks, c16 = idx - r * kChunks;
            v[u] = *reinterpret_cast<const uint4*>(staging + r * PITCH + c16 * 16);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int idx = (it + u) * kStep + warp_idx * 32 + lane;
            const int r = idx / kChunks, c16 = idx - r * kChunks;
            const int grow = row0 + r, gcol = col0 + c16 * Tr::kVec;
            if (grow >= M || gcol >= N) continue;
            uint4 x = v[u];
            if (bias != nullptr) x = add_bias16<OUT>(x, bias, sbias, gcol, N);
            const int64_t off = int64_t(grow) * sCm + gcol;
            if (gcol + Tr::kVec <= N) {
                for (int d = 0; d < n_dst; ++d) *reinterpret_cast<uint4*>(reinterpret_cast<T*>(dst[d]) + off) = x;
            } else {
                const T* e = reinterpret_cast<const T*>(&x);
                for (int d = 0; d < n_dst; ++d)
                    for (int t = 0; t < Tr::kVec && gcol + t < N; ++t) reinterpret_cast<T*>(dst[d])[off + t] = e[t];
            }
        }
    }
}

template <int OUT, int BM, int BN, int PITCH, int NWARPS>
__device__ __forceinline__ void store_staged_strided(const uint8_t* staging, void* const* dst, int n_dst, int64_t sCm,
                                                     int64_t sCn, int row0, int col0, int M, int N, int warp_idx,
                                                     int lane, const __half* bias, int64_t sbias) {
    using Tr = OutTraits<OUT>;
    using T = typename Tr::T;
    const bool along_row = sCn == 1;
    for (int idx = warp_idx * 32 + lane; idx < BM * BN; idx += NWARPS * 32) {
        const int r = along_row ? idx / BN : idx % BM;
        const int c = along_row ? idx % BN : idx / BM;
        const int grow = row0 + r, gcol = col0 + c;
        if (grow >= M || gcol >= N) continue;
        T v = *reinterpret_cast<const T*>(staging + r * PITCH + c * int(sizeof(T)));
        if (bias != nullptr) v = Tr::cvt(Tr::to_float(v) + __half2float(bias[int64_t(gcol) * sbias]));
        const int64_t off = int64_t(grow) * sCm + int64_t(gcol) * sCn;
        for (int d = 0; d < n_dst; ++d) reinterpret_cast<T*>(dst[d])[off] = v;
    }
}

template <int BN, int EPI_SPLIT, bool CHUNKED, bool B_MN, int OUT, bool REDO>
__global__ void __launch_bounds__(TcConfig<BN, EPI_SPLIT, OUT, CHUNKED>::THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ TcParams p) {
    using Cfg = TcConfig<BN, EPI_SPLIT, OUT, CHUNKED>;
    constexpr int BM = Cfg::BM, BK = Cfg::BK, STAGES = Cfg::STAGES, NBUF = Cfg::NBUF, CW = Cfg::CW;
    constexpr int ISSUERS = Cfg::MMA_WARPS;
    static_assert(!(CHUNKED && REDO), "the redo pass runs in FP32 mode");

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
    uint8_t* staging = smem + STAGES * Cfg::STAGE_BYTES;
    auto* ctrl = reinterpret_cast<typename Cfg::Ctrl*>(staging + Cfg::SBUF * Cfg::STAGING_BYTES);
    uint64_t* full = ctrl->full;
    uint64_t* empty = ctrl->empty;
    uint64_t* tfull = ctrl->tfull;
    uint64_t* tempty = ctrl->tempty;
    uint64_t* drain = &ctrl->drain;
    volatile int* abort_flag = &ctrl->abort_flag;
    volatile int* rq_tail = &ctrl->rq_tail;
    volatile int* rq_head = &ctrl->rq_head;
    volatile int* main_done = &ctrl->main_done;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);  // the commit of the MMA thread that read the stage
        }
        for (int b = 0; b < NBUF; ++b) {
            mbar_init(&tfull[b], 1);  // the commit of the MMA thread that filled it (chunked: pair b)
            mbar_init(&tempty[b], Cfg::EPI_WARPS);
        }
        for (int i = 0; i < kSchedDepth; ++i) {
            mbar_init(&ctrl->sched_full[i], 1);
            mbar_init(&ctrl->sched_empty[i], ISSUERS + Cfg::EPI_WARPS);  // the MMA threads, every epilogue warp
        }
        mbar_init(&ctrl->clc_bar, 1);
        mbar_init(drain, ISSUERS);
        mbar_init(&ctrl->split_written, Cfg::EPI_WARPS);
        mbar_init(&ctrl->split_decided, 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&ctrl->st_full[b], Cfg::EPI_WARPS);
            mbar_init(&ctrl->st_empty[b], Cfg::STORE_WARPS);
        }
        *abort_flag = 0;
        *rq_tail = 0;
        *rq_head = 0;
        *main_done = 0;
        ctrl->tile_bad[0] = ctrl->tile_bad[1] = 0;
        fence_mbarrier_init();
        tma_prefetch_desc(&p.tmA);
        tma_prefetch_desc(&p.tmB);
    }
    if (warp == 1) {
        tmem_alloc(&ctrl->tmem_slot, Cfg::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctrl->tmem_slot;

    // Every launch is a programmatic dependent launch: the CTAs may start while
    // the previous kernel on the stream drains, and everything above (barriers,
    // TMEM, descriptor prefetch) touches no global memory.  griddepcontrol.wait
    // returns once that kernel has completed and its writes are visible (the
    // redo pass: the main pass's flags and C).  The main pass then lets the
    // next launch on the stream get scheduled.
    grid_dep_wait();
    if constexpr (!REDO) grid_dep_launch();

    const int tiles = p.tiles_m * p.tiles_n;
    const int units = p.split_s > 1 ? p.units : tiles;  // work units of the main pass
    const int nkb = (p.K + BK - 1) / BK;
    const int nchunks = (p.K + 31) / 32;
    const int nk16 = (p.K + 15) / 16;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            uint32_t s = 0, ph = 0;
            uint32_t pending = 0, pend_parity = 0;  // stages with a load issued, and that load's phase parity
            auto load_tile = [&](int tm, int tn, int part) -> bool {
                int kb0, kb1;
                unit_stages(p, part, nkb, kb0, kb1);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, p.status, kStatusTimeoutProducer)) return false;
                    mbar_arrive_expect_tx(&full[s], Cfg::STAGE_BYTES);
                    pending |= 1u << s;
                    pend_parity = (pend_parity & ~(1u << s)) | (ph << s);
                    tma_load_2d(sA + s * Cfg::A_BYTES, &p.tmA, &full[s], kb * BK, tm * BM);
                    if constexpr (!B_MN) {
                        tma_load_2d(sB + s * Cfg::B_BYTES, &p.tmB, &full[s], kb * BK, tn * BN);
                    } else {
#pragma unroll
                        for (int j = 0; j < BN / 64; ++j)
                            tma_load_2d(sB + s * Cfg::B_BYTES + j * (64 * BK * 2), &p.tmB, &full[s], tn * BN + j * 64,
                                        kb * BK);
                    }
                    if (++s == STAGES) { s = 0; ph ^= 1u; }
                }
                return true;
            };
            // ---- tile scheduler: this thread decides the CTA's work items, in order,
            // and publishes each to the MMA warp and the epilogue through ctrl->sched.
            const bool inline_redo = CHUNKED && p.inline_redo != 0;
            int next_static = blockIdx.x;  // static order: this CTA's next main work unit
            bool clc_inflight = false;     // a cancel request not yet answered
            uint32_t clc_phase = 0;
            int issued_main = 0, taken = 0;
            auto clc_ask = [&]() {
                mbar_arrive_expect_tx(&ctrl->clc_bar, 16);
                clc_try_cancel(&ctrl->clc_resp, &ctrl->clc_bar);
                clc_inflight = true;
            };
            auto pop_redo = [&](int& tm, int& tn) -> bool {
                if (taken == *rq_tail) return false;
                __threadfence_block();  // the entry was written before the tail moved
                const int2 w = ctrl->redo_q[taken % kRedoQueue];
                tm = w.x;
                tn = w.y;
                *rq_head = ++taken;
                return true;
            };
            // Every main tile issued here has had its flag decided by the epilogue.
            auto wait_flags_decided = [&]() -> bool {
                const uint64_t t0 = globaltimer_ns();
                while (*main_done != issued_main) {
                    if (*abort_flag) return false;
                    if (globaltimer_ns() - t0 > kWaitLimitNs) {
                        atomicCAS(p.status, 0, kStatusTimeoutSchedule);
                        *abort_flag = 1;
                        return false;
                    }
                    __nanosleep(128);
                }
                return true;
            };
            // The next work item: a finished flagged tile's redo first, then a new
            // main tile, then (main tiles exhausted) the redo items still to come,
            // then the end.  False when a wait gave up.
            auto next_work = [&](int& kind, int& tm, int& tn, int& part) -> bool {
                kind = kWorkRedo;
                part = -1;
                if (inline_redo && pop_redo(tm, tn)) return true;
                kind = kWorkMain;
                if (p.dyn_sched) {
                    if (clc_inflight) {
                        if (!mbar_wait(&ctrl->clc_bar, clc_phase, abort_flag, p.status, kStatusTimeoutProducer))
                            return false;
                        clc_phase ^= 1u;
                        clc_inflight = false;
                        uint32_t cta;
                        if (clc_query(&ctrl->clc_resp, cta)) {  // that CTA's work unit is ours now
                            clc_ask();
                            unit_tile(p, static_cast<int>(cta), tm, tn, part);
                            return true;
                        }
                    }
                } else {
                    while (next_static < units) {
                        const int t = next_static;
                        next_static += gridDim.x;
                        unit_tile(p, t, tm, tn, part);
                        if (REDO && !tile_flagged(p.flags, static_cast<int64_t>(tm) * p.tiles_n + tn)) continue;
                        return true;
                    }
                }
                kind = kWorkRedo;
                part = -1;
                if (inline_redo) {
                    if (!wait_flags_decided()) return false;
                    if (pop_redo(tm, tn)) return true;
                }
                kind = kWorkEnd;
                return true;
            };
            int kind, tm, tn, part;
            if (p.dyn_sched) {  // this CTA's own work unit first, the next one asked for meanwhile
                kind = kWorkMain;
                unit_tile(p, static_cast<int>(blockIdx.x), tm, tn, part);
                clc_ask();
            } else if (!next_work(kind, tm, tn, part)) {
                goto producer_done;
            }
            for (uint32_t qi = 0, qph = 0;;) {
                if (!mbar_wait(&ctrl->sched_empty[qi], qph ^ 1u, abort_flag, p.status, kStatusTimeoutProducer))
                    goto producer_done;
                ctrl->sched[qi] = make_int4(tm, tn, kind, part);
                mbar_arrive(&ctrl->sched_full[qi]);
                if (++qi == kSchedDepth) { qi = 0; qph ^= 1u; }
                if (kind == kWorkEnd) break;
                if (kind == kWorkMain) ++issued_main;
                if (!load_tile(tm, tn, part)) goto producer_done;
                if (!next_work(kind, tm, tn, part)) goto producer_done;
            }
        producer_done:
            // Let every copy this CTA issued land before the CTA can exit
            // (they already have on a normal exit; this matters after an abort).
            for (int st = 0; st < STAGES; ++st)
                if (pending & (1u << st)) mbar_wait_drain(&full[st], (pend_parity >> st) & 1u);
            if (clc_inflight) mbar_wait_drain(&ctrl->clc_bar, clc_phase);  // only after an abort
        }
    } else if (warp < Cfg::FIRST_EPI) {
        // ------------------------------------------------------------ MMA issuers
        // Chunked kernel: two MMA warps on different SM sub-partitions take the
        // hand-offs (chunk pairs, FP32 redo tiles) alternately: hand-off n goes
        // through pair b = n & 1 and is issued by warp 1 + b, so one warp issues
        // pair n while the other issues pair n+1.  Pair b is reclaimed with
        // bar.sync on named barrier kPairBarrier + b, whose rounds are that one
        // warp plus every epilogue warp.  FP32 kernel: one thread, mbarriers only.
        // Hang freedom of the bar.sync: (1) each named barrier has one waiter,
        // warp 1 + b, which issues into pair b again only after the round
        // completes; (2) it checks the abort flag (warp-uniformly) before every
        // bar.sync and stops there once it is set; (3) an epilogue warp that
        // leaves early raises the flag and then arrives once for each hand-off
        // issued and not yet released by it (at most one per pair, found issued
        // by its tfull completing), so the round a waiter is in always fills,
        // and never overfills.
        constexpr int NB = 32 * (1 + Cfg::EPI_WARPS);  // release-barrier threads
        if (warp <= ISSUERS && (CHUNKED || lane == 0)) {
            const uint32_t mine = uint32_t(warp - 1);  // chunked: the pair this warp issues into
            const bool issue = lane == 0;
            constexpr uint32_t idesc = idesc_f16(!CHUNKED, B_MN, BM, BN);
            constexpr uint32_t idesc32 = idesc_f16(true, B_MN, BM, BN);
            // Operand descriptors of stage 0.  Stage s and K16 step ks are reached by
            // adding their byte offset / 16 to the start-address field, which cannot
            // carry out (shared addresses stay below 2^18), so the issue loop spends
            // one add per descriptor.
            const uint64_t a_desc0 = sdesc_sw128(smem_u32(sA), 16, 1024);
            const uint64_t b_desc0 = B_MN ? sdesc_sw128(smem_u32(sB), 64 * BK * 2, 1024)
                                          : sdesc_sw128(smem_u32(sB), 16, 1024);
            constexpr uint32_t kAStage = Cfg::A_BYTES >> 4, kBStage = Cfg::B_BYTES >> 4;
            constexpr uint32_t kAStep = 32 >> 4, kBStep = (B_MN ? 2048 : 32) >> 4;  // one K16 step
            uint32_t s = 0, ph = 0, b = 0, tph = 0;
            bool pending = false;  // chunked: a hand-off issued into `mine` and not yet reclaimed
            // A bounded mbarrier wait, uniform across the warp in the chunked kernel.
            auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
                const bool ok = mbar_wait(bar, parity, abort_flag, p.status, kStatusTimeoutMma);
                if constexpr (CHUNKED) return __all_sync(0xffffffffu, ok);
                return ok;
            };
            auto aborted = [&]() -> bool { return __any_sync(0xffffffffu, *abort_flag != 0); };
            // Before issuing into pair `mine` (chunked): wait until every epilogue
            // warp has loaded the hand-off issued into it before.  False when the
            // kernel is aborting.  The flag is checked before the bar.sync only:
            // the instructions between the barrier's release and the next MMAs are
            // the kernel's critical path (a check there cost 5 % at 4096^3).  A
            // hand-off issued after a round that an abort completed is harmless:
            // every epilogue warp has arrived, so none still reads the pair, and
            // the warp stops at its next check, before any further bar.sync.
            auto reclaim = [&]() -> bool {
                if (aborted()) return false;
                if (pending) {
                    named_bar_sync(kPairBarrier + int(mine), NB);
                    pending = false;
                }
                return true;
            };
            auto next_stage = [&]() {
                if (++s == STAGES) { s = 0; ph ^= 1u; }
            };
            // A whole tile's K loop with an FP32 accumulator in TMEM at d.
            auto fp32_tile = [&](uint32_t d) -> bool {
                for (int kb = 0; kb < nkb; ++kb) {
                    if (!wait(&full[s], ph)) return false;
                    tc_fence_after();
                    if (issue) {
                        const uint64_t a_st = a_desc0 + s * kAStage, b_st = b_desc0 + s * kBStage;
                        if ((kb + 1) * BK <= p.K) {
                            // a whole stage: four K16 steps, no tail checks (7 % of the
                            // stage's issue time at 4096^3)
                            umma_f16(d, a_st, b_st, idesc32, kb > 0 ? 1u : 0u);
                            umma_f16(d, a_st + kAStep, b_st + kBStep, idesc32, 1u);
                            umma_f16(d, a_st + 2 * kAStep, b_st + 2 * kBStep, idesc32, 1u);
                            umma_f16(d, a_st + 3 * kAStep, b_st + 3 * kBStep, idesc32, 1u);
                        } else {
#pragma unroll
                            for (int ks = 0; ks < BK / 16; ++ks) {
                                const int k16 = kb * (BK / 16) + ks;
                                if (k16 >= nk16) break;
                                umma_f16(d, a_st + ks * kAStep, b_st + ks * kBStep, idesc32, k16 > 0 ? 1u : 0u);
                            }
                        }
                        umma_commit(&empty[s]);
                    }
                    if constexpr (CHUNKED) __syncwarp();
                    next_stage();
                }
                return true;
            };
            bool normal_end = false;
            for (uint32_t qi = 0, qph = 0;;) {
                if (!wait(&ctrl->sched_full[qi], qph)) goto mma_done;
                const int kind = ctrl->sched[qi].z;
                const int part = ctrl->sched[qi].w;
                if constexpr (CHUNKED) __syncwarp();
                if (issue) mbar_arrive(&ctrl->sched_empty[qi]);
                if (++qi == kSchedDepth) { qi = 0; qph ^= 1u; }
                if (kind == kWorkEnd) {
                    normal_end = true;
                    break;
                }
                if (CHUNKED && kind == kWorkRedo) {
                    // A flagged tile in FP32 mode: the K16 MMA sequence of the FP32 kernel
                    // (so bit-identical results), accumulated in chunk buffer 2b and handed
                    // over through pair b like one chunk pair.  The other MMA warp steps
                    // over its stages.
                    if (b == mine) {
                        if (!reclaim()) goto mma_done;
                        tc_fence_after();
                        if (!fp32_tile(tmem + (2 * b) * Cfg::ACC_COLS)) goto mma_done;
                        if (issue) umma_commit(&tfull[b]);
                        __syncwarp();
                        pending = true;
                    } else {
                        for (int kb = 0; kb < nkb; ++kb) next_stage();
                    }
                    b ^= 1u;
                } else if constexpr (CHUNKED) {
                    // One hand-off per 64-wide stage of the work unit: its two 32-long
                    // chunks go to the chunk buffers 2b and 2b+1 of pair b, issued by
                    // warp 1 + b.
                    int kb0, kb1;
                    unit_stages(p, part, nkb, kb0, kb1);
                    for (int kb = kb0; kb < kb1; ++kb) {
                        if (b == mine) {
                            if (!wait(&full[s], ph)) goto mma_done;
                            // operands and accumulators of this hand-off, worked out before
                            // the pair is reclaimed
                            const uint64_t a_st = a_desc0 + s * kAStage, b_st = b_desc0 + s * kBStage;
                            const uint32_t d0 = tmem + (2 * b) * Cfg::ACC_COLS;
                            const bool whole_stage = (kb + 1) * BK <= p.K;
                            if (!reclaim()) goto mma_done;
                            tc_fence_after();
                            if (issue) {
                                if (whole_stage) {
                                    // a whole stage: chunk 2kb into buffer 2b, chunk 2kb+1 into 2b+1
                                    umma_f16(d0, a_st, b_st, idesc, 0u);
                                    umma_f16(d0, a_st + kAStep, b_st + kBStep, idesc, 1u);
                                    umma_f16(d0 + Cfg::ACC_COLS, a_st + 2 * kAStep, b_st + 2 * kBStep, idesc, 0u);
                                    umma_f16(d0 + Cfg::ACC_COLS, a_st + 3 * kAStep, b_st + 3 * kBStep, idesc, 1u);
                                } else {
#pragma unroll
                                    for (int cc = 0; cc < 2; ++cc) {
                                        const int c = kb * 2 + cc;
                                        if (c >= nchunks) break;
#pragma unroll
                                        for (int h = 0; h < 2; ++h) {
                                            const int ks = cc * 2 + h;
                                            if (h == 1 && c * 32 + 16 >= p.K) break;  // K16 step past the end adds nothing
                                            umma_f16(d0 + cc * Cfg::ACC_COLS, a_st + ks * kAStep, b_st + ks * kBStep,
                                                     idesc, h);
                                        }
                                    }
                                }
                                umma_commit(&tfull[b]);
                                umma_commit(&empty[s]);
                            }
                            __syncwarp();
                            pending = true;
                        }
                        b ^= 1u;
                        next_stage();
                    }
                } else {
                    if (!mbar_wait(&tempty[b], tph ^ 1u, abort_flag, p.status, kStatusTimeoutMma)) goto mma_done;
                    tc_fence_after();
                    if (!fp32_tile(tmem + b * Cfg::ACC_COLS)) goto mma_done;
                    umma_commit(&tfull[b]);
                    if (++b == NBUF) { b = 0; tph ^= 1u; }
                }
            }
        mma_done:
            if constexpr (CHUNKED) {
                // Reclaim the last hand-off in `mine` so every round of its barrier is
                // complete when the kernel ends (skipped when aborting: nothing waits
                // on this warp then).
                if (normal_end && pending && !aborted()) named_bar_sync(kPairBarrier + int(mine), NB);
            }
            // All MMAs issued by this thread complete before TMEM is freed.
            if (issue) {
                umma_commit(drain);
                mbar_wait_drain(drain, 0);
            }
            if constexpr (CHUNKED) __syncwarp();
        }
    } else if (warp < Cfg::FIRST_EPI + Cfg::EPI_WARPS) {
        // ------------------------------------------------------------ epilogue
        const int e = warp - Cfg::FIRST_EPI;  // epilogue warp index
        const int q = warp & 3;          // TMEM lane quarter this warp may access
        const int colg = e >> 2;         // column slice
        const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
        ChunkRing<NBUF> ring{tfull, tempty, tmem + lane_base + colg * CW, Cfg::ACC_COLS};    // FP32 mode
        constexpr int NB = 32 * (1 + Cfg::EPI_WARPS);  // pair-barrier threads: one MMA warp + the epilogue
        PairRing<CW> pairs{tfull, NB, tmem + lane_base + colg * CW, Cfg::ACC_COLS};     // chunked mode
        // Finished tiles go to the store warps through the staging tiles, in order:
        // tile k in staging k % SBUF.  take_staging waits until the store warps have
        // copied out that buffer's previous tile; hand_over passes the staged tile
        // (or the end marker) on.  The epilogue itself never waits for the copy-out.
        int handed = 0;
        auto take_staging = [&]() -> bool {
            const uint32_t par = (uint32_t(handed) / Cfg::SBUF) & 1u;
            return __all_sync(0xffffffffu, mbar_wait(&ctrl->st_empty[handed % Cfg::SBUF], par ^ 1u, abort_flag,
                                                     p.status, kStatusTimeoutEpilogue));
        };
        auto hand_over = [&](int tm, int tn, int kind, int half) {
            const int b = handed % Cfg::SBUF;
            if (e == 0 && lane == 0) ctrl->st_meta[b] = make_int4(tm, tn, kind, half);
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctrl->st_full[b]);
            ++handed;
        };
        const bool inline_redo = CHUNKED && p.inline_redo != 0;
        // Tail split: leave this warp's slice of the unit's FP32 partial in
        // split_part, count the unit in once every epilogue warp has written,
        // and, in the tile's last unit, replace acc with the tile's total
        // ((p0 + p1) + p2) + ... in part order, so the sum does not depend on
        // which unit finishes last.  1: last (acc holds the total), 0: not the
        // last, -1: a wait gave up.
        uint32_t split_phase = 0;
        auto split_combine = [&](int code, float (&a)[CW]) -> int {
            const int ts = code >> 3, S = p.split_s;
            auto slot = [&](int part) {
                return reinterpret_cast<float4*>(p.split_part) +
                       ((int64_t(ts) * S + part) * Cfg::EPI_WARPS + e) * (CW / 4) * 32 + lane;
            };
            float4* mine = slot(code & 7);
#pragma unroll
            for (int j = 0; j < CW / 4; ++j)
                __stcg(mine + j * 32, make_float4(a[4 * j], a[4 * j + 1], a[4 * j + 2], a[4 * j + 3]));
            __threadfence();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctrl->split_written);
            const uint32_t par = split_phase & 1u;
            ++split_phase;
            if (!__all_sync(0xffffffffu, mbar_wait(&ctrl->split_written, par, abort_flag, p.status,
                                                   kStatusTimeoutEpilogue)))
                return -1;
            if (e == 0 && lane == 0) {
                __threadfence();  // every epilogue warp's partial is visible before the count
                ctrl->split_last = atomicAdd(p.split_cnt + ts, 1) == S - 1 ? 1 : 0;
                mbar_arrive(&ctrl->split_decided);
            }
            if (!__all_sync(0xffffffffu, mbar_wait(&ctrl->split_decided, par, abort_flag, p.status,
                                                   kStatusTimeoutEpilogue)))
                return -1;
            if (*reinterpret_cast<volatile int*>(&ctrl->split_last) == 0) return 0;
            __threadfence();  // the other units' partials, counted in before this one
#pragma unroll
            for (int j = 0; j < CW / 4; ++j) {
                const float4 v = __ldcg(slot(0) + j * 32);
                a[4 * j] = v.x;
                a[4 * j + 1] = v.y;
                a[4 * j + 2] = v.z;
                a[4 * j + 3] = v.w;
            }
            for (int part = 1; part < S; ++part) {
                float4 v[CW / 4];
#pragma unroll
                for (int j = 0; j < CW / 4; ++j) v[j] = __ldcg(slot(part) + j * 32);
#pragma unroll
                for (int j = 0; j < CW / 4; ++j) {
                    a[4 * j] += v[j].x;
                    a[4 * j + 1] += v[j].y;
                    a[4 * j + 2] += v[j].z;
                    a[4 * j + 3] += v[j].w;
                }
            }
            return 1;
        };
        bool finished = false;  // left the loop at the end item (not by giving up on a wait)
        for (uint32_t qi = 0, qph = 0;;) {
            if (!__all_sync(0xffffffffu,
                            mbar_wait(&ctrl->sched_full[qi], qph, abort_flag, p.status, kStatusTimeoutEpilogue)))
                break;
            const int4 w = ctrl->sched[qi];
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctrl->sched_empty[qi]);
            if (++qi == kSchedDepth) { qi = 0; qph ^= 1u; }
            if (w.z == kWorkEnd) {
                finished = true;
                break;
            }
            const int tm = w.x, tn = w.y;
            const bool main_item = w.z == kWorkMain;
            float acc[CW];
            bool bad = false;
            if constexpr (CHUNKED) {
                if (main_item) {
                    int kb0, kb1;
                    unit_stages(p, w.w, nkb, kb0, kb1);
                    const int unit_chunks = min(2 * kb1, nchunks) - 2 * kb0;
                    if (!consume_chunk_pairs<CW>(acc, unit_chunks, pairs, abort_flag, p.status)) break;
                    if (w.w >= 0) {
                        // A unit of a split tile: the last one of the tile to finish goes on
                        // with the tile's total in acc; the others are done.
                        const int last = split_combine(w.w, acc);
                        if (last < 0) break;
                        if (last == 0) {
                            if (!take_staging()) break;
                            hand_over(tm, tn, kStoreNone, 0);
                            continue;
                        }
                    }
                    // eight independent probe chains (a 64-long chain costs ~300 cycles of
                    // latency at every tile end); NaN in any of them marks the tile
                    float z8[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                    for (int j = 0; j < CW; ++j) z8[j & 7] = nonfinite_probe(z8[j & 7], acc[j]);
                    const float z = ((z8[0] + z8[1]) + (z8[2] + z8[3])) + ((z8[4] + z8[5]) + (z8[6] + z8[7]));
                    bad = __any_sync(0xffffffffu, z != z);
                    if (lane == 0) {
                        uint8_t* slot = p.flags + (static_cast<int64_t>(tm) * p.tiles_n + tn) * kFlagBytesPerTile;
                        if constexpr (Cfg::FLAG_BYTES_PER_WARP == 2)
                            *reinterpret_cast<uint16_t*>(slot + 2 * e) = bad ? 1 : 0;
                        else
                            slot[e] = bad ? 1 : 0;
                    }
                } else {
                    if (!consume_fp32_pair<CW>(acc, pairs, abort_flag, p.status)) break;
                }
            } else {
                if (!ring.wait_full(abort_flag, p.status)) break;
#pragma unroll
                for (int j = 0; j < CW / 32; ++j) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(ring.addr() + j * 32, r);
                    tmem_wait_ld();
                    reg_fence(r);
#pragma unroll
                    for (int k = 0; k < 32; ++k) acc[j * 32 + k] = __uint_as_float(r[k]);
                }
                ring.release(lane);
            }
            // Stage the tile, rounded to the output type, for the store warps (in
            // HALVES column parts, one hand-over each; every epilogue warp takes
            // part in each hand-over, staging only the part its columns are in).
            bool staged = true;
            for (int h = 0; h < Cfg::HALVES; ++h) {
                if (!take_staging()) {
                    staged = false;
                    break;
                }
                const int b = handed % Cfg::SBUF;
                if (Cfg::HALVES == 1 || colg * CW / Cfg::STAGE_COLS == h) {
                    const int cin = colg * CW - h * Cfg::STAGE_COLS;  // column within the staged part
                    if (p.tma_store) {
                        // The bias (if any) goes on here, after the flag, to the product
                        // rounded to the output type.
                        const int col0 = tn * BN + colg * CW;
                        stage_row_swizzled<OUT, BM, CW>(staging + b * Cfg::STAGING_BYTES, q * 32 + lane, cin, acc,
                                                        p.bias != nullptr ? p.bias + int64_t(col0) * p.sbias : nullptr,
                                                        p.sbias, p.N - col0);
                        fence_proxy_async_smem();  // the TMA store reads these bytes
                    } else {
                        stage_row<OUT, CW, Cfg::STAGE_PITCH>(staging + b * Cfg::STAGING_BYTES, q * 32 + lane, cin, acc);
                    }
                }
                const bool decide = inline_redo && main_item;
                if (decide && bad && lane == 0) atomicOr(&ctrl->tile_bad[b], 1);
                hand_over(tm, tn, decide ? kStoreDecide : kStoreTile, h);
            }
            if (!staged) break;
        }
        if (CHUNKED && !finished) {
            // Leaving early (a wait gave up): raise the abort flag, then release the
            // pairs issued to this warp, so that an MMA warp waiting in bar.sync on
            // one wakes, sees the flag and stops.
            *abort_flag = 1;
            __threadfence_block();
            __syncwarp();
            pairs.release_issued_on_exit(lane);
        }
        if (finished && take_staging()) hand_over(0, 0, kStoreEnd, 0);
    } else {
        // ------------------------------------------------------------ store warps
        // Copy each staged tile out to C and to every peer's buffer (fused
        // all-gather): whole rows in coalesced 16-byte-per-lane stores when C
        // allows, else element by element.  The bias (after the flag: the
        // reference adds it outside the kernel) goes on here, to the product
        // already rounded to the output type.  For a main tile of the chunked
        // kernel with the in-kernel redo, store warp 0 reads the OR of the 16
        // epilogue warps' flags, queues the tile for its FP32 redo if it is set,
        // and counts the tile as decided for the scheduler.
        const int sw = warp - Cfg::FIRST_EPI - Cfg::EPI_WARPS;
        void* dsts[1 + kMaxPeers] = {p.C};  // this GPU's C, then the peers' copies
        for (int i = 0; i < p.n_peers; ++i) dsts[1 + i] = p.peers[i];
        int decided = 0;
        for (int k = 0;; ++k) {
            const int b = k % Cfg::SBUF;
            const uint32_t par = (uint32_t(k) / Cfg::SBUF) & 1u;
            if (!__all_sync(0xffffffffu,
                            mbar_wait(&ctrl->st_full[b], par, abort_flag, p.status, kStatusTimeoutStore)))
                break;
            const int4 m = ctrl->st_meta[b];
            if (m.z == kStoreEnd) break;
            if (m.z == kStoreNone) {  // a split unit whose tile another unit finishes: decided, nothing to store
                if (sw == 0 && lane == 0) {
                    __threadfence_block();
                    *main_done = ++decided;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&ctrl->st_empty[b]);
                continue;
            }
            const int tm = m.x, tn = m.y;
            const int c0 = tn * BN + m.w * Cfg::STAGE_COLS;  // first column of the staged part
            bool redo_queued = false;  // this main tile is redone later in this CTA
            if (m.z == kStoreDecide && sw == 0 && lane == 0) {
                if (atomicExch(&ctrl->tile_bad[b], 0) != 0) {
                    redo_queued = true;
                    const int tail = *rq_tail;
                    if (tail - *rq_head >= kRedoQueue) {
                        atomicCAS(p.status, 0, kStatusRedoQueueFull);
                        *abort_flag = 1;
                    } else {
                        ctrl->redo_q[tail % kRedoQueue] = make_int2(tm, tn);
                        __threadfence_block();
                        *rq_tail = tail + 1;
                    }
                }
                __threadfence_block();
                *main_done = ++decided;
            }
            const uint8_t* stg = staging + b * Cfg::STAGING_BYTES;
            if (p.tma_store) {
                // One bulk tensor store per 128-byte column box.  A tile queued for
                // its redo is not stored: the redo writes it, and two bulk stores
                // to the same place are not ordered.
                constexpr int BOX_COLS = 128 / Cfg::OUT_BYTES;
                if (sw == 0 && lane == 0) {
                    if (!redo_queued) {
#pragma unroll
                        for (int j = 0; j < Cfg::STAGE_COLS / BOX_COLS; ++j)
                            if (c0 + j * BOX_COLS < p.N)  // boxes wholly past the last column hold nothing
                                tma_store_2d(&p.tmC, stg + j * (BM * 128), c0 + j * BOX_COLS, tm * BM);
                        bulk_commit_group();
                        bulk_wait_group_read0();  // the staging tile may be reused once read
                    }
                }
            } else if (p.c_vec)
                store_staged<OUT, BM, Cfg::STAGE_COLS, Cfg::STAGE_PITCH, Cfg::STORE_WARPS>(
                    stg, dsts, 1 + p.n_peers, p.sCm, tm * BM, c0, p.M, p.N, sw, lane, p.bias, p.sbias);
            else
                store_staged_strided<OUT, BM, Cfg::STAGE_COLS, Cfg::STAGE_PITCH, Cfg::STORE_WARPS>(
                    stg, dsts, 1 + p.n_peers, p.sCm, p.sCn, tm * BM, c0, p.M, p.N, sw, lane, p.bias, p.sbias);
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctrl->st_empty[b]);  // the staging tile is free again
        }
        // bulk stores complete, and peer stores become visible system-wide, before
        // the kernel is seen complete
        if (p.tma_store && sw == 0 && lane == 0) bulk_wait_group0();
        if (p.n_peers > 0) __threadfence_system();
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, Cfg::TMEM_COLS);
}

}  // namespace f16acc
