/*
 * f16acc.h -- C ABI of the B200 (sm_100a) chunked FP16-accumulate GEMM.
 *
 * C = A @ B with FP16 operands.  K is walked in 32-long chunks from offset 0;
 * each chunk is accumulated in FP16 on the tensor cores and added into an
 * FP32 accumulator.  Tiles whose FP16 chunk overflowed (any accumulator not
 * finite at the end) are flagged on the device and recomputed with FP32
 * accumulation with no host sync: by default inside the same tcgen05 launch
 * (the CTA that met the flag queues the tile and redoes it between its main
 * tiles), otherwise by a second launch on the same stream (mma.sync path,
 * f16acc_gemm_main / f16acc_gemm_redo, F16ACC_REDO_SEPARATE).
 *
 * Plain C: pointers, element strides, sizes; no CUDA or framework types.
 * `stream` is a cudaStream_t (NULL = legacy default stream) on `device`.
 * All calls are asynchronous on that stream and never abort the process:
 * they return F16ACC_OK or an error code (f16acc_strerror).
 *
 * Reference interface replaced (steppergg/f16acc, file:line in that project):
 *   f16acc/kernel.py:84-105   mm(a, b, out_dtype=torch.float16, chunked=True)
 *     -> f16acc_gemm (checks :87-90, output + flag buffers :93-95, the 64-bit
 *        index choice :97-98, the `_gemm` launch :99 and the `_redo` launch
 *        :100-104 all happen behind this one call; C and the workspace are
 *        caller-owned here instead of allocated inside).
 *   f16acc/kernel.py:94-95    the int8 flag buffer sized for the smallest tile
 *     -> f16acc_workspace_bytes.
 *   f16acc/kernel.py:87-90    ValueError messages -> f16acc_strerror.
 */
#ifndef F16ACC_H_
#define F16ACC_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes. */
#define F16ACC_OK 0
#define F16ACC_ERR_INVALID_ARGUMENT 1 /* shapes, strides, dtype code, null pointers */
#define F16ACC_ERR_WORKSPACE 2        /* workspace too small or misaligned */
#define F16ACC_ERR_UNSUPPORTED 3      /* forced variant cannot take these operands */
#define F16ACC_ERR_CUDA 4             /* a CUDA runtime call or launch failed */
#define F16ACC_ERR_DEVICE_TIMEOUT 5   /* a kernel gave up on a wait (see f16acc_device_status) */
#define F16ACC_ERR_TOO_LARGE 6        /* more output tiles than f16acc_gemm_noalloc's fixed flag array holds */

/* Output element types (c_dtype); kernel.py:93 allocates C as out_dtype. */
#define F16ACC_OUT_F16 0
#define F16ACC_OUT_F32 1
#define F16ACC_OUT_BF16 2

/* Kernel variants for f16acc_gemm_ex (measurement and tests). */
#define F16ACC_VARIANT_AUTO 0     /* skinny for M <= 64 (M <= 32 when N > 32768), else tcgen05 when the operands
                                     allow TMA, else mma.sync */
#define F16ACC_VARIANT_TCGEN05 1  /* warp-specialised tcgen05/TMA kernel only */
#define F16ACC_VARIANT_MMA_SYNC 2 /* warp-level mma.sync kernel (any strides) */
#define F16ACC_VARIANT_SKINNY 3   /* few rows (M <= 64): mma.sync tiles, K split over a CTA cluster;
                                     K-contiguous A and K- or N-contiguous B with 16-byte aligned rows.
                                     The automatic choice for M <= 64 (M <= 32 when N > 32768). */

/*
 * C[M,N] = A[M,K] @ B[K,N].  Replaces kernel.py:84-105 `mm`.
 *   A, B     FP16 device pointers; element (i,k) of A at A + i*sAm + k*sAk,
 *            element (k,j) of B at B + k*sBk + j*sBn (strides in elements,
 *            any values: row-major, transposed views such as w.t(), padded rows).
 *   C        device pointer, element (i,j) at C + i*sCm + j*sCn, type c_dtype.
 *   chunked  1: chunked FP16 accumulate + flag + redo (kernel.py:48-49,70-71,75-81);
 *            0: plain FP32 accumulate (kernel.py:50-51).
 *   workspace, ws_bytes  device scratch of f16acc_workspace_bytes(M,N,K) bytes,
 *            16-byte aligned; holds the per-tile overflow flags (16 bytes per
 *            128x128 tile, the minimum accepted) and the tail split's counters
 *            and partial tiles (f16acc_set_tail_split).  It may be
 *            uninitialised and must stay untouched until the call's work on
 *            `stream` is done.  Unused (may be NULL) when chunked == 0.
 *   device   CUDA ordinal that owns A, B, C and the workspace.
 * K == 0 writes zeros; M == 0 or N == 0 does nothing.
 */
int f16acc_gemm(const void *A, int64_t sAm, int64_t sAk,
                const void *B, int64_t sBk, int64_t sBn,
                void *C, int64_t sCm, int64_t sCn, int c_dtype,
                int64_t M, int64_t N, int64_t K, int chunked,
                void *workspace, size_t ws_bytes, int device, void *stream);

/* Bytes of workspace f16acc_gemm needs for an M x N x K product (kernel.py:94-95:
 * the flags, sized for the smallest tile any variant uses), plus, when K is
 * long enough for a tail split, room for its counters and at most 148 FP32
 * partial tiles of 64 KB (about 9.5 MB). */
size_t f16acc_workspace_bytes(int64_t M, int64_t N, int64_t K);

/* Static message for a return code (the ValueError texts of kernel.py:87-90). */
const char *f16acc_strerror(int code);

/* ---- additions with no counterpart in the reference ---------------------- */

/* f16acc_gemm with a forced kernel variant (F16ACC_VARIANT_*): the warp-level
 * mma.sync variant is measured against the tcgen05 one through this call. */
int f16acc_gemm_ex(const void *A, int64_t sAm, int64_t sAk,
                   const void *B, int64_t sBk, int64_t sBn,
                   void *C, int64_t sCm, int64_t sCn, int c_dtype,
                   int64_t M, int64_t N, int64_t K, int chunked,
                   void *workspace, size_t ws_bytes, int device, void *stream,
                   int variant);

/* The two launches f16acc_gemm_ex makes, one call each (the reference's two
 * launches, kernel.py:99 `_gemm` and kernel.py:100-104 `_redo`):
 * f16acc_gemm_main writes C and, when chunked, the per-tile flags into the
 * workspace; f16acc_gemm_redo, issued later on the same stream with the same
 * arguments and workspace, recomputes the flagged tiles with FP32
 * accumulation (a no-op when chunked == 0).  Main followed by redo is exactly
 * f16acc_gemm_ex; splitting them lets a caller time or schedule each pass. */
int f16acc_gemm_main(const void *A, int64_t sAm, int64_t sAk,
                     const void *B, int64_t sBk, int64_t sBn,
                     void *C, int64_t sCm, int64_t sCn, int c_dtype,
                     int64_t M, int64_t N, int64_t K, int chunked,
                     void *workspace, size_t ws_bytes, int device, void *stream,
                     int variant);
int f16acc_gemm_redo(const void *A, int64_t sAm, int64_t sAk,
                     const void *B, int64_t sBk, int64_t sBn,
                     void *C, int64_t sCm, int64_t sCn, int c_dtype,
                     int64_t M, int64_t N, int64_t K, int chunked,
                     void *workspace, size_t ws_bytes, int device, void *stream,
                     int variant);

/* C[M,N] = A[M,K] @ B[K,N] + bias[N] with the bias added in the epilogue of
 * both passes.  Replaces patch.py:28-30 (`y = mm(x2, w.t()); y += b`, a
 * second full read and write of y): the product is rounded to c_dtype, the
 * FP16 bias (element stride sbias) added in FP32 and the sum rounded again,
 * so C is bit-identical to the unfused mm + in-place add.  Flags and the redo
 * pass see the product only (the bias cannot raise a flag, as in the
 * reference).  bias must be non-NULL unless M or N is 0; other arguments as
 * f16acc_gemm_ex. */
int f16acc_gemm_bias(const void *A, int64_t sAm, int64_t sAk,
                     const void *B, int64_t sBk, int64_t sBn,
                     const void *bias, int64_t sbias,
                     void *C, int64_t sCm, int64_t sCn, int c_dtype,
                     int64_t M, int64_t N, int64_t K, int chunked,
                     void *workspace, size_t ws_bytes, int device, void *stream,
                     int variant);

/* Fused GEMM + all-gather for an N-column-sharded product (no reference
 * counterpart; the reference is single-GPU).  This rank computes
 * A[M,K] @ B_shard[K,N] and stores every finished tile into n_outs output
 * blocks with identical strides: outs[0] is this GPU's block, outs[1..] are
 * the same block inside other GPUs' output buffers, mapped into this process
 * (peer memory written over NVLink by plain stores, tile by tile while the
 * product runs).  Typically each rank's outs[i] points at column offset
 * rank * N of rank i's full [M, world * N] row-major C.  Chunked mode's redo
 * pass rewrites its tiles in every output.  tcgen05 operands only (else
 * F16ACC_ERR_UNSUPPORTED); n_outs <= 8.  The caller synchronises the ranks
 * (a barrier after the call on each) before reading the gathered C. */
int f16acc_gemm_allgather(const void *A, int64_t sAm, int64_t sAk,
                          const void *B, int64_t sBk, int64_t sBn,
                          void *const *outs, int n_outs, int64_t sCm, int64_t sCn, int c_dtype,
                          int64_t M, int64_t N, int64_t K, int chunked,
                          void *workspace, size_t ws_bytes, int device, void *stream);

/* What f16acc_gemm_ex would run for these operands in chunked mode, without
 * launching: variant (F16ACC_VARIANT_TCGEN05 or _MMA_SYNC), output tile shape,
 * and the tile grid of the flags (flag slot of tile (tm, tn) = tm * tiles_n +
 * tn, each slot f16acc_flag_bytes_per_tile() bytes, non-zero bytes =
 * flagged).  A chunked == 0 call on the tcgen05 variant with N >= 256 may run
 * on 128x256 tiles (f16acc_set_fp32_tiles); it writes no flags. */
typedef struct f16acc_plan {
    int variant;
    int tile_m, tile_n;
    int64_t tiles_m, tiles_n;
} f16acc_plan;
int f16acc_get_plan(const void *A, int64_t sAm, int64_t sAk,
                    const void *B, int64_t sBk, int64_t sBn,
                    int64_t M, int64_t N, int64_t K, int variant, f16acc_plan *out);
int f16acc_flag_bytes_per_tile(void);

/* tcgen05 tile configuration for later calls, process-wide: output columns
 * per tile (128) and epilogue column slices per TMEM lane quarter (2 or 4,
 * i.e. 8 or 16 epilogue warps; 0 = the default, 2 for chunked accumulation
 * and 4 for FP32 accumulation).  It does not apply to the 128x256 tiles of
 * chunked == 0 calls.  A tuning knob; results do not depend on it. */
int f16acc_set_tc_config(int tile_n, int epi_split);

/* Cap the SMs a GEMM launch occupies, process-wide, for later calls (0 = all
 * SMs, the default).  The GEMM kernels are persistent (one CTA per SM); a cap
 * leaves SMs free for kernels on other streams, such as an NCCL collective
 * that overlaps a sharded product.  The tail split (f16acc_set_tail_split)
 * plans for the capped SM count, so with it on a cap can change which tiles
 * are split and the last bits of their FP32 sums.  Returns the previous cap. */
int f16acc_set_sm_limit(int max_sms);

/* Where a chunked tcgen05 call (f16acc_gemm, _ex, _bias, _allgather,
 * _noalloc) redoes its flagged tiles, process-wide, for later calls:
 * F16ACC_REDO_INLINE (the default) = inside the main kernel, each CTA
 * recomputing its own flagged tiles in FP32 mode after its main tiles, one
 * launch in all; F16ACC_REDO_SEPARATE = the reference's shape, a second
 * launch over the flags (kernel.py:100-104).  Results are bit-identical either
 * way.  f16acc_gemm_main / _redo always make the two separate launches.
 * Returns the previous mode. */
#define F16ACC_REDO_SEPARATE 0
#define F16ACC_REDO_INLINE 1
int f16acc_set_redo_mode(int mode);

/* Tile order of the chunked tcgen05 main pass, process-wide, for later calls:
 * F16ACC_SCHEDULE_DYNAMIC (the default) launches one CTA per output tile and
 * lets each running CTA take over the tiles of CTAs not started yet (sm_100
 * cluster launch control), so CTAs that spend time on in-kernel redo work take
 * fewer main tiles; F16ACC_SCHEDULE_STATIC runs one persistent CTA per SM over
 * a fixed round-robin share.  A cap set with f16acc_set_sm_limit implies the
 * static order.  Results are bit-identical either way.  Returns the previous
 * order. */
#define F16ACC_SCHEDULE_STATIC 0
#define F16ACC_SCHEDULE_DYNAMIC 1
int f16acc_set_schedule(int mode);

/* Tile width of FP32-mode calls (chunked == 0), process-wide, for later
 * calls: F16ACC_FP32_TILES_AUTO (the default) takes 128x256 tiles
 * when N >= 256 and they finish in fewer modelled tile-times than 128x128
 * ones (a wide tile costs about 1.5 narrow ones), F16ACC_FP32_TILES_WIDE takes
 * them whenever N >= 256, F16ACC_FP32_TILES_NARROW never.  Every output
 * element gets the same K16 MMA sequence either way, so results are
 * bit-identical.  Returns the previous setting. */
#define F16ACC_FP32_TILES_AUTO 0
#define F16ACC_FP32_TILES_WIDE 1
#define F16ACC_FP32_TILES_NARROW 2
int f16acc_set_fp32_tiles(int mode);

/* Tail split of chunked tcgen05 calls, process-wide, for later calls.  With
 * F16ACC_TAIL_SPLIT_ON (the default) the tiles past the last full wave of the
 * SMs (every tile when there are fewer tiles than SMs) are each computed as up
 * to 4 units over contiguous shares of K, so they spread over the idle SMs; the
 * unit that finishes last adds the units' FP32 partials in K order (the result
 * does not depend on which unit that is) and flags the tile on the total.
 * Within a split tile the FP32 sum is formed per K share and the shares added,
 * so those tiles can differ from F16ACC_TAIL_SPLIT_OFF in the last bits of the
 * FP32 sum; flags, redone tiles and every other tile are identical.  The split
 * needs the workspace size f16acc_workspace_bytes() reports (a workspace that
 * only holds the flags runs without it).  Returns the previous setting. */
#define F16ACC_TAIL_SPLIT_OFF 0
#define F16ACC_TAIL_SPLIT_ON 1
int f16acc_set_tail_split(int mode);

/* Raw-rate probes, the B200 counterparts of the reference's bench/rate.py and
 * bench/chunkrate.py (measurement aids).  tcgen05 modes: `grid` CTAs (one per
 * SM) each run `chunks` 32-long chunks of 128x128 MMAs on a fixed
 * shared-memory tile; mode 0 = MMA only, FP16 accumulator; 1 = MMA only, FP32
 * accumulator; 2 = the GEMM kernel's chunk-pair pipeline (MMA + TMEM load +
 * one FP32 add per element) with epi_split 2 or 4 (8 or 16 epilogue warps).
 * Warp-level mma.sync modes (`grid` blocks of 8 warps, `chunks` iterations of
 * 8 independent m16n8k16 products per warp on register operands): 30 = FP16
 * accumulate, 31 = FP32 accumulate, 32 = FP16 chunks of two K16 steps added
 * into FP32.  `out` is device memory for grid * (96 + 128 * epi_split) floats
 * (grid * 256 for modes 30-32).  Asynchronous on `stream`; time it with
 * events. */
int f16acc_probe_chunk_rate(int mode, int epi_split, int chunks, int grid, void *out, int device, void *stream);

/* Self-test of the bounded waits every kernel here uses (no counterpart in
 * the reference): one CTA waits on a barrier that nothing arrives on, gives up
 * after limit_ns nanoseconds (0 < limit_ns <= 4e9), records status 0x104 in
 * the device status word and stops the CTA's other waiters through its abort
 * flag, as a product kernel does when a wait runs out.  `out` is device memory
 * for 3 uint64: the nanoseconds waited, the number of other waiters (64) that
 * left on the abort flag, and 1 if the wait wrongly reported success.  The
 * status word stays set until f16acc_device_status(device, 1) resets it. */
int f16acc_selftest_wait_timeout(uint64_t limit_ns, void *out, int device, void *stream);

/* Device status word: 0, or the code of the first wait a kernel on `device`
 * gave up on since the last reset.  Synchronises the device.  reset != 0
 * clears it.  Returns -1 when the status cannot be read. */
int f16acc_device_status(int device, int reset);

/* f16acc_gemm for callers that cannot allocate device memory.  No counterpart
 * in the reference.  Same arguments as f16acc_gemm minus the workspace: the
 * per-tile overflow flags go to a fixed array compiled into the library
 * (F16ACC_NOALLOC_MAX_TILES tiles of 128 x 128, 1 MiB on every GPU that loads
 * the library, held until the process exits), so the call allocates nothing.
 * For callers that have no device allocator (a plain C or FFI host program
 * holding raw pointers) or must not call cudaMalloc on this path (it can
 * synchronise the device and can fail under memory pressure).
 * Limit: a chunked call whose output needs more than F16ACC_NOALLOC_MAX_TILES
 * tiles (e.g. beyond 32768 x 32768) returns F16ACC_ERR_TOO_LARGE without
 * launching.  The first chunked call on a device looks up the array's device
 * address (cudaGetSymbolAddress, with that device current) and must come
 * before any stream capture on that device.  All calls share the array, which
 * keeps the last call's flags; nothing needs clearing, because every chunked
 * main pass rewrites all flag bytes of the tiles it covers before they are
 * read.  The array holds flags only, so these calls run without the tail split
 * (f16acc_set_tail_split): their results equal f16acc_gemm's with
 * F16ACC_TAIL_SPLIT_OFF.  Calls whose work overlaps on the GPU (other streams, other host
 * threads) race on the array and must be serialised.  After a kernel gave up
 * on a wait (f16acc_device_status non-zero) the output of that call and the
 * array's flags are undefined until the status word is reset. */
#define F16ACC_NOALLOC_MAX_TILES 65536
int f16acc_gemm_noalloc(const void *A, int64_t sAm, int64_t sAk,
                        const void *B, int64_t sBk, int64_t sBn,
                        void *C, int64_t sCm, int64_t sCn, int c_dtype,
                        int64_t M, int64_t N, int64_t K, int chunked,
                        int device, void *stream);

/* Library build identification (static string). */
const char *f16acc_version(void);

#ifdef __cplusplus
}
#endif

#endif /* F16ACC_H_ */
