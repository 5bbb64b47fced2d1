// ptx.cuh -- thin inline-PTX wrappers for sm_100a: mbarriers, TMA, tcgen05
// (TMEM allocation, UMMA issue/commit, TMEM loads), grid-dependency control
// and bounded waits.  Everything here is hand written against the public PTX
// ISA; no library kernels are involved.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>

namespace f16acc {

// Device-side error codes written to the library's status word.  A kernel
// that gives up on a wait records one of these and leaves its loops; it never
// traps.
enum DeviceStatus : int {
    kStatusOk = 0,
    kStatusTimeoutProducer = 0x101,   // TMA producer waited too long for a free smem stage
    kStatusTimeoutMma = 0x102,        // MMA warp waited too long for data or a free TMEM buffer
    kStatusTimeoutEpilogue = 0x103,   // epilogue waited too long for an accumulator
    kStatusTimeoutProbe = 0x104,      // a probe or self-test kernel's wait ran out
    kStatusTimeoutSchedule = 0x105,   // the tile scheduler waited too long for the epilogue's flag decisions
    kStatusRedoQueueFull = 0x106,     // in-kernel redo queue overflow (a bug; the kernel stops)
    kStatusTimeoutStore = 0x107,      // store warps waited too long for a staged tile
};

// A wait gives up after this many nanoseconds of %globaltimer.  The longest
// legitimate wait is one tile's K loop (well under 100 ms even for K = 2^20).
constexpr uint64_t kWaitLimitNs = 4000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbarrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Wait for the phase with the given parity to complete.  Bounded: gives up
// after limit_ns (kWaitLimitNs in every product kernel; the wait self-test
// passes a short one), or at once when another thread of the CTA has already
// given up (*abort != 0).  On giving up it records `code` in *status and
// sets *abort.  Returns false when it gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* status,
                                          int code, uint64_t limit_ns = kWaitLimitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 0u) {
            if (*abort) return false;
            if (globaltimer_ns() - t0 > limit_ns) {
                atomicCAS(status, 0, code);
                *abort = 1;
                return false;
            }
        }
    }
}

// Named CTA barriers (IDs 1..15; 0 is __syncthreads).  `threads` counts every
// thread of the participating warps; both are executed by whole warps.
// bar.arrive marks arrival without waiting (release); bar.sync waits until
// `threads` arrivals (acquire).  A bar.sync has no time limit, so callers
// must guarantee that the arrivals it needs always come.
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void named_bar_arrive(int id, int threads) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Wait bounded by `limit_ns` of %globaltimer only (no abort flag): true when
// the phase completed in time.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer_ns() - t0 > limit_ns) return false;
    }
    return true;
}

// Wait used while shutting down after an abort: bounded by time only, so a
// CTA can let its own in-flight copies and MMAs land before it exits.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
    return true;
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* tm) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}
// 2-D tiled bulk tensor load global -> shared, completion counted on `bar`.
// c0 is the innermost coordinate (elements).  One destination CTA: this one.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, uint64_t* bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

// 2-D tiled bulk tensor store shared -> global (bulk-group completion).  c0 is
// the innermost coordinate; elements outside the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* tm, const void* src, int c0, int c1) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(tm)),
                 "r"(smem_u32(src)), "r"(c0), "r"(c1)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until every committed bulk store of this thread has read its shared-memory source.
__device__ __forceinline__ void bulk_wait_group_read0() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Wait until every committed bulk store of this thread has completed.
__device__ __forceinline__ void bulk_wait_group0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// A read-only global FP16 load and a 16-byte shared store as volatile asm:
// kept in program order with each other (bounds register live ranges).
__device__ __forceinline__ __half ldg_half_ordered(const __half* p) {
    unsigned short v;
    asm volatile("ld.global.nc.b16 %0, [%1];" : "=h"(v) : "l"(p));
    return __ushort_as_half(v);
}
__device__ __forceinline__ void st_shared_v4_ordered(void* p, uint4 v) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(p)), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

// Order this thread's generic-proxy shared-memory writes before later async-proxy
// (TMA) accesses to them.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05
// TMEM allocation: executed by one whole warp; the base address lands in smem.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (f16 inputs, f16 or f32 D
// per the instruction descriptor).  accumulate == 0 overwrites D.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on `bar` once every tcgen05 op issued so far by this thread is done.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 columns of 32-bit words -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
// 32 lanes x 64 columns of 16-bit values, two adjacent columns packed per
// register -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x32_pack16(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.pack::16b.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
// 32 lanes x 32 columns of 16-bit values, packed -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x16_pack16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.pack::16b.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// Shared-memory matrix descriptor (tcgen05 form): 128-byte swizzle, start
// address / leading byte offset / stride byte offset in 16-byte units,
// descriptor version 1 at bits 46-47, base offset 0 (tiles are 1024-byte
// aligned), swizzle mode 2 (128B) at bits 61-63.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(2) << 61;
    return d;
}

// Instruction descriptor for tcgen05.mma kind::f16 with f16 A and B:
// bits 4-5 D format (0 f16, 1 f32), 7-9 / 10-12 A / B format (0 = f16),
// 15 / 16 A / B major (0 K-major, 1 MN-major), 17-22 N >> 3, 24-28 M >> 4.
__host__ __device__ constexpr uint32_t idesc_f16(bool d_f32, bool b_mn_major, int m, int n) {
    return (d_f32 ? 1u : 0u) << 4 | (b_mn_major ? 1u : 0u) << 16 | static_cast<uint32_t>(n >> 3) << 17 |
           static_cast<uint32_t>(m >> 4) << 24;
}

// ---------------------------------------------------------------- grid dependency control (PDL)
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- dynamic tile scheduling
// Cluster launch control (sm_100): ask the hardware to cancel one CTA of this
// grid that has not started yet; the 16-byte response lands in `resp16` (smem,
// 16-byte aligned) and completes 16 bytes of transaction on `bar`, which the
// caller armed with mbar_arrive_expect_tx(bar, 16).  Never issued again after
// a response that reports failure.
__device__ __forceinline__ void clc_try_cancel(void* resp16, uint64_t* bar) {
    asm volatile("clusterlaunchcontrol.try_cancel.async.shared::cta.mbarrier::complete_tx::bytes.b128 [%0], [%1];" ::"r"(
                     smem_u32(resp16)),
                 "r"(smem_u32(bar))
                 : "memory");
}
// Decode a landed response: true and the cancelled CTA's blockIdx.x (whose work
// the caller now owns), or false when no CTA was left to cancel.
__device__ __forceinline__ bool clc_query(const void* resp16, uint32_t& ctaid_x) {
    uint32_t ok, x = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t.reg .b128 r;\n\t"
        "ld.shared.b128 r, [%2];\n\t"
        "clusterlaunchcontrol.query_cancel.is_canceled.pred.b128 p, r;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t"
        "@p clusterlaunchcontrol.query_cancel.get_first_ctaid::x.b32.b128 %1, r;\n\t"
        "}"
        : "=r"(ok), "+r"(x)
        : "r"(smem_u32(resp16))
        : "memory");
    ctaid_x = x;
    return ok != 0;
}

// ---------------------------------------------------------------- arithmetic
// acc += (float)h for the two FP16 halves of `packed` (low half -> a0).  One
// mixed-precision FP32 add per element (PTX add.f32.f16, sm_100+): the FP16
// value converts exactly, the add rounds to nearest in FP32.
__device__ __forceinline__ void add_f16x2_to_f32(float& a0, float& a1, uint32_t packed) {
    asm("{\n\t.reg .f16 lo, hi;\n\t"
        "mov.b32 {lo, hi}, %2;\n\t"
        "add.rn.f32.f16 %0, lo, %0;\n\t"
        "add.rn.f32.f16 %1, hi, %1;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "r"(packed));
}

// The first chunk of a tile: acc = (float)h + 0 for both halves, the value of
// the mixed add into a zeroed accumulator (signed zeros included) without the
// zeroing.
__device__ __forceinline__ void init_f16x2_to_f32(float& a0, float& a1, uint32_t packed) {
    asm("{\n\t.reg .f16 lo, hi;\n\t"
        "mov.b32 {lo, hi}, %2;\n\t"
        "add.rn.f32.f16 %0, lo, 0f00000000;\n\t"
        "add.rn.f32.f16 %1, hi, 0f00000000;\n\t}"
        : "=f"(a0), "=f"(a1)
        : "r"(packed));
}

// Non-finite test used for the tile flag: fma(x, 0, s) stays 0 for finite x
// and turns NaN for +-inf and NaN, so one NaN check at the end of a tile
// covers every element (|x| < inf is false exactly when x is inf or NaN).
__device__ __forceinline__ float nonfinite_probe(float s, float x) { return __fmaf_rn(x, 0.0f, s); }

}  // namespace f16acc
