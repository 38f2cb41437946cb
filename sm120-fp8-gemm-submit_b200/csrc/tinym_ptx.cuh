// tinym_ptx.cuh -- hand-written sm_100a PTX primitives for the tiny-M FP8 GEMM.
//
// Covers what the reference's primitive layer covers
// (include/fp8_gemm_tinym.cuh:48-283: TMA tile loads, mbarriers, proxy
// fence, swizzle math, FP8 widening) but for the Blackwell datacenter
// pipeline: TMA -> mbarrier ring -> tcgen05.mma with the accumulator in
// tensor memory (TMEM) -> tcgen05.ld epilogue, plus cluster (DSMEM)
// primitives for the split-K reduction.  Every bulk copy here targets only
// the issuing CTA's own shared memory.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace tinym {

// ---------------------------------------------------------------- basics
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// ---------------------------------------------------------------- dependent launch
// Block until the grids this one depends on (programmatic stream
// serialisation) have completed and their memory is visible; a no-op when
// the kernel was launched without the attribute.
__device__ __forceinline__ void grid_dependency_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
// Allow the next dependent grid in the stream to be scheduled.
__device__ __forceinline__ void grid_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Make mbarrier initialisation visible to the async proxy (TMA, tcgen05)
// and to the other CTAs of the cluster.
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait state shared by the roles of one CTA.  A wait that exceeds
// timeout_ns sets *abort (shared memory) and ORs `code` into the device
// error word; every other wait of the CTA then gives up within a few
// iterations, so the CTA always reaches its teardown.
struct WaitGuard {
    volatile uint32_t* abort;  // shared-memory flag
    uint32_t* err_word;        // global error word (may be null)
    uint64_t timeout_ns;
    uint32_t* err_host;        // host-mapped pending-error word (may be null)
};

// Report a wait that ran out: the device error word, and the host-mapped
// word that the host reads without synchronising (system scope).
__device__ __forceinline__ void report_timeout(uint32_t* err_word, uint32_t* err_host,
                                               uint32_t code) {
    if (err_word) atomicOr(err_word, code);
    if (err_host) atomicOr_system(err_host, code);
}

__device__ __noinline__ bool mbar_wait_slow(uint32_t bar, uint32_t parity, const WaitGuard& g,
                                            uint32_t code, bool honour_abort) {
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 31u) == 0) {
            if (honour_abort && *g.abort) return false;
            if (globaltimer_ns() - t0 > g.timeout_ns) {
                *g.abort = 1u;
                report_timeout(g.err_word, g.err_host, code);
                return false;
            }
        }
    }
}

// Returns true when the phase with parity `parity` has completed; false if
// the CTA is aborting or this wait timed out.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const WaitGuard& g,
                                          uint32_t code) {
    if (mbar_try_wait(bar, parity)) return true;
    return mbar_wait_slow(bar, parity, g, code, true);
}

// The same bounded wait, inlined at the call site: for waits on the
// output path with many live registers (no call, so nothing is saved to and
// reloaded from the stack around it).
__device__ __forceinline__ bool mbar_wait_inline(uint32_t bar, uint32_t parity, const WaitGuard& g,
                                                 uint32_t code, bool honour_abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 31u) == 0) {
            if (honour_abort && *g.abort) return false;
            if (globaltimer_ns() - t0 > g.timeout_ns) {
                *g.abort = 1u;
                report_timeout(g.err_word, g.err_host, code);
                return false;
            }
        }
    }
}

// Teardown variant: ignores the abort flag (used to drain copies or MMAs
// that are still in flight before shared/tensor memory is released).
__device__ __forceinline__ bool mbar_drain(uint32_t bar, uint32_t parity, const WaitGuard& g,
                                           uint32_t code) {
    if (mbar_try_wait(bar, parity)) return true;
    return mbar_wait_slow(bar, parity, g, code, false);
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled bulk tensor copy global -> shared (this CTA), completing its
// bytes on `bar`.  c0 is the innermost (K, bytes) coordinate and must be a
// multiple of 16; c1 is the row.  Out-of-range boxes are zero-filled.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int32_t c0, int32_t c1, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "l"(policy)
        : "memory");
}

// 3-D tiled bulk tensor copy global -> shared (this CTA); c0 innermost.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int32_t c0, int32_t c1, int32_t c2, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
        : "memory");
}

// L2 eviction policies for the streamed weight (read once) and the
// activation (re-read by every CTA).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Build-time tuning knob: L2 priority of the streamed W tiles
// (1 = evict_first, the default; 0 = evict_normal).
#ifndef TINYM_W_EVICT_FIRST
#define TINYM_W_EVICT_FIRST 1
#endif
__device__ __forceinline__ uint64_t l2_policy_w() {
    return TINYM_W_EVICT_FIRST ? l2_policy_evict_first() : l2_policy_evict_normal();
}

// ---------------------------------------------------------------- tcgen05
// Tensor-memory allocation (whole warp, .sync.aligned).  The allocated base
// address is written to shared memory at dst.
__device__ __forceinline__ void tmem_alloc(uint32_t dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand stored with the
// 128-byte swizzle: rows of 128 bytes, 8-row (1024-byte) swizzle atoms
// stacked at a stride of 1024 bytes (SBO).  Bit layout: start address>>4
// [0,14), leading byte offset>>4 [16,30) (1 = unused for swizzled K-major),
// stride byte offset>>4 [32,46), fixed version 1 at [46,48), base offset
// [49,52) = 0 (atoms are 1024-byte aligned), swizzle mode [61,64) = 2
// (128B).  Advancing the start address by 32 bytes steps K by one MMA.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

// Instruction descriptor for tcgen05.mma kind::f8f6f4: D=F32 [4,6)=1,
// A=E4M3 [7,10)=0, B=E4M3 [10,13)=0, both K-major [15],[16]=0,
// N>>3 at [17,23), M>>4 at [24,29).
__host__ __device__ constexpr uint32_t idesc_e4m3_f32(int mma_m, int mma_n) {
    return (1u << 4) | (static_cast<uint32_t>(mma_n >> 3) << 17) |
           (static_cast<uint32_t>(mma_m >> 4) << 24);
}

// One lane of the (converged) warp, chosen by the hardware: the issuing
// lane of the tcgen05.mma / commit sequence.  Issuing from a converged warp
// under elect.sync, with descriptors derived from warp-uniform values, keeps
// the issue loop on the uniform datapath: measured ~40 cycles per
// 128x16x32 E4M3 MMA on B200, against ~70 for the same loop run by lane 0
// alone with per-MMA descriptor construction.
__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "elect.sync _|P, 0xffffffff;\n\t"
        "selp.u32 %0, 1, 0, P;\n\t}\n"
        : "=r"(pred));
    return pred != 0;
}

// D[tmem] (+)= A[smem] * B[smem]^T, one elected thread, asynchronous.
__device__ __forceinline__ void umma_e4m3(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive (once) on `bar` when every tcgen05 op issued so far by this
// thread has completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
        : "memory");
}

// 32 lanes x 8 / 16 consecutive 32-bit columns: thread t of the warp gets
// TMEM lane (addr.lane + t), columns addr.col .. +7 / +15.
__device__ __forceinline__ void tmem_ld_x8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld_x16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// ---------------------------------------------------------------- cluster / DSMEM
// Address of the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t dsmem_map(uint32_t local_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void dsmem_st_f32(uint32_t cluster_addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(cluster_addr), "f"(v) : "memory");
}
// Asynchronous 16-byte store into another CTA's shared memory (cluster
// address from dsmem_map); its bytes complete on the mbarrier at the
// cluster address `remote_bar` in the destination CTA.
__device__ __forceinline__ void st_async_v4(uint32_t cluster_addr, const float (&v)[4],
                                            uint32_t remote_bar) {
    asm volatile(
        "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, "
        "[%5];" ::"r"(cluster_addr),
        "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "r"(remote_bar)
        : "memory");
}

__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- system scope (peer GPUs)
// Release fence at system scope, then relaxed adds: the release pattern for
// counters that may live in another GPU's memory.
__device__ __forceinline__ void fence_acq_rel_sys() {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
}
__device__ __forceinline__ void red_relaxed_sys_add_u64(unsigned long long* addr,
                                                        unsigned long long v) {
    asm volatile("red.relaxed.sys.global.add.u64 [%0], %1;" ::"l"(addr), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* addr) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(addr) : "memory");
    return v;
}

// ---------------------------------------------------------------- FP8 widening
// Two E4M3 codes (low 16 bits) -> two floats, exactly, via CUDA's
// fp8x2 -> half2 conversion intrinsic.
__device__ __forceinline__ float2 e4m3x2_to_f32x2(uint32_t packed16) {
    __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(
        static_cast<__nv_fp8x2_storage_t>(packed16 & 0xFFFFu), __NV_E4M3);
    return __half22float2(__half2(h));
}

}  // namespace tinym
