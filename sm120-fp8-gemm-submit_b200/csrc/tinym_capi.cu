// tinym_capi.cu -- host launcher, shape-dispatch table and C ABI.
//
// Replaces the reference's launch plumbing (include/fp8_gemm_tinym.cuh:
// 79-132 tensor-map encoding, 724-808 ::run, 810-824 the cudaError_t
// wrapper) and the shape gate / template dispatch of
// src/torch_candidate_extension.cu:33-81.  Differences that matter on B200:
//   * shapes are runtime values and the dispatch table is a function of
//     (M, N, K, SM count) instead of six hard-coded template instances;
//   * TMA descriptors are cached per (pointer, shape) instead of being
//     re-encoded on every call (reference :742-755, :794-799), and the
//     shared-memory attribute is set once per device (reference :769-770);
//   * alpha may stay on the device (no host synchronisation);
//   * errors come back as status codes with a per-thread message, never as
//     exceptions.
// cuTensorMapEncodeTiled is fetched through cudaGetDriverEntryPoint, so the
// library links only the static CUDA runtime and loads on machines without
// a GPU driver (its entry points then return TINYM_ERR_CUDA).
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cmath>
#include <cstring>
#include <mutex>

#include "../../include/tinym_b200.h"
#include "tinym_kernels.cuh"
#include "tinym_quant.cuh"

namespace {

using tinym::kBlockK;
using tinym::kMaxSplit;  // portable cluster size
using tinym::kTcThreads;
using tinym::kTileRows;
using tinym::TinymParams;

constexpr int kMaxDevices = 64;
constexpr int kMaxStages = 32;
constexpr int kSmemLimit = 232448; // 227 KiB opt-in per CTA on sm_100
constexpr uint64_t kDefaultTimeoutNs = 1000000000ull;  // 1 s per wait

// Build-time knob: launch with programmatic dependent launch (1, default).
#ifndef TINYM_USE_PDL
#define TINYM_USE_PDL 1
#endif
constexpr bool kUsePdl = TINYM_USE_PDL != 0;

// Build-time tuning knob: L2 sector promotion of the TMA tensor maps.
#ifndef TINYM_L2_PROMOTION
#define TINYM_L2_PROMOTION CU_TENSOR_MAP_L2_PROMOTION_L2_256B
#endif

thread_local char t_last_error[512] = "";

int fail(int status, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
    va_end(ap);
    return status;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(TINYM_ERR_CUDA, "%s failed: %s (%s)", what, cudaGetErrorName(e),
                cudaGetErrorString(e));
}

// ---------------------------------------------------------------- driver entry point
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
cudaError_t g_encode_err = cudaSuccess;

// cuMemGetAddressRange (driver API, fetched like the encoder): the base of
// the allocation that holds a pointer, for CUDA IPC export.
using AddrRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
AddrRangeFn get_addr_range() {
    static std::once_flag once;
    static AddrRangeFn fn_ptr = nullptr;
    std::call_once(once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn_ptr = reinterpret_cast<AddrRangeFn>(fn);
    });
    return fn_ptr;
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        g_encode_err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
        if (g_encode_err == cudaSuccess && q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    return g_encode;
}

// ---------------------------------------------------------------- per-device state
struct DeviceInfo {
    std::atomic<int> ready{0};
    int sm_count = 0;
    int cc_major = 0, cc_minor = 0;
    std::atomic<uint32_t> attr_done{0};  // bit per kernel instance: smem attribute set
    // Pending-error word: one pinned, device-mapped host word per device.
    // Kernels whose bounded waits run out OR their bit into it (system
    // scope), so the host sees a timeout at its next call without
    // synchronising.  Allocated on the first GEMM call of the device.
    std::atomic<volatile uint32_t*> err_host{nullptr};
    uint32_t* err_host_dev = nullptr;
};
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

int device_info(int dev, DeviceInfo** out) {
    if (dev < 0 || dev >= kMaxDevices) return fail(TINYM_ERR_CUDA, "device ordinal %d out of range", dev);
    DeviceInfo& d = g_dev[dev];
    if (!d.ready.load(std::memory_order_acquire)) {
        std::lock_guard<std::mutex> lk(g_dev_mu);
        if (!d.ready.load(std::memory_order_relaxed)) {
            cudaError_t e;
            if ((e = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
                return cuda_fail(e, "cudaDeviceGetAttribute(MultiProcessorCount)");
            if ((e = cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess)
                return cuda_fail(e, "cudaDeviceGetAttribute(ComputeCapabilityMajor)");
            if ((e = cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess)
                return cuda_fail(e, "cudaDeviceGetAttribute(ComputeCapabilityMinor)");
            d.ready.store(1, std::memory_order_release);
        }
    }
    if (d.cc_major != 10 || d.cc_minor != 0)
        return fail(TINYM_ERR_UNSUPPORTED_DEVICE,
                    "device %d is sm_%d%d; this library is built for sm_100a (B200)", dev,
                    d.cc_major, d.cc_minor);
    *out = &d;
    return TINYM_OK;
}

// The device's pending-error word: its device address in *dev_ptr (null
// when allocate is false and the word does not exist yet).
int pending_word(DeviceInfo* d, bool allocate, uint32_t** dev_ptr) {
    *dev_ptr = nullptr;
    if (d->err_host.load(std::memory_order_acquire)) {
        *dev_ptr = d->err_host_dev;
        return TINYM_OK;
    }
    if (!allocate) return TINYM_OK;
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (!d->err_host.load(std::memory_order_relaxed)) {
        void* h = nullptr;
        cudaError_t e = cudaHostAlloc(&h, sizeof(uint32_t), cudaHostAllocMapped | cudaHostAllocPortable);
        if (e != cudaSuccess) return cuda_fail(e, "cudaHostAlloc(pending-error word)");
        *static_cast<volatile uint32_t*>(h) = 0u;
        void* dp = nullptr;
        e = cudaHostGetDevicePointer(&dp, h, 0);
        if (e != cudaSuccess) {
            cudaFreeHost(h);
            return cuda_fail(e, "cudaHostGetDevicePointer(pending-error word)");
        }
        d->err_host_dev = static_cast<uint32_t*>(dp);
        d->err_host.store(static_cast<volatile uint32_t*>(h), std::memory_order_release);
    }
    *dev_ptr = d->err_host_dev;
    return TINYM_OK;
}

// ---------------------------------------------------------------- tensor-map cache
struct MapKey {
    const void* ptr;
    int64_t rows, cols;
    int32_t box_rows, swizzle, chunks, dev, packed;
    bool operator==(const MapKey& o) const {
        return ptr == o.ptr && rows == o.rows && cols == o.cols && box_rows == o.box_rows &&
               swizzle == o.swizzle && chunks == o.chunks && dev == o.dev && packed == o.packed;
    }
};
struct MapEntry {
    MapKey key;
    alignas(64) CUtensorMap map;
    uint64_t stamp;
    bool used;
};
constexpr int kMapCacheSize = 256;
MapEntry g_maps[kMapCacheSize];
uint64_t g_map_clock = 0;
std::mutex g_map_mu;

// Encodes (or fetches) the map of a row-major [rows, cols] uint8 matrix read
// in boxes of `chunks` x [box_rows, 128 bytes]; swizzle 1 = 128B, 0 = none.
// chunks == 1: a 2-D map {cols, rows}.  chunks > 1 (cols % 128 == 0): a 3-D
// view {128, rows, cols / 128} with strides {cols, 128} whose box
// {128, box_rows, chunks} lands as `chunks` consecutive [box_rows x 128 B]
// tiles -- several K chunks per TMA instruction.
int get_map(const void* ptr, int64_t rows, int64_t cols, int box_rows, int swizzle, int chunks,
            int dev, CUtensorMap* out, int packed = 0) {
    const MapKey key{ptr, rows, cols, box_rows, swizzle, chunks, dev, packed};
    std::lock_guard<std::mutex> lk(g_map_mu);
    MapEntry* victim = &g_maps[0];
    for (auto& e : g_maps) {
        if (e.used && e.key == key) {
            e.stamp = ++g_map_clock;
            *out = e.map;
            return TINYM_OK;
        }
        if (!e.used || e.stamp < victim->stamp) victim = &e;
        if (!victim->used) break;
    }
    auto encode = get_encode();
    if (!encode)
        return fail(TINYM_ERR_CUDA, "cuTensorMapEncodeTiled unavailable (%s)",
                    cudaGetErrorString(g_encode_err));
    const bool three = chunks > 1 || packed;
    cuuint64_t dims[3], strides[2];
    cuuint32_t box[3], estr[3] = {1, 1, 1};
    if (packed) {
        // [tiles * KC chunks][kPackRows rows][128 B], chunk blocks contiguous.
        const int64_t kc = tinym::packed_chunks(cols);
        const int64_t tiles = (rows + tinym::kPackRows - 1) / tinym::kPackRows;
        dims[0] = static_cast<cuuint64_t>(kBlockK);
        dims[1] = static_cast<cuuint64_t>(tinym::kPackRows);
        dims[2] = static_cast<cuuint64_t>(tiles * kc);
        strides[0] = static_cast<cuuint64_t>(kBlockK);
        strides[1] = static_cast<cuuint64_t>(tinym::kPackRows) * kBlockK;
        box[0] = static_cast<cuuint32_t>(kBlockK);
        box[1] = static_cast<cuuint32_t>(box_rows);
        box[2] = static_cast<cuuint32_t>(chunks);
    } else if (!three) {
        dims[0] = static_cast<cuuint64_t>(cols);
        dims[1] = static_cast<cuuint64_t>(rows);
        strides[0] = static_cast<cuuint64_t>(cols);
        box[0] = static_cast<cuuint32_t>(kBlockK);
        box[1] = static_cast<cuuint32_t>(box_rows);
    } else {
        dims[0] = static_cast<cuuint64_t>(kBlockK);
        dims[1] = static_cast<cuuint64_t>(rows);
        dims[2] = static_cast<cuuint64_t>(cols / kBlockK);
        strides[0] = static_cast<cuuint64_t>(cols);
        strides[1] = static_cast<cuuint64_t>(kBlockK);
        box[0] = static_cast<cuuint32_t>(kBlockK);
        box[1] = static_cast<cuuint32_t>(box_rows);
        box[2] = static_cast<cuuint32_t>(chunks);
    }
    CUtensorMap map;
    CUresult r = encode(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, three ? 3 : 2, const_cast<void*>(ptr),
                        dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        TINYM_L2_PROMOTION, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(TINYM_ERR_CUDA,
                    "cuTensorMapEncodeTiled failed (CUresult %d) for [%lld x %lld] box %d rows",
                    static_cast<int>(r), static_cast<long long>(rows),
                    static_cast<long long>(cols), box_rows);
    victim->key = key;
    victim->map = map;
    victim->stamp = ++g_map_clock;
    victim->used = true;
    *out = map;
    return TINYM_OK;
}

// ---------------------------------------------------------------- plans
int plan_chunks(const tinym_plan& p) { return p.block_k / kBlockK; }

int w_stage_bytes(const tinym_plan& p) { return plan_chunks(p) * p.tile_m * kBlockK; }

int x_stage_bytes(const tinym_plan& p) {
    return p.kernel == TINYM_KERNEL_TC ? plan_chunks(p) * p.mma_n * kBlockK : kBlockK;
}

// Dynamic shared memory of a plan: the rings plus the split-K receive
// blocks ((split - 1) x rows owned x padded MMA_N floats for the TC kernel,
// (split - 1) x 128 floats for the SIMT kernel).
uint32_t plan_smem_bytes(const tinym_plan& p) {
    if (p.kernel == TINYM_KERNEL_TC)
        return tinym::smem_layout(p.stages, w_stage_bytes(p), x_stage_bytes(p), p.split_k,
                                  tinym::tc_red_rank_bytes(p.mma_n, p.tile_m, p.split_k))
            .bytes;
    return tinym::smem_layout(p.stages, w_stage_bytes(p), x_stage_bytes(p), p.split_k,
                              kTileRows * 4).bytes;
}

int fill_derived(int64_t m, int64_t n, int64_t k, tinym_plan* p) {
    if (p->block_k == 0) p->block_k = kBlockK;  // 0 selects the defaults
    if (p->tile_m == 0) p->tile_m = kTileRows;
    if (p->kernel != TINYM_KERNEL_TC && p->kernel != TINYM_KERNEL_SIMT_M1)
        return fail(TINYM_ERR_BAD_PLAN, "plan.kernel %d is not a kernel family", p->kernel);
    if (p->tile_m != 128 && !(p->tile_m == 64 && p->kernel == TINYM_KERNEL_TC))
        return fail(TINYM_ERR_BAD_PLAN, "plan.tile_m must be 128, or 64 for the TC kernel");
    const int64_t tiles = (n + p->tile_m - 1) / p->tile_m;
    if (p->block_k != 128 && p->block_k != 256 && p->block_k != 512)
        return fail(TINYM_ERR_BAD_PLAN, "plan.block_k must be 128, 256 or 512");
    if (p->block_k != kBlockK && (p->kernel != TINYM_KERNEL_TC || k % kBlockK != 0))
        return fail(TINYM_ERR_BAD_PLAN,
                    "plan.block_k > 128 needs the TC kernel and K %% 128 == 0 (K = %lld)",
                    (long long)k);
    const int64_t kb = (k + p->block_k - 1) / p->block_k;  // K stages
    if (p->kernel == TINYM_KERNEL_TC) {
        if (p->mma_n != 8 && p->mma_n != 16)
            return fail(TINYM_ERR_BAD_PLAN, "plan.mma_n must be 8 or 16");
        if (p->mma_n < m) return fail(TINYM_ERR_BAD_PLAN, "plan.mma_n %d < M %lld", p->mma_n, (long long)m);
        p->consumer_warps = 0;
        p->threads = kTcThreads;
    } else {
        if (m != 1) return fail(TINYM_ERR_BAD_PLAN, "the SIMT kernel handles M == 1 only");
        if (p->consumer_warps != 4 && p->consumer_warps != 8)
            return fail(TINYM_ERR_BAD_PLAN, "plan.consumer_warps must be 4 or 8");
        p->mma_n = 0;
        p->threads = 32 * (p->consumer_warps + 1);
    }
    if (p->split_k < 1 || p->split_k > kMaxSplit)
        return fail(TINYM_ERR_BAD_PLAN, "plan.split_k must be in 1..%d", kMaxSplit);
    const int64_t per = (kb + p->split_k - 1) / p->split_k;
    if ((p->split_k - 1) * per >= kb)
        return fail(TINYM_ERR_BAD_PLAN, "split_k %d leaves an empty K range (K blocks %lld)",
                    p->split_k, (long long)kb);
    if (p->stages < 2 || p->stages > kMaxStages)
        return fail(TINYM_ERR_BAD_PLAN, "plan.stages must be in 2..%d", kMaxStages);
    if (tiles > 65535) return fail(TINYM_ERR_UNSUPPORTED_SHAPE, "N too large (%lld tiles)", (long long)tiles);
    const uint32_t smem = plan_smem_bytes(*p);
    if (smem > static_cast<uint32_t>(kSmemLimit))
        return fail(TINYM_ERR_BAD_PLAN, "plan needs %u bytes of shared memory (> %d)", smem,
                    kSmemLimit);
    p->tiles_n = static_cast<int32_t>(tiles);
    p->grid_ctas = static_cast<int32_t>(tiles * p->split_k);
    p->smem_bytes = static_cast<int32_t>(smem);
    return TINYM_OK;
}

int check_shape(int64_t m, int64_t n, int64_t k) {
    if (m < 1 || n < 1 || k < 1)
        return fail(TINYM_ERR_INVALID_ARGUMENT, "M, N, K must be positive (got %lld, %lld, %lld)",
                    (long long)m, (long long)n, (long long)k);
    if (m > 16)
        return fail(TINYM_ERR_UNSUPPORTED_SHAPE, "unsupported shape M=%lld, K=%lld, N=%lld: M must be <= 16",
                    (long long)m, (long long)k, (long long)n);
    if (k % 16 != 0)
        return fail(TINYM_ERR_UNSUPPORTED_SHAPE,
                    "unsupported shape M=%lld, K=%lld, N=%lld: K must be a multiple of 16",
                    (long long)m, (long long)k, (long long)n);
    if (k > (int64_t(1) << 31) - 1024 || n > (int64_t(1) << 31) - 1)
        return fail(TINYM_ERR_UNSUPPORTED_SHAPE, "K or N exceeds the 32-bit index range");
    return TINYM_OK;
}

// Largest ring depth (>= 2) whose shared memory fits `limit` bytes, or -1
// if not even two stages fit.
int max_stages_fitting(const tinym_plan& p, uint32_t limit) {
    for (int st = kMaxStages; st >= 2; --st) {
        tinym_plan q = p;
        q.stages = st;
        if (plan_smem_bytes(q) <= limit) return st;
    }
    return -1;
}

// W bytes a CTA keeps in flight (ring depth x W stage): 128 KiB measured
// best on B200 -- deeper rings (192 KiB) lose in the single-launch protocols
// without gaining back-to-back throughput.
constexpr int kTargetRingBytes = 128 * 1024;
// Host-only flag bit (above the kernel's TinymParams::flags): the GEMM
// follows the quantise prologue, which keeps the default plan.
constexpr uint32_t kFlagQuantPrologue = 1u << 16;
// With TINYM_FLAG_STATIC_W the dispatch instead cuts the work into twice as
// many CTAs with a 64 KiB ring each (small enough for two per SM), so that
// the next GEMM's CTAs take over SMs as the previous GEMM's finish and
// stream W during its tail: measured 4-9 % more back-to-back throughput at
// M = 9 on the official points.
constexpr int kOverlapRingBytes = 64 * 1024;
// W in flight per CTA for plans with 64 KiB stages (block_k = 512).
constexpr int kWideRingBytes = 192 * 1024;
constexpr uint32_t kHalfSmSmem = (233472u - 2u * 1024u) / 2u;  // two CTAs' share of an SM

// Ring depth for a TC plan: ring_bytes of W in flight, at most what fits
// and at most the CTA's K blocks (more is useless), at least 2; -1 if not
// even two stages fit.
int tc_stages_for(const tinym_plan& p, int64_t kb_per_cta, int ring_bytes = kTargetRingBytes) {
    const int max_st = max_stages_fitting(p, static_cast<uint32_t>(kSmemLimit));
    if (max_st < 0) return -1;
    const int64_t want = std::max(2, ring_bytes / w_stage_bytes(p));
    return static_cast<int>(std::max<int64_t>(2, std::min<int64_t>({kb_per_cta, want, max_st})));
}

// Heuristic part of the dispatch table, fitted to B200 measurements of the
// official points (plan sweeps, per-CTA cycle traces):
//  * one CTA per SM with a deep ring (two CTAs per SM never won);
//  * block_k = 256 -- one 32 KiB 3-D TMA box of W per stage -- whenever
//    K % 128 == 0, else 128.  A CTA's TMA stream costs ~150 ns per box
//    whatever its size up to 32 KiB (54 GB/s per CTA with 8 KiB boxes, 106
//    with 16 KiB, ~150-190 with 32 KiB, measured with few CTAs);
//  * 128-row W tiles and the largest K split (cluster size <= 8) that keeps
//    tiles * split CTAs within one CTA per SM and gives every CTA >= 2
//    stages, with a ring of ~128 KiB of W (tc_stages_for);
//  * block_k = 512 instead (one 64 KiB box of 128 rows x 512 B per stage,
//    a ~192 KiB ring) when K % 512 == 0 and every CTA of that split keeps
//    at least four such stages: 0.3 us faster back to back and 0.25-0.5 us
//    per single launch at (1..16, 6144, 5120) than 32 KiB stages (and than
//    64-row tiles with full K), the same at N = 8192 and 16384.
// overlap = true: the TINYM_FLAG_STATIC_W variant (two CTAs per SM).
tinym_plan heuristic_plan(int64_t m, int64_t n, int64_t k, int sm_count, bool overlap = false) {
    tinym_plan p{};
    p.kernel = TINYM_KERNEL_TC;
    p.mma_n = m <= 8 ? 8 : 16;
    p.block_k = (k % kBlockK == 0) ? 2 * kBlockK : kBlockK;
    p.split_k = 1;
    p.tile_m = kTileRows;
    const int ring = overlap ? kOverlapRingBytes : kTargetRingBytes;
    const int64_t slots = static_cast<int64_t>(sm_count) * (overlap ? 2 : 1);
    const int64_t tiles = (n + p.tile_m - 1) / p.tile_m;
    const int64_t kb = (k + p.block_k - 1) / p.block_k;
    for (int s = 2; s <= kMaxSplit; ++s) {
        if (tiles * s > slots) break;
        const int64_t per = (kb + s - 1) / s;
        if (per < 2 || (s - 1) * per >= kb) continue;
        tinym_plan q = p;
        q.split_k = s;
        const int st = tc_stages_for(q, per, ring);
        if (st < 0) continue;
        if (overlap) {
            q.stages = st;
            if (plan_smem_bytes(q) > kHalfSmSmem) continue;
        }
        p.split_k = s;
    }
    p.stages = tc_stages_for(p, (kb + p.split_k - 1) / p.split_k, ring);
    if (!overlap && k % (4 * kBlockK) == 0) {
        // 64 KiB stages (one 3-D box of 128 rows x 512 B) when every CTA of
        // the split keeps at least four of them.
        tinym_plan q = p;
        q.block_k = 4 * kBlockK;
        const int64_t kb4 = k / q.block_k;
        const int64_t per4 = (kb4 + q.split_k - 1) / q.split_k;
        const int st = tc_stages_for(q, per4, kWideRingBytes);
        if (per4 >= 4 && (q.split_k - 1) * per4 < kb4 && st >= 3) {
            q.stages = st;
            p = q;
        }
    }
    return p;
}

// Kernel entry for a plan; sets the shared-memory opt-in once per device.
int kernel_for(const tinym_plan& p, DeviceInfo* di, const void** fn) {
#define TINYM_TC(N, C, T) reinterpret_cast<const void*>(&tinym::tinym_tc_kernel<N, C, T>)
    static const void* const kTc[2][3][2] = {
        {{TINYM_TC(8, 1, 64), TINYM_TC(8, 1, 128)},
         {TINYM_TC(8, 2, 64), TINYM_TC(8, 2, 128)},
         {TINYM_TC(8, 4, 64), TINYM_TC(8, 4, 128)}},
        {{TINYM_TC(16, 1, 64), TINYM_TC(16, 1, 128)},
         {TINYM_TC(16, 2, 64), TINYM_TC(16, 2, 128)},
         {TINYM_TC(16, 4, 64), TINYM_TC(16, 4, 128)}}};
#undef TINYM_TC
    uint32_t attr_bit = 0;
    if (p.kernel == TINYM_KERNEL_TC) {
        const int ni = p.mma_n == 8 ? 0 : 1;
        const int ci = p.block_k == 128 ? 0 : (p.block_k == 256 ? 1 : 2);
        const int ti = p.tile_m == 64 ? 0 : 1;
        *fn = kTc[ni][ci][ti];
        attr_bit = 1u << ((ni * 3 + ci) * 2 + ti);
    } else {
        *fn = p.consumer_warps == 4 ? reinterpret_cast<const void*>(&tinym::tinym_simt_m1_kernel<4>)
                                    : reinterpret_cast<const void*>(&tinym::tinym_simt_m1_kernel<8>);
        attr_bit = p.consumer_warps == 4 ? 1u << 12 : 1u << 13;
    }
    if (!(di->attr_done.load(std::memory_order_acquire) & attr_bit)) {
        cudaError_t e = cudaFuncSetAttribute(*fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(MaxDynamicSharedMemorySize)");
        // The whole L1/shared array as shared memory.  Plans above half an SM
        // get this carveout at launch anyway; stating it makes the occupancy
        // calculator (the launcher's residency check) count two CTAs per SM
        // for plans that fit twice instead of assuming the default carveout.
        e = cudaFuncSetAttribute(*fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 cudaSharedmemCarveoutMaxShared);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(PreferredSharedMemoryCarveout)");
        // (clusters stay within the portable size: fill_derived caps split_k at 8)
        di->attr_done.fetch_or(attr_bit, std::memory_order_acq_rel);
    }
    return TINYM_OK;
}

// Grid (split_k x tiles_n), block, shared memory, cluster attribute and
// programmatic dependent launch.  `attrs` must hold 2 entries.  With PDL
// the kernel may be scheduled while the previous kernel in the stream is
// finishing; it runs its prologue and then blocks in griddepcontrol.wait
// before touching global memory, so stream semantics are unchanged.
void launch_config(const tinym_plan& p, void* stream, cudaLaunchConfig_t* cfg,
                   cudaLaunchAttribute* attrs) {
    *cfg = cudaLaunchConfig_t{};
    cfg->gridDim = dim3(static_cast<unsigned>(p.split_k), static_cast<unsigned>(p.tiles_n), 1);
    cfg->blockDim = dim3(static_cast<unsigned>(p.threads), 1, 1);
    cfg->dynamicSmemBytes = static_cast<size_t>(p.smem_bytes);
    cfg->stream = static_cast<cudaStream_t>(stream);
    unsigned n = 0;
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = kUsePdl ? 1 : 0;
    ++n;
    if (p.split_k > 1) {
        attrs[n].id = cudaLaunchAttributeClusterDimension;
        attrs[n].val.clusterDim.x = static_cast<unsigned>(p.split_k);
        attrs[n].val.clusterDim.y = 1;
        attrs[n].val.clusterDim.z = 1;
        ++n;
    }
    cfg->attrs = attrs;
    cfg->numAttrs = n;
}

// How many clusters of this plan can be resident at once (cached).
struct ClusterOccEntry {
    const void* fn;
    int32_t split, smem, value;
};
constexpr int kOccCacheSize = 64;
ClusterOccEntry g_occ[kMaxDevices][kOccCacheSize];
int g_occ_used[kMaxDevices];
std::mutex g_occ_mu;

int max_active_clusters(const tinym_plan& p, int dev, DeviceInfo* di, int* out) {
    const void* fn = nullptr;
    int st = kernel_for(p, di, &fn);
    if (st != TINYM_OK) return st;
    {
        std::lock_guard<std::mutex> lk(g_occ_mu);
        for (int i = 0; i < g_occ_used[dev]; ++i) {
            const ClusterOccEntry& e = g_occ[dev][i];
            if (e.fn == fn && e.split == p.split_k && e.smem == p.smem_bytes) {
                *out = e.value;
                return TINYM_OK;
            }
        }
    }
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attrs[2];
    launch_config(p, nullptr, &cfg, attrs);
    int n = 0;
    if (p.split_k > 1) {
        cudaError_t e = cudaOccupancyMaxActiveClusters(&n, fn, &cfg);
        if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveClusters");
    } else {
        cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, p.threads,
                                                                      static_cast<size_t>(p.smem_bytes));
        if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
        n *= di->sm_count;
    }
    std::lock_guard<std::mutex> lk(g_occ_mu);
    if (g_occ_used[dev] < kOccCacheSize) g_occ[dev][g_occ_used[dev]++] = {fn, p.split_k, p.smem_bytes, n};
    *out = n;
    return TINYM_OK;
}

// Workspace of the no-allocation form of the fused activation path: a
// file-scope device array (one per device context), sized for M * K up to
// kNoAllocMaxElems.  Its address is taken once per device with
// cudaGetSymbolAddress.
constexpr int64_t kNoAllocMaxElems = int64_t(16) * 32768;
static __device__ __align__(256) uint8_t g_quant_scratch[tinym::kQuantWsHeader + kNoAllocMaxElems];
std::atomic<void*> g_scratch_addr[kMaxDevices];

int scratch_address(int dev, void** out) {
    void* p = g_scratch_addr[dev].load(std::memory_order_acquire);
    if (!p) {
        cudaError_t e = cudaGetSymbolAddress(&p, g_quant_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(scratch)");
        g_scratch_addr[dev].store(p, std::memory_order_release);
    }
    *out = p;
    return TINYM_OK;
}

}  // namespace

// =====================================================================
// C ABI
// =====================================================================
extern "C" {

int32_t tinym_abi_version(void) { return TINYM_ABI_VERSION; }

const char* tinym_last_error(void) { return t_last_error; }

const char* tinym_status_string(int32_t status) {
    switch (status) {
        case TINYM_OK: return "TINYM_OK";
        case TINYM_ERR_INVALID_ARGUMENT: return "TINYM_ERR_INVALID_ARGUMENT";
        case TINYM_ERR_UNSUPPORTED_SHAPE: return "TINYM_ERR_UNSUPPORTED_SHAPE";
        case TINYM_ERR_MISALIGNED: return "TINYM_ERR_MISALIGNED";
        case TINYM_ERR_CUDA: return "TINYM_ERR_CUDA";
        case TINYM_ERR_UNSUPPORTED_DEVICE: return "TINYM_ERR_UNSUPPORTED_DEVICE";
        case TINYM_ERR_DEVICE_TIMEOUT: return "TINYM_ERR_DEVICE_TIMEOUT";
        case TINYM_ERR_BAD_PLAN: return "TINYM_ERR_BAD_PLAN";
        default: return "TINYM_ERR_UNKNOWN";
    }
}

int tinym_check_plan(int64_t m, int64_t n, int64_t k, tinym_plan* plan) {
    t_last_error[0] = '\0';
    if (!plan) return fail(TINYM_ERR_INVALID_ARGUMENT, "plan is NULL");
    int st = check_shape(m, n, k);
    if (st != TINYM_OK) return st;
    return fill_derived(m, n, k, plan);
}

int tinym_select_plan(int64_t m, int64_t n, int64_t k, int32_t sm_count, tinym_plan* out) {
    t_last_error[0] = '\0';
    if (!out) return fail(TINYM_ERR_INVALID_ARGUMENT, "out is NULL");
    if (sm_count < 1) return fail(TINYM_ERR_INVALID_ARGUMENT, "sm_count must be positive");
    int st = check_shape(m, n, k);
    if (st != TINYM_OK) return st;
    *out = heuristic_plan(m, n, k, sm_count);
    return fill_derived(m, n, k, out);
}

// The dispatch table's plan as a launch on device `dev` runs it: the
// heuristic plan, then -- since the table assumes every cluster of the grid
// is resident at once -- the K split lowered until the device confirms that
// it is, to the next split that still gives every CTA some K.  The
// static-W plan (overlap) is built to stream more, smaller CTAs than fit
// one wave (clusters are independent, so that is correct) and is left as
// chosen: measured faster than any shrunken variant.
static int device_table_plan(int64_t m, int64_t n, int64_t k, bool overlap, int dev, DeviceInfo* di,
                             tinym_plan* out) {
    tinym_plan p = heuristic_plan(m, n, k, di->sm_count, overlap);
    int st = fill_derived(m, n, k, &p);
    if (st != TINYM_OK) return st;
    const int ring = overlap ? kOverlapRingBytes : kTargetRingBytes;
    while (!overlap && p.split_k > 1) {
        int clusters = 0;
        if ((st = max_active_clusters(p, dev, di, &clusters)) != TINYM_OK) return st;
        if (clusters >= p.tiles_n) break;
        // e.g. 20 K blocks: 7 -> 5, since a split of 6 leaves rank 5 nothing
        const int64_t kb = (k + p.block_k - 1) / p.block_k;
        do {
            --p.split_k;
        } while (p.split_k > 1 && (p.split_k - 1) * ((kb + p.split_k - 1) / p.split_k) >= kb);
        const int s2 = p.kernel == TINYM_KERNEL_TC
                           ? tc_stages_for(p, (kb + p.split_k - 1) / p.split_k,
                                           p.block_k == 4 * kBlockK ? kWideRingBytes : ring)
                           : p.stages;
        if (s2 > 0) p.stages = s2;
        if ((st = fill_derived(m, n, k, &p)) != TINYM_OK) return st;
    }
    *out = p;
    return TINYM_OK;
}

// Everything one GEMM launch needs, built and validated by gemm_prepare
// before anything is queued on the stream (the fused activation path
// validates the GEMM before it launches its prologue).
struct GemmLaunch {
    CUtensorMap tm_w, tm_x;  // 64-byte aligned by their type
    CUtensorMap tm_w1;       // TC kernel: W one 128-byte K chunk per box (its last stage)
    TinymParams prm;
    tinym_plan plan;
    const void* fn;
};

// may_allocate = false: use the device's pending-error word only if an
// earlier call has already allocated it (the no-allocation entry point).
static int gemm_prepare(const void* x, const void* w, void* y, int64_t ldy, int64_t m, int64_t n,
                        int64_t k, const float* alpha_dev, float alpha, const tinym_plan* plan,
                        uint32_t flags, uint64_t timeout_ns, bool w_packed,
                        const tinym_gather_desc* gd, GemmLaunch* out, bool may_allocate = true) {
    if (!x || !w || !y) return fail(TINYM_ERR_INVALID_ARGUMENT, "X, W and Y must be non-null");
    int st = check_shape(m, n, k);
    if (st != TINYM_OK) return st;
    if (ldy < n) return fail(TINYM_ERR_INVALID_ARGUMENT, "ldy (%lld) < N (%lld)", (long long)ldy, (long long)n);
    if (ldy > (int64_t(1) << 31) - 1) return fail(TINYM_ERR_UNSUPPORTED_SHAPE, "ldy exceeds the 32-bit range");
    if ((reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(w) & 15u))
        return fail(TINYM_ERR_MISALIGNED, "X and W must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(y) & 1u) return fail(TINYM_ERR_MISALIGNED, "Y must be 2-byte aligned");
    if (!alpha_dev && !std::isfinite(alpha)) return fail(TINYM_ERR_INVALID_ARGUMENT, "alpha must be finite");

    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    DeviceInfo* di = nullptr;
    if ((st = device_info(dev, &di)) != TINYM_OK) return st;

    tinym_plan p{};
    if (plan) {
        p = *plan;
        if ((st = fill_derived(m, n, k, &p)) != TINYM_OK) return st;
    } else {
        const bool overlap = (flags & tinym::kFlagEarlyW) && !(flags & kFlagQuantPrologue);
        if ((st = device_table_plan(m, n, k, overlap, dev, di, &p)) != TINYM_OK) return st;
    }

    if (w_packed && p.kernel != TINYM_KERNEL_TC)
        return fail(TINYM_ERR_BAD_PLAN, "packed weights need the TC kernel");
    if (gd && p.kernel != TINYM_KERNEL_TC)
        return fail(TINYM_ERR_BAD_PLAN, "the fused all-gather needs the TC kernel");
    const int chunks = plan_chunks(p);
    if ((st = get_map(w, n, k, p.tile_m, 1, chunks, dev, &out->tm_w, w_packed ? 1 : 0)) != TINYM_OK)
        return st;
    if (p.kernel == TINYM_KERNEL_TC) {
        if ((st = get_map(x, m, k, p.mma_n, 1, chunks, dev, &out->tm_x)) != TINYM_OK) return st;
        out->tm_w1 = out->tm_w;
        if (chunks > 1 &&
            (st = get_map(w, n, k, p.tile_m, 1, 1, dev, &out->tm_w1, w_packed ? 1 : 0)) != TINYM_OK)
            return st;
    } else {
        if ((st = get_map(x, m, k, 1, 0, 1, dev, &out->tm_x)) != TINYM_OK) return st;
    }

    TinymParams& prm = out->prm;
    prm = TinymParams{};
    prm.y = static_cast<__nv_bfloat16*>(y);
    prm.alpha_ptr = alpha_dev;
    prm.alpha = alpha;
    prm.m = static_cast<int32_t>(m);
    prm.n = static_cast<int32_t>(n);
    prm.k = static_cast<int32_t>(k);
    prm.ldy = static_cast<int32_t>(ldy);
    prm.kb_total = static_cast<int32_t>((k + p.block_k - 1) / p.block_k);
    prm.kb_per_split = (prm.kb_total + p.split_k - 1) / p.split_k;
    prm.split = p.split_k;
    prm.stages = p.stages;
    prm.flags = flags & 0xFFFFu;  // the kernel's kFlag* bits only
    prm.timeout_ns = timeout_ns;
    prm.w_packed_kc = w_packed ? static_cast<int32_t>(tinym::packed_chunks(k)) : 0;
    prm.rpo = tinym::tc_rows_per_owner(p.tile_m, p.split_k);
    if ((st = pending_word(di, may_allocate, &prm.err_host)) != TINYM_OK) return st;
    if (gd) {
        // CTA (0,0) waits for the other ranks: the whole grid must be resident
        // at once, or a waiting CTA could hold an SM another CTA needs.
        int resident = 0;
        if ((st = max_active_clusters(p, dev, di, &resident)) != TINYM_OK) return st;
        if (resident < p.tiles_n)
            return fail(TINYM_ERR_BAD_PLAN,
                        "the fused all-gather needs the whole grid resident (%d of %d %s)",
                        resident, p.tiles_n, p.split_k > 1 ? "clusters" : "CTAs");
        prm.n_peers = gd->world;
        prm.rank = gd->rank;
        prm.gather_target = gd->target;
        for (int r = 0; r < gd->world; ++r) {
            prm.peer_y[r] = static_cast<__nv_bfloat16*>(gd->y_full[r]) + gd->col0;
            prm.peer_flag[r] = static_cast<unsigned long long*>(gd->flag[r]);
        }
    }

    out->fn = nullptr;
    if ((st = kernel_for(p, di, &out->fn)) != TINYM_OK) return st;
    out->plan = p;
    return TINYM_OK;
}

static int gemm_launch(GemmLaunch& g, void* stream) {
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attrs[2];
    launch_config(g.plan, stream, &cfg, attrs);
    void* tc_args[4] = {&g.tm_w, &g.tm_x, &g.tm_w1, &g.prm};
    void* simt_args[3] = {&g.tm_w, &g.tm_x, &g.prm};
    const cudaError_t e =
        cudaLaunchKernelExC(&cfg, g.fn, g.plan.kernel == TINYM_KERNEL_TC ? tc_args : simt_args);
    if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
    return TINYM_OK;
}

static int gemm_impl(const void* x, const void* w, void* y, int64_t ldy, int64_t m, int64_t n,
                     int64_t k, const float* alpha_dev, float alpha, const tinym_plan* plan,
                     void* stream, uint32_t flags, uint64_t timeout_ns, bool w_packed = false,
                     const tinym_gather_desc* gd = nullptr) {
    t_last_error[0] = '\0';
    GemmLaunch g;
    const int st = gemm_prepare(x, w, y, ldy, m, n, k, alpha_dev, alpha, plan, flags, timeout_ns,
                                w_packed, gd, &g);
    if (st != TINYM_OK) return st;
    return gemm_launch(g, stream);
}

int tinym_fp8_gemm_ex(const void* x, const void* w, void* y, int64_t ldy, int64_t m, int64_t n,
                      int64_t k, const float* alpha_dev, float alpha, const tinym_plan* plan,
                      void* stream) {
    return gemm_impl(x, w, y, ldy, m, n, k, alpha_dev, alpha, plan, stream, 0u,
                     kDefaultTimeoutNs);
}

int tinym_select_plan_ex(int64_t m, int64_t n, int64_t k, int32_t sm_count, uint32_t flags,
                         tinym_plan* out) {
    t_last_error[0] = '\0';
    if (!out) return fail(TINYM_ERR_INVALID_ARGUMENT, "out is NULL");
    if (sm_count < 1) return fail(TINYM_ERR_INVALID_ARGUMENT, "sm_count must be positive");
    if (flags & ~static_cast<uint32_t>(TINYM_FLAG_STATIC_W))
        return fail(TINYM_ERR_INVALID_ARGUMENT, "unknown flags 0x%x", flags);
    int st = check_shape(m, n, k);
    if (st != TINYM_OK) return st;
    *out = heuristic_plan(m, n, k, sm_count, (flags & TINYM_FLAG_STATIC_W) != 0);
    return fill_derived(m, n, k, out);
}

int tinym_launch_plan(int64_t m, int64_t n, int64_t k, uint32_t flags, tinym_plan* out) {
    t_last_error[0] = '\0';
    if (!out) return fail(TINYM_ERR_INVALID_ARGUMENT, "out is NULL");
    if (flags & ~static_cast<uint32_t>(TINYM_FLAG_STATIC_W))
        return fail(TINYM_ERR_INVALID_ARGUMENT, "unknown flags 0x%x", flags);
    int st = check_shape(m, n, k);
    if (st != TINYM_OK) return st;
    int dev = 0;
    const cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    DeviceInfo* di = nullptr;
    if ((st = device_info(dev, &di)) != TINYM_OK) return st;
    return device_table_plan(m, n, k, (flags & TINYM_FLAG_STATIC_W) != 0, dev, di, out);
}

int tinym_fp8_gemm_ex2(const void* x, const void* w, void* y, int64_t ldy, int64_t m, int64_t n,
                       int64_t k, const float* alpha_dev, float alpha, const tinym_plan* plan,
                       uint32_t flags, void* stream) {
    t_last_error[0] = '\0';
    if (flags & ~static_cast<uint32_t>(TINYM_FLAG_STATIC_W))
        return fail(TINYM_ERR_INVALID_ARGUMENT, "unknown flags 0x%x", flags);
    const uint32_t kflags = (flags & TINYM_FLAG_STATIC_W) ? tinym::kFlagEarlyW : 0u;
    return gemm_impl(x, w, y, ldy, m, n, k, alpha_dev, alpha, plan, stream, kflags,
                     kDefaultTimeoutNs);
}

int tinym_quant_workspace_bytes(int64_t m, int64_t k, int64_t* bytes) {
    t_last_error[0] = '\0';
    if (!bytes) return fail(TINYM_ERR_INVALID_ARGUMENT, "bytes is NULL");
    int st = check_shape(m, 1, k);
    if (st != TINYM_OK) return st;
    *bytes = tinym::kQuantWsHeader + (m * k + 255) / 256 * 256;
    return TINYM_OK;
}

static int quant_act_impl(const void* x_act, int32_t act_dtype, const void* w,
                          const float* w_scale_dev, void* y, int64_t ldy, int64_t m, int64_t n,
                          int64_t k, void* workspace, const tinym_plan* plan, void* stream,
                          bool may_allocate) {
    if (!x_act || !w || !w_scale_dev || !y || !workspace)
        return fail(TINYM_ERR_INVALID_ARGUMENT, "X, W, w_scale, Y and workspace must be non-null");
    if (act_dtype != TINYM_ACT_BF16 && act_dtype != TINYM_ACT_F32)
        return fail(TINYM_ERR_INVALID_ARGUMENT, "act_dtype %d is not TINYM_ACT_BF16 / TINYM_ACT_F32",
                    act_dtype);
    int st = check_shape(m, n, k);
    if (st != TINYM_OK) return st;
    if ((reinterpret_cast<uintptr_t>(x_act) & 15u) || (reinterpret_cast<uintptr_t>(workspace) & 255u))
        return fail(TINYM_ERR_MISALIGNED, "X must be 16-byte and the workspace 256-byte aligned");
    if ((reinterpret_cast<uintptr_t>(w_scale_dev) & 3u))
        return fail(TINYM_ERR_MISALIGNED, "w_scale must be 4-byte aligned");
    // The GEMM (shapes, alignment, plan, tensor maps) is validated before the
    // prologue is queued, so a failing call leaves the workspace untouched.
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    GemmLaunch g;
    if ((st = gemm_prepare(ws + tinym::kQuantWsHeader, w, y, ldy, m, n, k,
                           reinterpret_cast<const float*>(ws) + 1, 0.0f, plan,
                           tinym::kFlagEarlyW | kFlagQuantPrologue, kDefaultTimeoutNs, false,
                           nullptr, &g, may_allocate)) != TINYM_OK)
        return st;
    // Ordinary stream order (no programmatic attribute): everything before
    // this kernel has completed when it starts, which is what lets the GEMM
    // read W ahead of its griddepcontrol.wait.  It must stay that way for
    // the no-allocation form too: its static workspace is rewritten by this
    // kernel, so the previous call's GEMM (launched with the programmatic
    // attribute, reading the workspace) must have completed first.
    auto s = static_cast<cudaStream_t>(stream);
    if (act_dtype == TINYM_ACT_BF16)
        tinym::tinym_quant_act_kernel<__nv_bfloat16>
            <<<tinym::kQuantCtas, tinym::kQuantThreads, 0, s>>>(
                static_cast<const __nv_bfloat16*>(x_act), m * k, ws, w_scale_dev);
    else
        tinym::tinym_quant_act_kernel<float><<<tinym::kQuantCtas, tinym::kQuantThreads, 0, s>>>(
            static_cast<const float*>(x_act), m * k, ws, w_scale_dev);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "quantise kernel launch");
    return gemm_launch(g, stream);
}

int tinym_fp8_gemm_quant_act(const void* x_act, int32_t act_dtype, const void* w,
                             const float* w_scale_dev, void* y, int64_t ldy, int64_t m,
                             int64_t n, int64_t k, void* workspace, const tinym_plan* plan,
                             void* stream) {
    t_last_error[0] = '\0';
    return quant_act_impl(x_act, act_dtype, w, w_scale_dev, y, ldy, m, n, k, workspace, plan,
                          stream, true);
}

int tinym_fp8_gemm_quant_act_noalloc(const void* x_act, int32_t act_dtype, const void* w,
                                     const float* w_scale_dev, void* y, int64_t ldy, int64_t m,
                                     int64_t n, int64_t k, const tinym_plan* plan, void* stream) {
    t_last_error[0] = '\0';
    int st = check_shape(m, n, k);
    if (st != TINYM_OK) return st;
    if (m * k > kNoAllocMaxElems)
        return fail(TINYM_ERR_UNSUPPORTED_SHAPE,
                    "M*K = %lld exceeds the static workspace (%lld elements)",
                    static_cast<long long>(m * k), static_cast<long long>(kNoAllocMaxElems));
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return fail(TINYM_ERR_CUDA, "device ordinal %d out of range", dev);
    void* ws = nullptr;
    if ((st = scratch_address(dev, &ws)) != TINYM_OK) return st;
    return quant_act_impl(x_act, act_dtype, w, w_scale_dev, y, ldy, m, n, k, ws, plan, stream,
                          false);
}

int tinym_ipc_export(const void* ptr, void* handle, int64_t* offset) {
    t_last_error[0] = '\0';
    if (!ptr || !handle || !offset) return fail(TINYM_ERR_INVALID_ARGUMENT, "null argument");
    AddrRangeFn range = get_addr_range();
    if (!range) return fail(TINYM_ERR_CUDA, "cuMemGetAddressRange unavailable");
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
        return fail(TINYM_ERR_CUDA, "cuMemGetAddressRange failed for %p", ptr);
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
    std::memcpy(handle, &h, sizeof(h));
    *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
    return TINYM_OK;
}

int tinym_ipc_open(const void* handle, void** base) {
    t_last_error[0] = '\0';
    if (!handle || !base) return fail(TINYM_ERR_INVALID_ARGUMENT, "null argument");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
    return TINYM_OK;
}

int tinym_ipc_close(void* base) {
    t_last_error[0] = '\0';
    cudaError_t e = cudaIpcCloseMemHandle(base);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
    return TINYM_OK;
}

int tinym_fp8_gemm_allgather(const void* x, const void* w_local, int64_t m, int64_t n_local,
                             int64_t k, const float* alpha_dev, float alpha,
                             const tinym_gather_desc* gd, const tinym_plan* plan, void* stream) {
    t_last_error[0] = '\0';
    if (!gd) return fail(TINYM_ERR_INVALID_ARGUMENT, "gather descriptor is NULL");
    if (gd->world < 1 || gd->world > tinym::kMaxPeers || gd->rank < 0 || gd->rank >= gd->world)
        return fail(TINYM_ERR_INVALID_ARGUMENT, "world %d / rank %d out of range (1..%d ranks)",
                    gd->world, gd->rank, tinym::kMaxPeers);
    if (gd->col0 < 0 || gd->col0 + n_local > gd->n_full)
        return fail(TINYM_ERR_INVALID_ARGUMENT, "columns [%lld, %lld) exceed N_full %lld",
                    (long long)gd->col0, (long long)(gd->col0 + n_local), (long long)gd->n_full);
    for (int r = 0; r < gd->world; ++r)
        if (!gd->y_full[r] || !gd->flag[r] || (reinterpret_cast<uintptr_t>(gd->flag[r]) & 7u))
            return fail(TINYM_ERR_INVALID_ARGUMENT, "rank %d: null Y or unaligned counter", r);
    return gemm_impl(x, w_local, static_cast<__nv_bfloat16*>(gd->y_full[gd->rank]) + gd->col0,
                     gd->n_full, m, n_local, k, alpha_dev, alpha, plan, stream, 0u,
                     kDefaultTimeoutNs, false, gd);
}

int tinym_packed_weight_bytes(int64_t n, int64_t k, int64_t* bytes) {
    t_last_error[0] = '\0';
    if (!bytes) return fail(TINYM_ERR_INVALID_ARGUMENT, "bytes is NULL");
    int st = check_shape(1, n, k);
    if (st != TINYM_OK) return st;
    const int64_t tiles = (n + tinym::kPackRows - 1) / tinym::kPackRows;
    *bytes = tiles * tinym::packed_chunks(k) * tinym::kPackRows * kBlockK;
    return TINYM_OK;
}

int tinym_pack_weights(const void* w, void* w_packed, int64_t n, int64_t k, void* stream) {
    t_last_error[0] = '\0';
    if (!w || !w_packed) return fail(TINYM_ERR_INVALID_ARGUMENT, "W and W_packed must be non-null");
    int64_t bytes = 0;
    int st = tinym_packed_weight_bytes(n, k, &bytes);
    if (st != TINYM_OK) return st;
    if ((reinterpret_cast<uintptr_t>(w) & 15u) || (reinterpret_cast<uintptr_t>(w_packed) & 15u))
        return fail(TINYM_ERR_MISALIGNED, "W and W_packed must be 16-byte aligned");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    DeviceInfo* di = nullptr;
    if ((st = device_info(dev, &di)) != TINYM_OK) return st;
    const int64_t vecs = bytes / 16;
    const int64_t blocks = std::min<int64_t>((vecs + 255) / 256, int64_t(di->sm_count) * 16);
    tinym::tinym_pack_weights_kernel<<<static_cast<unsigned>(blocks), 256, 0,
                                       static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(w), static_cast<uint4*>(w_packed), n, k,
        tinym::packed_chunks(k), vecs);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "pack kernel launch");
    return TINYM_OK;
}

int tinym_fp8_gemm_packed(const void* x, const void* w_packed, void* y, int64_t ldy, int64_t m,
                          int64_t n, int64_t k, const float* alpha_dev, float alpha,
                          const tinym_plan* plan, void* stream) {
    return gemm_impl(x, w_packed, y, ldy, m, n, k, alpha_dev, alpha, plan, stream, 0u,
                     kDefaultTimeoutNs, true);
}

int tinym_selftest_wait_timeout(const void* x, const void* w, void* y, int64_t m, int64_t n,
                                int64_t k, const tinym_plan* plan, uint64_t timeout_ns,
                                void* stream) {
    if (timeout_ns == 0 || timeout_ns > 10ull * kDefaultTimeoutNs)
        return fail(TINYM_ERR_INVALID_ARGUMENT, "timeout_ns must be in 1 .. 1e10");
    return gemm_impl(x, w, y, n, m, n, k, nullptr, 1.0f, plan, stream,
                     tinym::kFlagInjectNoLoads, timeout_ns);
}

int tinym_fp8_gemm(const void* x, const void* w, void* y, int64_t m, int64_t n, int64_t k,
                   float x_scale, float w_scale, void* stream) {
    return tinym_fp8_gemm_ex(x, w, y, n, m, n, k, nullptr, x_scale * w_scale, nullptr, stream);
}

int tinym_fp8_gemm_dev_alpha(const void* x, const void* w, void* y, int64_t m, int64_t n,
                             int64_t k, const float* alpha_dev, void* stream) {
    if (!alpha_dev) return fail(TINYM_ERR_INVALID_ARGUMENT, "alpha_dev must be non-null");
    return tinym_fp8_gemm_ex(x, w, y, n, m, n, k, alpha_dev, 0.0f, nullptr, stream);
}

int tinym_plan_max_active_clusters(int64_t m, int64_t n, int64_t k, const tinym_plan* plan,
                                   int32_t* out) {
    t_last_error[0] = '\0';
    if (!plan || !out) return fail(TINYM_ERR_INVALID_ARGUMENT, "plan and out must be non-null");
    int st = check_shape(m, n, k);
    if (st != TINYM_OK) return st;
    tinym_plan p = *plan;
    if ((st = fill_derived(m, n, k, &p)) != TINYM_OK) return st;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    DeviceInfo* di = nullptr;
    if ((st = device_info(dev, &di)) != TINYM_OK) return st;
    int v = 0;
    if ((st = max_active_clusters(p, dev, di, &v)) != TINYM_OK) return st;
    *out = v;
    return TINYM_OK;
}

int tinym_device_status(uint32_t* flags, int32_t clear) {
    t_last_error[0] = '\0';
    if (!flags) return fail(TINYM_ERR_INVALID_ARGUMENT, "flags is NULL");
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
    e = cudaMemcpyFromSymbol(flags, tinym::g_err_word, sizeof(uint32_t));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyFromSymbol(error word)");
    if (clear) {
        const uint32_t zero = 0;
        e = cudaMemcpyToSymbol(tinym::g_err_word, &zero, sizeof(uint32_t));
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyToSymbol(error word)");
    }
    // The same bits were also posted to the pending-error word (if the
    // device has one); after a synchronising read both are consumed.
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kMaxDevices) {
        volatile uint32_t* h = g_dev[dev].err_host.load(std::memory_order_acquire);
        if (h) {
            uint32_t* word = const_cast<uint32_t*>(h);
            *flags |= clear ? __atomic_exchange_n(word, 0u, __ATOMIC_ACQ_REL)
                            : __atomic_load_n(word, __ATOMIC_ACQUIRE);
        }
    }
    return *flags ? fail(TINYM_ERR_DEVICE_TIMEOUT, "device error word 0x%x", *flags) : TINYM_OK;
}

int tinym_pending_errors(uint32_t* flags, int32_t clear) {
    t_last_error[0] = '\0';
    if (!flags) return fail(TINYM_ERR_INVALID_ARGUMENT, "flags is NULL");
    *flags = 0u;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return fail(TINYM_ERR_CUDA, "device ordinal %d out of range", dev);
    volatile uint32_t* h = g_dev[dev].err_host.load(std::memory_order_acquire);
    if (h) {
        uint32_t* word = const_cast<uint32_t*>(h);
        *flags = clear ? __atomic_exchange_n(word, 0u, __ATOMIC_ACQ_REL)
                       : __atomic_load_n(word, __ATOMIC_ACQUIRE);
    }
    return *flags ? fail(TINYM_ERR_DEVICE_TIMEOUT,
                         "a kernel that finished earlier on device %d ran out of a bounded wait "
                         "(error bits 0x%x): its output is unspecified", dev, *flags)
                  : TINYM_OK;
}

}  // extern "C"
