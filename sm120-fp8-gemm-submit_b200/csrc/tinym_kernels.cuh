// tinym_kernels.cuh -- sm_100a kernels of the tiny-M FP8 GEMM.
//
//   Y[m, n] = bf16( alpha * sum_k X[m,k] * W[n,k] ),  1 <= M <= 16.
//
// The work is cut into 128-row W tiles ("tiles", blockIdx.y) and, when the
// tiles alone cannot fill the GPU, into split_k contiguous K ranges
// (blockIdx.x).  The split_k CTAs of one tile form a thread-block cluster and
// combine their FP32 partial sums through distributed shared memory -- a
// deterministic, single-launch split-K with no global scratch memory.  The
// TC kernel reduce-scatters (each CTA sums and stores a block of the tile's
// rows); the SIMT kernel reduces into the cluster's rank-0 CTA.
//
// Two consumers share this skeleton:
//
//  * tinym_tc_kernel<MMA_N, CHUNKS, TILE_M> ("swap-AB"): the W tile
//    [TILE_M x 128 B] is the A operand of tcgen05.mma.kind::f8f6f4 (MMA M =
//    TILE_M = 128, or 64) and X, padded by TMA zero fill to MMA_N (8 or 16)
//    rows, is the B operand.  The accumulator D[TILE_M x MMA_N] (FP32) lives
//    in tensor memory; four epilogue warps read it with tcgen05.ld, scale it,
//    convert it to BF16 and store it -- to Y, or (fused all-gather) to every
//    rank's Y over NVLink.  Replaces the reference's M<=16 mma.sync kernel
//    (include/fp8_gemm_tinym.cuh:321-461), whose m16n8k32 warp MMA put M on
//    the MMA's M side.
//
//  * tinym_simt_m1_kernel<CWARPS>: M = 1 only.  Consumer warps widen the
//    E4M3 W bytes to FP32 and FMA them against X on the CUDA cores; eight
//    lanes share one W row (one 16-byte chunk each) and are reduced with
//    warp shuffles.  The M=1 counterpart of the reference's scalar kernel
//    (include/fp8_gemm_tinym.cuh:521-722).
//
// Both stream W with TMA into a ring of `stages` shared-memory slots guarded
// by full/empty mbarriers, using the 128-byte swizzle: one stage is CHUNKS
// K chunks of [TILE_M rows x 128 B], fetched by one 3-D box when CHUNKS > 1
// (2-D boxes of 128 rows x 128 B for the SIMT kernel).  Every wait is bounded
// (WaitGuard): a wait that runs out sets a bit in the device error word and
// the CTA drains what it has in flight, frees its tensor memory and exits.
#pragma once

#include "tinym_ptx.cuh"

namespace tinym {

// Device error word (one per device; read by tinym_device_status).
__device__ uint32_t g_err_word;

// Timeline trace points.  They compile to nothing unless a diagnostic build
// defines TINYM_TRACE_POINTS, in which case the SM cycle counter of each
// event is recorded per CTA in g_trace, and %globaltimer at the CTA's first
// and last event in g_trace_ns (to align CTAs and convert cycles; the
// timer itself ticks in coarse steps).  Latency analysis only; the shipped
// library never defines it.
#ifdef TINYM_TRACE_POINTS
__device__ uint64_t g_trace[8192][24];
__device__ uint64_t g_trace_ns[8192][2];
#define TINYM_TRACE(id) (g_trace[blockIdx.y * gridDim.x + blockIdx.x][(id)] = clock64())
#define TINYM_TRACE_NS(slot) (g_trace_ns[blockIdx.y * gridDim.x + blockIdx.x][(slot)] = globaltimer_ns())
#else
#define TINYM_TRACE(id) ((void)0)
#define TINYM_TRACE_NS(slot) ((void)0)
#endif

enum : uint32_t {
    kErrProducerWait = 1u << 0,
    kErrMmaWait = 1u << 1,
    kErrEpilogueWait = 1u << 2,
    kErrDrain = 1u << 3,
    kErrConsumerWait = 1u << 4,
    kErrReduceWait = 1u << 5,
    kErrPeerWait = 1u << 6,
};

constexpr int kTileRows = 128;   // W rows per tile of the SIMT kernel (and the TC default)
constexpr int kBlockK = 128;     // K bytes of one chunk (= one 128B swizzle row)
constexpr int kWStageBytes = kTileRows * kBlockK;  // one W chunk: 16 KiB
constexpr int kTcThreads = 192;  // warp0 TMA, warp1 MMA, warps2-5 epilogue
constexpr int kTmemCols = 32;    // minimum allocation; MMA_N <= 16 columns used
constexpr int kMaxSplit = 8;     // CTAs per cluster (K split), portable cluster size

struct TinymParams {
    __nv_bfloat16* y;
    const float* alpha_ptr;  // if non-null, alpha is read here on the device
    float alpha;
    int32_t m, n, k, ldy;
    int32_t kb_total;      // K stages: ceil(K / (128 * chunks per stage))
    int32_t kb_per_split;  // K stages per CTA (last CTA of a cluster may get fewer)
    int32_t split;         // CTAs per tile (cluster size along x)
    int32_t stages;
    uint32_t flags;        // kFlag* bits (0 in normal operation)
    uint64_t timeout_ns;   // limit of every mbarrier wait
    int32_t w_packed_kc;   // 0: W row-major [N, K]; else W packed, this many K chunks per tile
    int32_t rpo;           // TC split-K: tile rows each cluster rank owns (tc_rows_per_owner)
    // Fused all-gather of the N-sharded wrapper (n_peers > 0): the BF16 rows
    // go to every rank's full Y (peer_y[r] = rank r's Y + this rank's first
    // column, row stride ldy) instead of y, each CTA then adds the number of
    // elements it stored to every rank's arrival counter, and CTA (0,0)
    // waits until this rank's counter reaches gather_target, so the grid
    // completes only when this rank's full Y has arrived.
    int32_t n_peers;
    int32_t rank;
    unsigned long long gather_target;
    __nv_bfloat16* peer_y[8];
    unsigned long long* peer_flag[8];
    // Host-mapped pending-error word (device address), or null: a wait that
    // runs out also sets its bit here, where the host can see it at the next
    // call without synchronising the device.
    uint32_t* err_host;
};
constexpr int kMaxPeers = 8;

// Packed weight layout (TC kernel only): W cut into kPackRows-row tiles and
// 128-byte K chunks; chunk c of tile t is one contiguous [kPackRows][128 B]
// block at byte offset (t * KC + c) * kPackRows * 128, zero-filled past N
// and K.  KC = ceil(K / 128) rounded up to a multiple of kPackChunkAlign
// (the largest stage), so a stage never reaches into the next tile.  A
// stage of CHUNKS chunks is then a single contiguous HBM range (64 KiB at
// block_k = 512).
constexpr int kPackRows = 128;
constexpr int kPackChunkAlign = 4;
__host__ __device__ constexpr int64_t packed_chunks(int64_t k) {
    return ((k + 127) / 128 + kPackChunkAlign - 1) / kPackChunkAlign * kPackChunkAlign;
}

// TinymParams::flags.  kFlagInjectNoLoads makes the producer issue no TMA
// copies: nothing ever completes the full barriers, the consumers' bounded
// waits run out, and the kernel reports through g_err_word and exits
// cleanly.  Used only by the failure-detection self-test.
constexpr uint32_t kFlagInjectNoLoads = 1u;
// kFlagEarlyW: the previous kernel in the stream (launched without the
// programmatic-serialisation attribute, so everything before it has
// completed) writes only X and alpha -- the fused activation-quantise
// prologue.  The producer then puts the first ring-full of W loads in
// flight before griddepcontrol.wait and only the X loads after it, so W
// streams while X is being quantised.
constexpr uint32_t kFlagEarlyW = 2u;

// Shared-memory carve-up, identical on host (size) and device (offsets).
struct SmemLayout {
    uint32_t w_off, x_off, red_off, bar_off, misc_off, bytes;
};

// red_rank_bytes: split-K partial-sum bytes one CTA receives from each other
// CTA of its cluster (it reserves (split - 1) of them).
__host__ __device__ inline SmemLayout smem_layout(int stages, int w_stage_bytes, int x_stage_bytes,
                                                  int split, int red_rank_bytes) {
    SmemLayout L;
    L.w_off = 0;
    L.x_off = L.w_off + static_cast<uint32_t>(stages) * static_cast<uint32_t>(w_stage_bytes);
    L.red_off = L.x_off + static_cast<uint32_t>(stages * x_stage_bytes);
    L.red_off = (L.red_off + 15u) & ~15u;
    const uint32_t red_bytes = static_cast<uint32_t>((split - 1) * red_rank_bytes);
    L.bar_off = (L.red_off + red_bytes + 7u) & ~7u;
    // barriers: full and empty per stage, accumulator, reduction, TMEM
    // release, and up to three chunk barriers of the TC kernel's last stage
    L.misc_off = L.bar_off + static_cast<uint32_t>(2 * stages + 6) * 8u;
    // +1024: the dynamic window is re-aligned to 1024 bytes in the kernel.
    L.bytes = L.misc_off + 16u + 1024u;
    return L;
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
    const uint32_t a = smem_u32(p);
    return p + (((a + 1023u) & ~1023u) - a);
}

// Split-K reduce-scatter of the TC kernel: rank o of a cluster of `split`
// CTAs owns tile rows [o * rpo, o * rpo + cnt_o), rpo = ceil(tile_m / split)
// rounded up to 8 rows (whole 16-byte BF16 output vectors), cnt_o = rows
// left for rank o (0 for trailing ranks when 8-row rounding runs out).
// Every CTA sends its partial rows to their owners and sums/stores its own.
__host__ __device__ constexpr int tc_rows_per_owner(int tile_m, int split) {
    return ((tile_m + split - 1) / split + 7) / 8 * 8;
}
__host__ __device__ constexpr int tc_rows_owned(int tile_m, int split, int rank) {
    return tile_m - rank * tc_rows_per_owner(tile_m, split) <= 0
               ? 0
               : (tile_m - rank * tc_rows_per_owner(tile_m, split) <
                          tc_rows_per_owner(tile_m, split)
                      ? tile_m - rank * tc_rows_per_owner(tile_m, split)
                      : tc_rows_per_owner(tile_m, split));
}
// Row stride (FP32 elements) of a received partial block: MMA_N values
// padded by 4 so that 16-byte shared-memory accesses of consecutive rows
// are bank-conflict free.
__host__ __device__ constexpr int tc_red_stride(int mma_n) { return mma_n + 4; }
// Bytes of one received block (one source rank); a CTA holds split - 1.
__host__ __device__ constexpr int tc_red_rank_bytes(int mma_n, int tile_m, int split) {
    return tc_rows_per_owner(tile_m, split) * tc_red_stride(mma_n) * 4;
}

// Named barrier 1 over the 128 epilogue threads (warps 2..5) of the TC kernel.
__device__ __forceinline__ void epilogue_bar_sync() {
    asm volatile("bar.sync 1, 128;" ::: "memory");
}

__device__ __forceinline__ float load_alpha(const TinymParams& p) {
    return p.alpha_ptr ? __ldg(p.alpha_ptr) : p.alpha;
}

// =====================================================================
// tcgen05 swap-AB kernel
// =====================================================================
template <int MMA_N, int CHUNKS, int TILE_M>
__global__ void __launch_bounds__(kTcThreads, 1)
    tinym_tc_kernel(const __grid_constant__ CUtensorMap tm_w,
                    const __grid_constant__ CUtensorMap tm_x,
                    const __grid_constant__ CUtensorMap tm_w1, const TinymParams p) {
    static_assert(MMA_N == 8 || MMA_N == 16, "MMA_N must be 8 or 16");
    static_assert(CHUNKS == 1 || CHUNKS == 2 || CHUNKS == 4, "1, 2 or 4 K chunks per stage");
    static_assert(TILE_M == 64 || TILE_M == 128, "W tiles of 64 or 128 rows (MMA M)");
    // One stage = CHUNKS K chunks of 128 bytes.  Each W chunk is a standard
    // [TILE_M rows x 128 B] 128B-swizzled tile, each X chunk
    // [MMA_N rows x 128 B]; with CHUNKS > 1 one 3-D TMA box fetches all of
    // a stage's chunks, which raises the bytes moved per TMA instruction
    // (a single CTA's stream is bound by instructions, not bytes).
    // TILE_M = 64 halves the tile so that more CTAs cover N without a K
    // split; its M=64 accumulator occupies TMEM lanes 32q..32q+15 (rows
    // 16q..16q+15) of each 32-lane subpartition q.
    constexpr int kWChunk = TILE_M * kBlockK;
    constexpr int kXChunkBytes = MMA_N * kBlockK;  // 1 or 2 KiB, 1024-aligned
    constexpr int kWStage = CHUNKS * kWChunk;
    constexpr int kXStageBytes = CHUNKS * kXChunkBytes;
    constexpr uint32_t kStageTx = kWStage + kXStageBytes;
    constexpr uint32_t kIdesc = idesc_e4m3_f32(TILE_M, MMA_N);
    constexpr int kRedStride = tc_red_stride(MMA_N);
    constexpr int kRowsPerWarp = TILE_M / 4;                // accumulator rows per epilogue warp

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);
    // Rows of the tile each cluster rank sums and stores (host-computed
    // tc_rows_per_owner: no division on the device).
    const int rpo = p.rpo;
    const int red_rank_bytes = rpo * kRedStride * 4;  // tc_red_rank_bytes
    const SmemLayout L = smem_layout(p.stages, kWStage, kXStageBytes, p.split, red_rank_bytes);
    const uint32_t s_base = smem_u32(smem);
    const uint32_t w_ring = s_base + L.w_off;
    const uint32_t x_ring = s_base + L.x_off;
    const uint32_t bars = s_base + L.bar_off;
    const int stages = p.stages;
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (stages + s); };
    const uint32_t acc_bar = bars + 8u * (2 * stages);
    const uint32_t red_bar = bars + 8u * (2 * stages + 1);
    // One arrive per epilogue warp once its accumulator reads are complete:
    // the MMA warp then frees TMEM while the epilogue is still running.
    const uint32_t tmem_bar = bars + 8u * (2 * stages + 2);
    // The CTA's last stage (CHUNKS > 1) is loaded one 128-byte K chunk per box
    // (tm_w1): chunk 0 and X complete on the stage's full barrier, chunk c on
    // tail_bar(c), so the MMAs of the first chunks run while later ones land.
    auto tail_bar = [&](int c) { return bars + 8u * (2 * stages + 2 + c); };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.misc_off);
    volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + L.misc_off + 4);
    // Partial sums from the other ranks land in their own region.
    float* red = reinterpret_cast<float*>(smem + L.red_off);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int split_idx = blockIdx.x;
    const int tile = blockIdx.y;
    const bool clustered = p.split > 1;
    // Rows of the tile this CTA sums and stores (tc_rows_owned), and the
    // partial-sum columns that carry data (X rows m < M, in groups of four).
    const int own_lo = split_idx * rpo;
    const int own_cnt = max(0, min(rpo, TILE_M - own_lo));
    const int red_cols = (p.m + 3) & ~3;
    const int kb0 = split_idx * p.kb_per_split;
    const int kb1 = min(kb0 + p.kb_per_split, p.kb_total);
    const int nkb = kb1 - kb0;  // >= 1 by construction of the plan
    // Fault injection (self-test only): issue no copies, so the consumers'
    // bounded waits run out and report through the error word.
    const int n_issue = (p.flags & kFlagInjectNoLoads) ? 0 : nkb;

    const WaitGuard guard{abort_flag, &g_err_word, p.timeout_ns, p.err_host};

    // The producer thread initialises the barriers and immediately puts the
    // first ring-full of loads in flight, so the DRAM latency of the first
    // bytes overlaps the TMEM allocation and the CTA-wide sync below.
    int issued = 0;
    uint64_t pol_w = 0, pol_x = 0;
    // One stage = expect_tx(W + X bytes), then the W box and the X box on the
    // stage's full barrier (issue_w posts the expect_tx).
    // Stage i of this CTA's K range goes to ring slot s (= i mod stages; the
    // loops below keep s and the slot's phase parity in running counters,
    // since a runtime division per stage measurably slows the issue loops).
    // K chunks of this CTA's last stage that lie inside K (K % 128 == 0
    // whenever CHUNKS > 1); the others carry no data and get no MMA.
    const int last_chunks = min(CHUNKS, p.k / kBlockK - (kb0 + nkb - 1) * CHUNKS);
    auto issue_w = [&](int i, int s) {
        const int chunk = (kb0 + i) * CHUNKS;  // first 128-byte K chunk of the stage
        if constexpr (CHUNKS > 1) {
            if (i == nkb - 1) {
                mbar_expect_tx(full_bar(s), static_cast<uint32_t>(kWChunk + kXStageBytes));
                for (int c = 0; c < last_chunks; ++c) {
                    const uint32_t bar = c == 0 ? full_bar(s) : tail_bar(c);
                    if (c > 0) mbar_expect_tx(bar, static_cast<uint32_t>(kWChunk));
                    const uint32_t dst = w_ring + s * kWStage + c * kWChunk;
                    if (p.w_packed_kc) {
                        const int r0 = tile * TILE_M;
                        tma_load_3d(dst, &tm_w1, bar, 0, r0 % kPackRows,
                                    (r0 / kPackRows) * p.w_packed_kc + chunk + c, pol_w);
                    } else {
                        tma_load_2d(dst, &tm_w1, bar, (chunk + c) * kBlockK, tile * TILE_M, pol_w);
                    }
                }
                return;
            }
        }
        mbar_expect_tx(full_bar(s), kStageTx);
        if (p.w_packed_kc) {
            const int r0 = tile * TILE_M;
            tma_load_3d(w_ring + s * kWStage, &tm_w, full_bar(s), 0, r0 % kPackRows,
                        (r0 / kPackRows) * p.w_packed_kc + chunk, pol_w);
        } else if constexpr (CHUNKS == 1) {
            tma_load_2d(w_ring + s * kWStage, &tm_w, full_bar(s), chunk * kBlockK, tile * TILE_M,
                        pol_w);
        } else {
            tma_load_3d(w_ring + s * kWStage, &tm_w, full_bar(s), 0, tile * TILE_M, chunk, pol_w);
        }
    };
    auto issue_x = [&](int i, int s) {
        const int chunk = (kb0 + i) * CHUNKS;
        if constexpr (CHUNKS == 1)
            tma_load_2d(x_ring + s * kXStageBytes, &tm_x, full_bar(s), chunk * kBlockK, 0, pol_x);
        else
            tma_load_3d(x_ring + s * kXStageBytes, &tm_x, full_bar(s), 0, 0, chunk, pol_x);
    };
    auto issue = [&](int i, int s) {
        issue_w(i, s);
        issue_x(i, s);
    };
    if (threadIdx.x == 0) {
        TINYM_TRACE_NS(0);
        TINYM_TRACE(0);
        tma_prefetch_desc(&tm_w);
        tma_prefetch_desc(&tm_x);
        // The first ring-full of loads goes out before anything else: only
        // the full barriers are initialised (and published to the async
        // proxy) ahead of it; the other barriers follow while it is in flight.
        for (int s = 0; s < stages; ++s) mbar_init(full_bar(s), 1);
        if constexpr (CHUNKS > 1)
            for (int c = 1; c < CHUNKS; ++c) mbar_init(tail_bar(c), 1);
        fence_mbar_init();
        fence_proxy_async_smem();
        TINYM_TRACE(10);
        pol_w = l2_policy_w();
        pol_x = l2_policy_evict_last();
        // Programmatic dependent launch: everything above overlaps the
        // previous kernel's tail; no global memory is read before it has
        // completed and its writes are visible -- except W under
        // kFlagEarlyW, which that kernel does not write.
        const int first = min(stages, n_issue);
        if (p.flags & kFlagEarlyW) {
            for (int i = 0; i < first; ++i) issue_w(i, i);
            grid_dependency_wait();
            for (; issued < first; ++issued) issue_x(issued, issued);
        } else {
            grid_dependency_wait();
            for (; issued < first; ++issued) {
                issue(issued, issued);
                if (issued == 0) TINYM_TRACE(11);
            }
        }
        // Let the next kernel in the stream start its own prologue on SMs
        // as they free up (it still waits for this grid to complete).
        grid_launch_dependents();
        for (int s = 0; s < stages; ++s) mbar_init(empty_bar(s), 1);
        mbar_init(acc_bar, 1);
        mbar_init(red_bar, 1);
        mbar_init(tmem_bar, 4);
        *abort_flag = 0u;
        fence_mbar_init();
        TINYM_TRACE(1);
        // This CTA's rows arrive from every other rank of the cluster
        // (st.async, completing their bytes on red_bar).
        if (clustered && own_cnt > 0)
            mbar_expect_tx(red_bar, static_cast<uint32_t>((p.split - 1) * own_cnt * red_cols * 4));
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem_d = *tmem_slot;
    if (threadIdx.x == 0) TINYM_TRACE(2);
    // Cluster barrier, one phase: it completes once every CTA of the cluster
    // is resident with its barriers initialised (published by
    // fence.mbarrier_init.release.cluster); waited on only before the first
    // remote store, long after it has completed.  The arrive is relaxed: a
    // release arrive here measurably delays the first ring-full's landing.
    // (red_bar's expect_tx needs no ordering against the remote
    // complete_tx: the transaction count may go transiently negative.)
    if (clustered) cluster_arrive_relaxed();

    float acc[MMA_N];
    bool have_acc = false;
    float alpha = 0.f;

    // Epilogue thread (warp w, lane t) holds TMEM lane 32*(w%4)+t, which is
    // tile row (w%4)*kRowsPerWarp + t for t < kRowsPerWarp.
    const int row = (warp & 3) * kRowsPerWarp + lane;
    const bool epi = warp >= 2;
    const bool row_ok = epi && lane < kRowsPerWarp;
    const bool row_mine = row_ok && row >= own_lo && row < own_lo + own_cnt;
    // Split-K senders: the owner's receive slot and barrier in cluster
    // addresses, computed while the mainloop runs (off the output path).
    uint32_t send_dst = 0u, send_bar = 0u;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer (refills the ring as slots free up)
            // issued == min(stages, n_issue) here: slot 0 comes round again with
            // the parity of its first use (0).
            int s = 0;
            uint32_t ph = 0u;
            for (; issued < n_issue; ++issued) {
                if (!mbar_wait_inline(empty_bar(s), ph, guard, kErrProducerWait, true)) break;
                issue(issued, s);
                if (++s == stages) {
                    s = 0;
                    ph ^= 1u;
                }
            }
            if (*abort_flag) {
                // Drain the copies still in flight before shared memory is released.
                for (int j = max(0, issued - stages); j < issued; ++j)
                    mbar_drain(full_bar(j % stages), (j / stages) & 1, guard, kErrDrain);
                if (CHUNKS > 1 && issued == nkb)
                    for (int c = 1; c < last_chunks; ++c) mbar_drain(tail_bar(c), 0, guard, kErrDrain);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer: the whole warp runs the loop, lane 0
        // waits for each stage, one elected lane issues its MMAs and the
        // commit.  The shared-memory descriptors are a per-ring base plus the
        // stage offset plus compile-time K steps (the start-address field
        // [0,14) cannot carry: every address is below 2^18).
        const uint32_t tmem_u = __shfl_sync(0xFFFFFFFFu, tmem_d, 0);
        const uint64_t da0 = sw128_kmajor_desc(w_ring);
        const uint64_t db0 = sw128_kmajor_desc(x_ring);
        int s = 0;
        uint32_t ph = 0u;
        int i = 0;
        for (; i < nkb; ++i) {
            bool ok = true;
            if (lane == 0) ok = mbar_wait_inline(full_bar(s), ph, guard, kErrMmaWait, true);
            if (!__shfl_sync(0xFFFFFFFFu, ok, 0)) break;
            if (lane == 0 && i == 0) TINYM_TRACE(3);
            if (lane == 0 && i == nkb - 1) TINYM_TRACE(4);
            tc_fence_after_sync();
            const uint64_t da = da0 + static_cast<uint64_t>((s * kWStage) >> 4);
            const uint64_t db = db0 + static_cast<uint64_t>((s * kXStageBytes) >> 4);
            const uint32_t acc0 = i > 0 ? 1u : 0u;  // the CTA's first MMA overwrites D
            const bool split_last = CHUNKS > 1 && i == nkb - 1;
            if (elect_one()) {
#pragma unroll
                for (int c = 0; c < CHUNKS; ++c) {
                    if (split_last && c > 0) {
                        if (c >= last_chunks) break;
                        if (!mbar_wait_inline(tail_bar(c), 0u, guard, kErrMmaWait, true)) break;
                        tc_fence_after_sync();
                    }
#pragma unroll
                    for (int kk = 0; kk < kBlockK / 32; ++kk) {
                        umma_e4m3(tmem_u, da + static_cast<uint64_t>((c * kWChunk + kk * 32) >> 4),
                                  db + static_cast<uint64_t>((c * kXChunkBytes + kk * 32) >> 4),
                                  kIdesc, (c | kk) ? 1u : acc0);
                    }
                }
                // frees the slot once these MMAs retire; the last stage's
                // commit completes the accumulator instead
                umma_commit(i < nkb - 1 ? empty_bar(s) : acc_bar);
            }
            __syncwarp();
            if (++s == stages) {
                s = 0;
                ph ^= 1u;
            }
        }
        if (i < nkb) {
            // An abort: the accumulator barrier completes once every MMA
            // issued so far has retired (committed by the lane that issued
            // them, as in the loop).
            if (elect_one()) umma_commit(acc_bar);
            __syncwarp();
        }
        if (lane == 0) {
            if (*abort_flag) mbar_drain(acc_bar, 0, guard, kErrDrain);
            // Free TMEM as soon as every epilogue warp has read it (each
            // arrives even without an accumulator), off the output path.
            mbar_drain(tmem_bar, 0, guard, kErrDrain);
        }
        __syncwarp();
        tc_fence_after_sync();
        tmem_dealloc(tmem_d, kTmemCols);
        if (threadIdx.x == 32) TINYM_TRACE(9);
    } else {
        // ---------------- epilogue warps 2..5: TMEM lanes 32*(warp%4) ..
        grid_dependency_wait();  // alpha may be written by the previous kernel
        // issued early (a volatile load stays ahead of the accumulator wait):
        // its latency hides behind the mainloop
        if (p.alpha_ptr)
            asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(alpha) : "l"(p.alpha_ptr) : "memory");
        else
            alpha = p.alpha;
        // The cluster barrier (every CTA of the cluster resident, barriers
        // initialised) completes long before the first remote store; waiting
        // here keeps the wait off the output path.
        if (clustered) cluster_wait_acquire();
        if (clustered && row_ok && !row_mine) {
            const int owner = row / rpo;
            const int slot = split_idx < owner ? split_idx : split_idx - 1;
            send_dst = dsmem_map(smem_u32(red), static_cast<uint32_t>(owner)) +
                       static_cast<uint32_t>(slot * red_rank_bytes +
                                             (row - owner * rpo) * kRedStride * 4);
            send_bar = dsmem_map(red_bar, static_cast<uint32_t>(owner));
        }
        // tcgen05.ld is .sync.aligned: the whole warp takes the same branch.
        const bool ready =
            mbar_wait_inline(acc_bar, 0, guard, kErrEpilogueWait, true) && !*abort_flag;
        if (threadIdx.x == 64) TINYM_TRACE(16);
        if (__all_sync(0xFFFFFFFFu, ready)) {
            tc_fence_after_sync();
            const uint32_t taddr = tmem_d + (static_cast<uint32_t>((warp & 3) * 32) << 16);
            if constexpr (MMA_N == 8) {
                tmem_ld_x8(taddr, acc);
            } else {
                tmem_ld_x16(taddr, acc);
            }
            have_acc = true;
            if (threadIdx.x == 64) TINYM_TRACE(5);
        }
        if (clustered && row_ok && !row_mine) {
            // Split-K: push this row's partial sums to the owner's block for
            // this rank straight away (TMEM is released just after).  Every
            // such thread always sends (zeros if it has no accumulator) so
            // the owner's wait ends.
#pragma unroll
            for (int c = 0; c < MMA_N; c += 4) {
                if (c < red_cols) {
                    float v[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) v[j] = have_acc ? acc[c + j] : 0.f;
                    st_async_v4(send_dst + 16u * (c / 4), v, send_bar);
                }
            }
            if (threadIdx.x == 160) TINYM_TRACE(14);
        }
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(tmem_bar);
    }
    // Warps 0 and 1 are done (the producer and the MMA warp exit here; the
    // MMA warp has freed TMEM).  No CTA-wide barrier follows: the epilogue
    // warps finish the reduction and the stores on their own.
    if (warp < 2) return;

    // ---------------- split-K reduce-scatter through distributed shared memory
    // (the senders pushed their rows right after reading the accumulator)
    if (clustered) {
        if (threadIdx.x == 64) TINYM_TRACE(6);
        if (row_mine) {
            // Owner: wait for the other ranks' partials of this row (bounded),
            // then add all ranks in K order (rank 0 first), so the result
            // does not depend on arrival order or on which rank owns the row.
            const bool got = mbar_wait_inline(red_bar, 0, guard, kErrReduceWait, false);
            if (threadIdx.x == 64) TINYM_TRACE(7);
            if (got && have_acc) {
                // Ranks in order (rank 0 first); the loop is unrolled so that
                // the compiler can issue every rank's loads before the adds.
                const float* mine = red + (row - own_lo) * kRedStride;
                float sum[MMA_N];
#pragma unroll
                for (int c = 0; c < MMA_N; ++c) sum[c] = 0.f;
#pragma unroll
                for (int r = 0; r < kMaxSplit; ++r) {
                    if (r < p.split) {
                        if (r == split_idx) {
#pragma unroll
                            for (int c = 0; c < MMA_N; ++c) sum[c] += acc[c];
                        } else {
                            const float4* part = reinterpret_cast<const float4*>(
                                mine + (r < split_idx ? r : r - 1) * (red_rank_bytes / 4));
#pragma unroll
                            for (int c = 0; c < MMA_N / 4; ++c) {
                                if (4 * c < red_cols) {
                                    const float4 q = part[c];
                                    sum[4 * c + 0] += q.x;
                                    sum[4 * c + 1] += q.y;
                                    sum[4 * c + 2] += q.z;
                                    sum[4 * c + 3] += q.w;
                                }
                            }
                        }
                    }
                }
#pragma unroll
                for (int c = 0; c < MMA_N; ++c) acc[c] = sum[c];
            } else {
                have_acc = false;
            }
            if (threadIdx.x == 64) TINYM_TRACE(12);
        }
    }

    // ---------------- output: each owner thread converts its row's M values
    // and stores them straight from registers (for each m, the lanes of a
    // warp write consecutive N: one coalesced segment per warp and m).
    if (threadIdx.x == 64) TINYM_TRACE(15);
    if (have_acc && row_mine) {
        const int n = tile * TILE_M + row;
        if (n < p.n) {
            // Destinations: y, or this rank's column block of every rank's
            // full Y (peer stores over NVLink for r != rank).
            const int ndst = p.n_peers > 0 ? p.n_peers : 1;
#pragma unroll 1
            for (int d = 0; d < ndst; ++d) {
                __nv_bfloat16* dst = (p.n_peers > 0 ? p.peer_y[d] : p.y) + n;
#pragma unroll
                for (int m = 0; m < MMA_N; ++m)
                    if (m < p.m) dst[static_cast<size_t>(m) * p.ldy] = __float2bfloat16_rn(acc[m] * alpha);
            }
        }
    }
    if (threadIdx.x == 64) TINYM_TRACE(8);
    if (p.n_peers > 0) {
        // Every store of this CTA (the named barrier orders them before
        // thread 64), then one release per rank at system scope: its
        // counter grows by the elements this CTA wrote.
        epilogue_bar_sync();
        if (threadIdx.x == 64 && !*abort_flag) {
            const int n0 = tile * TILE_M;
            const int cols = max(0, min(own_cnt, p.n - (n0 + own_lo)));
            const unsigned long long cnt = static_cast<unsigned long long>(p.m) * cols;
            fence_acq_rel_sys();
            for (int d = 0; d < p.n_peers; ++d) red_relaxed_sys_add_u64(p.peer_flag[d], cnt);
            if (blockIdx.x == 0 && blockIdx.y == 0) {
                // Bounded wait for every rank's rows of this call.
                const uint64_t t0 = globaltimer_ns();
                while (ld_acquire_sys_u64(p.peer_flag[p.rank]) < p.gather_target) {
                    if (globaltimer_ns() - t0 > p.timeout_ns) {
                        report_timeout(&g_err_word, p.err_host, kErrPeerWait);
                        break;
                    }
                    __nanosleep(32);
                }
            }
        }
    }
    if (threadIdx.x == 64) {
        TINYM_TRACE(17);
        TINYM_TRACE_NS(1);
    }
}

// =====================================================================
// CUDA-core M = 1 kernel
// =====================================================================
template <int CWARPS>
__global__ void __launch_bounds__(32 * (CWARPS + 1), 1)
    tinym_simt_m1_kernel(const __grid_constant__ CUtensorMap tm_w,
                         const __grid_constant__ CUtensorMap tm_x, const TinymParams p) {
    static_assert(CWARPS == 4 || CWARPS == 8, "CWARPS must be 4 or 8");
    constexpr int kXStageBytes = kBlockK;  // one unswizzled 128-byte X row
    constexpr uint32_t kStageTx = kWStageBytes + kXStageBytes;
    constexpr int kRowsPerWarp = kTileRows / CWARPS;
    constexpr int kPasses = kRowsPerWarp / 4;  // 4 rows per warp instruction

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);
    const SmemLayout L = smem_layout(p.stages, kWStageBytes, kXStageBytes, p.split, kTileRows * 4);
    const uint32_t s_base = smem_u32(smem);
    const uint32_t w_ring = s_base + L.w_off;
    const uint32_t x_ring = s_base + L.x_off;
    const uint32_t bars = s_base + L.bar_off;
    const int stages = p.stages;
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (stages + s); };
    volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + L.misc_off + 4);
    float* red = reinterpret_cast<float*>(smem + L.red_off);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int split_idx = blockIdx.x;
    const int tile = blockIdx.y;
    const int kb0 = split_idx * p.kb_per_split;
    const int kb1 = min(kb0 + p.kb_per_split, p.kb_total);
    const int nkb = kb1 - kb0;
    const int n_issue = (p.flags & kFlagInjectNoLoads) ? 0 : nkb;

    const WaitGuard guard{abort_flag, &g_err_word, p.timeout_ns, p.err_host};

    int issued = 0;
    uint64_t pol_w = 0, pol_x = 0;
    auto issue = [&](int i, int s) {  // stage i into ring slot s (= i mod stages)
        const int kc = (kb0 + i) * kBlockK;
        mbar_expect_tx(full_bar(s), kStageTx);
        tma_load_2d(w_ring + s * kWStageBytes, &tm_w, full_bar(s), kc, tile * kTileRows, pol_w);
        tma_load_2d(x_ring + s * kXStageBytes, &tm_x, full_bar(s), kc, 0, pol_x);
    };
    if (threadIdx.x == 0) {
        tma_prefetch_desc(&tm_w);
        tma_prefetch_desc(&tm_x);
        for (int s = 0; s < stages; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), CWARPS);
        }
        *abort_flag = 0u;
        fence_mbar_init();
        fence_proxy_async_smem();
        pol_w = l2_policy_w();
        pol_x = l2_policy_evict_last();
        grid_dependency_wait();
        for (; issued < min(stages, n_issue); ++issued) issue(issued, issued);  // first ring-full
        grid_launch_dependents();
    }
    __syncthreads();
    if (p.split > 1) cluster_arrive_relaxed();

    float acc[kPasses];
#pragma unroll
    for (int i = 0; i < kPasses; ++i) acc[i] = 0.f;
    bool have_acc = false;
    const int sub = lane >> 3;    // which of the 4 rows of a pass
    const int chunk = lane & 7;   // which 16-byte chunk of the 128-byte row
    const int rbase = (warp - 1) * kRowsPerWarp;

    if (warp == 0) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0u;
            for (; issued < n_issue; ++issued) {
                if (!mbar_wait(empty_bar(s), ph, guard, kErrProducerWait)) break;
                issue(issued, s);
                if (++s == stages) {
                    s = 0;
                    ph ^= 1u;
                }
            }
            if (*abort_flag) {
                for (int j = max(0, issued - stages); j < issued; ++j)
                    mbar_drain(full_bar(j % stages), (j / stages) & 1, guard, kErrDrain);
            }
        }
    } else {
        bool ok = true;
        int s = 0;
        uint32_t ph = 0u;
        for (int i = 0; i < nkb; ++i) {
            if (!mbar_wait(full_bar(s), ph, guard, kErrConsumerWait)) {
                ok = false;
                break;
            }
            const uint8_t* xs = smem + L.x_off + s * kXStageBytes;
            const uint8_t* ws = smem + L.w_off + s * kWStageBytes;
            float xv[16];
            {
                const uint4 raw = *reinterpret_cast<const uint4*>(xs + chunk * 16);
                const uint32_t wd[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 lo = e4m3x2_to_f32x2(wd[j]);
                    const float2 hi = e4m3x2_to_f32x2(wd[j] >> 16);
                    xv[4 * j + 0] = lo.x;
                    xv[4 * j + 1] = lo.y;
                    xv[4 * j + 2] = hi.x;
                    xv[4 * j + 3] = hi.y;
                }
            }
#pragma unroll
            for (int pp = 0; pp < kPasses; ++pp) {
                const int r = rbase + pp * 4 + sub;
                const int phys = chunk ^ (r & 7);  // 128B swizzle: 16B chunk c of row r
                const uint4 raw = *reinterpret_cast<const uint4*>(ws + r * kBlockK + phys * 16);
                const uint32_t wd[4] = {raw.x, raw.y, raw.z, raw.w};
                float a = acc[pp];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 lo = e4m3x2_to_f32x2(wd[j]);
                    const float2 hi = e4m3x2_to_f32x2(wd[j] >> 16);
                    a = fmaf(lo.x, xv[4 * j + 0], a);
                    a = fmaf(lo.y, xv[4 * j + 1], a);
                    a = fmaf(hi.x, xv[4 * j + 2], a);
                    a = fmaf(hi.y, xv[4 * j + 3], a);
                }
                acc[pp] = a;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty_bar(s));
            if (++s == stages) {
                s = 0;
                ph ^= 1u;
            }
        }
        if (ok && !*abort_flag) {
#pragma unroll
            for (int pp = 0; pp < kPasses; ++pp) {
                float v = acc[pp];
                v += __shfl_xor_sync(0xFFFFFFFFu, v, 1);
                v += __shfl_xor_sync(0xFFFFFFFFu, v, 2);
                v += __shfl_xor_sync(0xFFFFFFFFu, v, 4);
                acc[pp] = v;
            }
            have_acc = true;
        }
    }
    __syncwarp();

    const bool writer = have_acc && chunk == 0;
    if (p.split == 1) {
        if (writer) {
            grid_dependency_wait();
            const float alpha = load_alpha(p);
#pragma unroll
            for (int pp = 0; pp < kPasses; ++pp) {
                const int n_idx = tile * kTileRows + rbase + pp * 4 + sub;
                if (n_idx < p.n) p.y[n_idx] = __float2bfloat16_rn(acc[pp] * alpha);
            }
        }
    } else {
        __syncwarp();
        cluster_wait_acquire();
        if (writer && split_idx > 0) {
            const uint32_t remote = dsmem_map(smem_u32(red), 0);
#pragma unroll
            for (int pp = 0; pp < kPasses; ++pp)
                dsmem_st_f32(remote + 4u * ((split_idx - 1) * kTileRows + rbase + pp * 4 + sub),
                             acc[pp]);
        }
        __syncwarp();
        cluster_arrive_release();
        cluster_wait_acquire();
        if (writer && split_idx == 0) {
            grid_dependency_wait();
            const float alpha = load_alpha(p);
#pragma unroll
            for (int pp = 0; pp < kPasses; ++pp) {
                const int r = rbase + pp * 4 + sub;
                const int n_idx = tile * kTileRows + r;
                if (n_idx < p.n) {
                    float v = acc[pp];
                    for (int q = 1; q < p.split; ++q) v += red[(q - 1) * kTileRows + r];
                    p.y[n_idx] = __float2bfloat16_rn(v * alpha);
                }
            }
        }
    }
    __syncthreads();
}

// =====================================================================
// Weight repack into the packed layout (run once, e.g. by prepare_weights)
// =====================================================================
// One thread per 16-byte vector of the packed tensor: coalesced stores, and
// each warp reads two 128-byte row segments of W.
__global__ void __launch_bounds__(256)
    tinym_pack_weights_kernel(const uint4* __restrict__ w, uint4* __restrict__ out, int64_t n,
                              int64_t k, int64_t kc, int64_t total_vecs) {
    for (int64_t v = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; v < total_vecs;
         v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t b16 = v & 7;                   // 16-byte column within the chunk
        const int64_t r = (v >> 3) & (kPackRows - 1);  // row within the tile
        const int64_t tc = v >> 10;                  // tile * kc + chunk
        const int64_t row = (tc / kc) * kPackRows + r;
        const int64_t col = (tc % kc) * 128 + b16 * 16;
        uint4 val = make_uint4(0u, 0u, 0u, 0u);
        if (row < n && col < k) val = __ldg(w + (row * k + col) / 16);
        out[v] = val;
    }
}

}  // namespace tinym
