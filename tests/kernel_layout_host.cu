// Host-side checks of the index arithmetic the sm_100a kernels share with the
// launcher (csrc/tinym_kernels.cuh: smem_layout, tc_rows_per_owner,
// tc_rows_owned, tc_red_rank_bytes, packed_chunks), over every plan shape the
// launcher accepts.  Built with nvcc and run on the CPU by
// tests/test_kernel_layout.py; no GPU is touched.
//
// What each group guards:
//  * split-K row ownership: every tile row has exactly one owner rank, the
//    owner the senders compute (row / rpo) is that rank, and owned ranges are
//    whole 8-row groups (16-byte BF16 vectors) laid end to end;
//  * shared-memory carve-up: every W and X stage starts on a 1024-byte
//    boundary (the 128-byte swizzle atom the tcgen05 descriptors assume),
//    the split-K receive blocks are 16-byte aligned for st.async v4, the
//    mbarriers 8-byte aligned with room for the last stage's chunk
//    barriers, and the whole carve-up matches the size the host requests
//    (the CUDA-core M = 1 kernel's carve-up as well);
//  * K ranges of a cluster: with the plan check's rule every rank gets at
//    least one K stage, and the last stage's in-range chunk count (the
//    chunked last stage of the TC kernel) lies in [1, chunks].
#include <cstdio>

#include "tinym_kernels.cuh"

namespace {

int g_failures = 0;
long g_checks = 0;

void expect(bool ok, const char* what, long a, long b, long c, long d) {
    ++g_checks;
    if (ok) return;
    if (++g_failures <= 20)
        std::printf("FAIL %s (%ld, %ld, %ld, %ld)\n", what, a, b, c, d);
}

void check_row_ownership() {
    const int tile_ms[2] = {64, 128};
    for (int tile_m : tile_ms) {
        for (int split = 1; split <= tinym::kMaxSplit; ++split) {
            const int rpo = tinym::tc_rows_per_owner(tile_m, split);
            expect(rpo % 8 == 0, "rows per owner is a multiple of 8", tile_m, split, rpo, 0);
            expect(rpo * split >= tile_m, "owners cover the tile", tile_m, split, rpo, 0);
            int next = 0, total = 0;
            for (int r = 0; r < split; ++r) {
                const int cnt = tinym::tc_rows_owned(tile_m, split, r);
                expect(cnt >= 0 && cnt <= rpo, "owned rows within [0, rpo]", tile_m, split, r, cnt);
                if (cnt > 0) {
                    expect(r * rpo == next, "owned ranges end to end", tile_m, split, r, next);
                    expect(cnt % 8 == 0, "owned rows in whole 8-row groups", tile_m, split, r, cnt);
                }
                next += cnt;
                total += cnt;
            }
            expect(total == tile_m, "every row owned once", tile_m, split, total, 0);
            for (int row = 0; row < tile_m; ++row) {
                const int o = row / rpo;  // the senders' owner of this row
                expect(o < split, "owner is a rank of the cluster", tile_m, split, row, o);
                expect(row >= o * rpo && row < o * rpo + tinym::tc_rows_owned(tile_m, split, o),
                       "owner's range holds the row", tile_m, split, row, o);
            }
        }
    }
}

void check_tc_layout() {
    const int chunk_opts[3] = {1, 2, 4};
    const int tile_ms[2] = {64, 128};
    const int mma_ns[2] = {8, 16};
    for (int chunks : chunk_opts)
        for (int tile_m : tile_ms)
            for (int mma_n : mma_ns)
                for (int split = 1; split <= tinym::kMaxSplit; ++split)
                    for (int stages = 2; stages <= 32; ++stages) {
                        const int w_stage = chunks * tile_m * tinym::kBlockK;
                        const int x_stage = chunks * mma_n * tinym::kBlockK;
                        const int red_rank = tinym::tc_red_rank_bytes(mma_n, tile_m, split);
                        const tinym::SmemLayout L =
                            tinym::smem_layout(stages, w_stage, x_stage, split, red_rank);
                        const long key = chunks * 1000 + tile_m;
                        expect(L.w_off % 1024 == 0 && w_stage % 1024 == 0,
                               "W stages on 1024-byte boundaries", key, mma_n, split, stages);
                        expect(tinym::kBlockK * tile_m % 1024 == 0,
                               "W chunks on 1024-byte boundaries", key, mma_n, split, stages);
                        expect(L.x_off == L.w_off + static_cast<uint32_t>(stages * w_stage),
                               "X ring follows the W ring", key, mma_n, split, stages);
                        expect(L.x_off % 1024 == 0 && x_stage % 1024 == 0 &&
                                   (mma_n * tinym::kBlockK) % 1024 == 0,
                               "X stages and chunks on 1024-byte boundaries", key, mma_n, split,
                               stages);
                        expect(L.red_off % 16 == 0 &&
                                   L.red_off >= L.x_off + static_cast<uint32_t>(stages * x_stage),
                               "receive blocks 16-byte aligned after the X ring", key, mma_n,
                               split, stages);
                        expect(red_rank % 16 == 0 &&
                                   (tinym::tc_red_stride(mma_n) * 4) % 16 == 0,
                               "receive rows 16-byte aligned", key, mma_n, split, stages);
                        expect(L.bar_off % 8 == 0 &&
                                   L.bar_off >= L.red_off +
                                                    static_cast<uint32_t>((split - 1) * red_rank),
                               "mbarriers 8-byte aligned after the receive blocks", key, mma_n,
                               split, stages);
                        // full + empty per stage, accumulator, reduction, TMEM
                        // release, chunk barriers 1..chunks-1 of the last stage
                        const uint32_t last_bar = 2u * stages + 2u + (chunks - 1);
                        expect(L.bar_off + 8u * (last_bar + 1) <= L.misc_off,
                               "chunk barriers inside the barrier block", key, mma_n, split,
                               stages);
                        expect(L.misc_off % 4 == 0 && L.bytes == L.misc_off + 16u + 1024u,
                               "misc words and the re-alignment slack", key, mma_n, split, stages);
                    }
}

void check_k_ranges() {
    const int chunk_opts[3] = {1, 2, 4};
    for (int chunks : chunk_opts) {
        const int block_k = chunks * tinym::kBlockK;
        const int k_step = chunks > 1 ? tinym::kBlockK : 16;  // K % 128 == 0 when chunks > 1
        for (int k = k_step; k <= 16384; k += k_step) {
            const int kb = (k + block_k - 1) / block_k;
            for (int split = 1; split <= tinym::kMaxSplit; ++split) {
                const int per = (kb + split - 1) / split;
                if ((split - 1) * per >= kb) continue;  // rejected by the plan check
                int covered = 0;
                for (int r = 0; r < split; ++r) {
                    const int kb0 = r * per;
                    const int kb1 = kb0 + per < kb ? kb0 + per : kb;
                    const int nkb = kb1 - kb0;
                    expect(nkb >= 1, "every rank has a K stage", k, chunks, split, r);
                    covered += nkb;
                    if (chunks > 1) {
                        const int last = k / tinym::kBlockK - (kb1 - 1) * chunks;
                        const int last_chunks = last < chunks ? last : chunks;
                        expect(last_chunks >= 1 && last_chunks <= chunks,
                               "last stage has 1..chunks in-range chunks", k, chunks, split, r);
                    }
                }
                expect(covered == kb, "the ranks cover every K stage once", k, chunks, split, kb);
            }
        }
    }
}

// The CUDA-core M = 1 kernel: 128-row W stages (128-byte swizzle) and one
// unswizzled 128-byte X row per stage; split-K partials of 128 FP32 rows per
// sending rank land in rank 0's receive region.
void check_simt_layout() {
    for (int split = 1; split <= tinym::kMaxSplit; ++split)
        for (int stages = 2; stages <= 32; ++stages) {
            const int x_stage = tinym::kBlockK;
            const int red_rank = tinym::kTileRows * 4;
            const tinym::SmemLayout L =
                tinym::smem_layout(stages, tinym::kWStageBytes, x_stage, split, red_rank);
            expect(L.w_off % 1024 == 0 && tinym::kWStageBytes % 1024 == 0,
                   "SIMT W stages on 1024-byte boundaries", split, stages, 0, 0);
            expect(L.x_off % 128 == 0 && x_stage % 128 == 0,
                   "SIMT X rows on 128-byte boundaries", split, stages, 0, 0);
            expect(L.red_off % 16 == 0 && red_rank % 16 == 0 &&
                       L.red_off >= L.x_off + static_cast<uint32_t>(stages * x_stage),
                   "SIMT receive region 16-byte aligned after the X ring", split, stages, 0, 0);
            expect(L.bar_off % 8 == 0 &&
                       L.bar_off >= L.red_off + static_cast<uint32_t>((split - 1) * red_rank) &&
                       L.bar_off + 8u * (2u * stages + 2u) <= L.misc_off,
                   "SIMT mbarriers 8-byte aligned with room for every stage", split, stages, 0, 0);
        }
}

void check_packed_chunks() {
    for (int64_t k = 16; k <= 16384; k += 16) {
        const int64_t kc = tinym::packed_chunks(k);
        expect(kc % tinym::kPackChunkAlign == 0 && kc * tinym::kBlockK >= k &&
                   (kc - tinym::kPackChunkAlign) * tinym::kBlockK < k,
               "packed K chunks: smallest multiple of the stage that covers K", static_cast<long>(k),
               static_cast<long>(kc), 0, 0);
    }
}

}  // namespace

int main() {
    check_row_ownership();
    check_tc_layout();
    check_simt_layout();
    check_k_ranges();
    check_packed_chunks();
    if (g_failures) {
        std::printf("%d kernel layout check(s) failed\n", g_failures);
        return 1;
    }
    std::printf("kernel layout checks ok (%ld checks)\n", g_checks);
    return 0;
}
