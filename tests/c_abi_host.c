/*
 * c_abi_host.c -- a plain C99 caller of libtinym_b200.so (no Python, no
 * torch), the way a non-Python binding (cgo, JNI, a C++ server) reaches the
 * library.  Exercises only host-side entry points, so it runs on machines
 * without a GPU: the ABI version, status strings, the shape-dispatch table
 * at the official points, plan validation, the shape gate and the argument
 * checks that reject a call before any CUDA work.  Built and run by
 * tests/test_capi_host.py; prints one line per official point and exits 0
 * when every check holds.
 */
#include <stdio.h>
#include <string.h>

#include "tinym_b200.h"

static int g_fails = 0;

#define CHECK(cond)                                                          \
    do {                                                                     \
        if (!(cond)) {                                                       \
            fprintf(stderr, "check failed at line %d: %s (last error: %s)\n", \
                    __LINE__, #cond, tinym_last_error());                    \
            ++g_fails;                                                       \
        }                                                                    \
    } while (0)

int main(void) {
    static const int64_t points[6][3] = {{1, 6144, 5120}, {9, 6144, 5120}, {1, 5120, 8192},
                                         {9, 5120, 8192}, {1, 5120, 16384}, {9, 5120, 16384}};
    tinym_plan p;
    int64_t bytes = 0;
    int i;

    CHECK(tinym_abi_version() == TINYM_ABI_VERSION);
    CHECK(strcmp(tinym_status_string(TINYM_OK), "TINYM_OK") == 0);
    CHECK(strcmp(tinym_status_string(TINYM_ERR_BAD_PLAN), "TINYM_ERR_BAD_PLAN") == 0);

    /* the dispatch table at the official points (M, K, N) on 148 SMs */
    for (i = 0; i < 6; ++i) {
        const int64_t m = points[i][0], k = points[i][1], n = points[i][2];
        memset(&p, 0, sizeof p);
        CHECK(tinym_select_plan(m, n, k, 148, &p) == TINYM_OK);
        CHECK(p.kernel == TINYM_KERNEL_TC);
        CHECK(p.mma_n >= m);
        CHECK(p.grid_ctas == p.tiles_n * p.split_k && p.grid_ctas <= 148);
        CHECK(p.smem_bytes > 0 && p.smem_bytes <= 232448);
        printf("M=%lld K=%lld N=%lld split=%d stages=%d block_k=%d tile_m=%d ctas=%d\n",
               (long long)m, (long long)k, (long long)n, p.split_k, p.stages, p.block_k,
               p.tile_m, p.grid_ctas);
    }

    /* an explicit plan validates and gets its derived fields */
    memset(&p, 0, sizeof p);
    p.kernel = TINYM_KERNEL_TC;
    p.split_k = 2;
    p.stages = 4;
    p.mma_n = 16;
    CHECK(tinym_check_plan(9, 1000, 4096, &p) == TINYM_OK);
    CHECK(p.block_k == 128 && p.tile_m == 128 && p.tiles_n == 8 && p.grid_ctas == 16);
    p.mma_n = 8; /* MMA N below M */
    CHECK(tinym_check_plan(9, 1000, 4096, &p) == TINYM_ERR_BAD_PLAN);

    /* the shape gate and argument checks, before any CUDA call */
    CHECK(tinym_select_plan(17, 128, 128, 148, &p) == TINYM_ERR_UNSUPPORTED_SHAPE);
    CHECK(strstr(tinym_last_error(), "M must be <= 16") != NULL);
    CHECK(tinym_select_plan(1, 128, 40, 148, &p) == TINYM_ERR_UNSUPPORTED_SHAPE);
    CHECK(tinym_fp8_gemm(NULL, NULL, NULL, 1, 128, 128, 1.0f, 1.0f, NULL) ==
          TINYM_ERR_INVALID_ARGUMENT);
    CHECK(tinym_fp8_gemm_ex((const void*)16, (const void*)32, (void*)64, 64, 1, 128, 128, NULL,
                            1.0f, NULL, NULL) == TINYM_ERR_INVALID_ARGUMENT); /* ldy < N */
    CHECK(tinym_fp8_gemm_ex((const void*)17, (const void*)32, (void*)64, 128, 1, 128, 128, NULL,
                            1.0f, NULL, NULL) == TINYM_ERR_MISALIGNED);

    /* packed-weight and workspace sizes are host arithmetic */
    CHECK(tinym_packed_weight_bytes(5120, 6144, &bytes) == TINYM_OK);
    CHECK(bytes == (int64_t)40 * 48 * 128 * 128);
    CHECK(tinym_quant_workspace_bytes(9, 6144, &bytes) == TINYM_OK);
    CHECK(bytes == 256 + 55296);

    if (g_fails) {
        fprintf(stderr, "%d check(s) failed\n", g_fails);
        return 1;
    }
    printf("c abi host checks ok\n");
    return 0;
}
