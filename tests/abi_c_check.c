/* abi_c_check.c -- a plain C (C99) caller of include/bwgemm.h, as a maintainer's cgo / FFI binding would be: the
 * header compiles as C, the library links, and the host-only entries answer without a GPU.  Prints the layout of
 * bw_plan (size and field offsets) for the ctypes mirror in gemm-ladder_b200/bwgemm.py to be compared against, then
 * "OK".  Exit status 1 on a wrong answer. */
#include <stddef.h>
#include <stdio.h>
#include <string.h>

#include "bwgemm.h"

#define CHECK(cond)                                             \
    do {                                                        \
        if (!(cond)) {                                          \
            printf("FAIL line %d: %s\n", __LINE__, #cond);      \
            return 1;                                           \
        }                                                       \
    } while (0)

int main(void)
{
    bw_plan p;
    memset(&p, 0, sizeof p);
    /* the rule, host only: BASELINE config 1 on 148 SMs takes SM-pair tiles of 256 x 512 (198 tiles, 2.7 waves) */
    CHECK(bw_gemm_plan(4608, 5632, 8192, 148, 0, &p) == BW_OK);
    CHECK(p.kernel == BW_KERNEL_PAIR && p.bn == 512 && p.tiles == 18 * 11 && p.kblocks == 128);
    /* M = 16: swap-AB, 256-column tiles with their K cut in three on clusters of three SMs */
    CHECK(bw_gemm_plan(16, 8192, 8192, 148, 0, &p) == BW_OK);
    CHECK(p.kernel == BW_KERNEL_SWAP && p.bn == 16 && p.ksplit == 3 && p.wm == 2 && p.grid == 96);
    /* any M >= 1 (M = 1: the tokens rounded up to 16 inside the kernel); N % 64, K % 64 and bad arguments refused
     * before any GPU work */
    CHECK(bw_gemm_plan(1, 8192, 8192, 148, 0, &p) == BW_OK && p.kernel == BW_KERNEL_SWAP && p.bn == 16);
    CHECK(bw_gemm_plan(16, 96, 64, 148, 0, &p) == BW_ERR_SHAPE);
    CHECK(bw_gemm_plan(16, 64, 64, 148, bw_gemm_variant_count(), &p) == BW_ERR_ARG);
    CHECK(bw_gemm_f16((const void*)16, (const void*)16, (void*)16, 16, 32, 64, NULL) == BW_ERR_SHAPE);
    CHECK(bw_gemm_f16(NULL, (const void*)16, (void*)16, 16, 64, 64, NULL) == BW_ERR_ARG);
    CHECK(bw_gemm_variant_count() >= 1 && bw_gemm_variant_name(0) != NULL);
    CHECK(bw_gemm_variant_name(-1) == NULL);
    CHECK(strlen(bw_status_string(BW_ERR_TIMEOUT)) > 0);
    /* the fused reduce-scatter's context: bad ranks and shapes refused first; without a GPU no context is made */
    {
        bw_rs* rs = (bw_rs*)&p; /* not NULL: a refused create must set it to NULL */
        unsigned char handle[BW_RS_HANDLE_BYTES];
        CHECK(bw_rs_create(512, 512, 1, 0, &rs) == BW_ERR_ARG && rs == NULL);
        CHECK(bw_rs_create(512, 512, 2, 2, &rs) == BW_ERR_ARG && rs == NULL);
        CHECK(bw_rs_create(512, 512, 9, 0, &rs) == BW_ERR_ARG);
        CHECK(bw_rs_create(768, 512, 2, 0, &rs) == BW_ERR_SHAPE); /* M % (256 world) != 0 */
        CHECK(bw_rs_create(512, 500, 2, 0, &rs) == BW_ERR_SHAPE);
        CHECK(bw_rs_create(512, 512, 2, 0, NULL) == BW_ERR_ARG);
        CHECK(bw_rs_create(512, 512, 2, 0, &rs) != BW_OK && rs == NULL); /* no device here */
        CHECK(bw_gemm_f16_rs(NULL, (const void*)16, (const void*)16, (void*)16, 64, NULL) == BW_ERR_ARG);
        CHECK(bw_rs_handle(NULL, handle) == BW_ERR_ARG && bw_rs_connect(NULL, handle) == BW_ERR_ARG);
        CHECK(bw_rs_region_bytes(NULL) == 0 && bw_rs_destroy(NULL) == BW_OK);
    }
    printf("bw_plan size %zu kernel %zu bn %zu stages %zu tiles_m %zu tiles_n %zu tiles %zu kblocks %zu grid %zu "
           "dp_tiles %zu sk_tiles %zu splits %zu sk_iters %zu group_rows %zu workspace_bytes %zu counters %zu "
           "smem_bytes %zu tmem_cols %zu ksplit %zu wm %zu dyn %zu\n",
           sizeof(bw_plan), offsetof(bw_plan, kernel), offsetof(bw_plan, bn), offsetof(bw_plan, stages),
           offsetof(bw_plan, tiles_m), offsetof(bw_plan, tiles_n), offsetof(bw_plan, tiles), offsetof(bw_plan, kblocks),
           offsetof(bw_plan, grid), offsetof(bw_plan, dp_tiles), offsetof(bw_plan, sk_tiles),
           offsetof(bw_plan, splits), offsetof(bw_plan, sk_iters), offsetof(bw_plan, group_rows),
           offsetof(bw_plan, workspace_bytes), offsetof(bw_plan, counters), offsetof(bw_plan, smem_bytes),
           offsetof(bw_plan, tmem_cols), offsetof(bw_plan, ksplit), offsetof(bw_plan, wm), offsetof(bw_plan, dyn));
    printf("OK\n");
    return 0;
}
