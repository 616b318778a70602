/* Compiled by tests/test_abi.py with gcc against the public headers and linked
 * against libsmeai_b200.so: checks that a plain C caller (written like the
 * reference's examples/demo_linear.c, with __fp16 arrays) builds against the
 * headers, that the struct layouts match the reference ABI, and that the
 * GPU-free entry points answer. */
#include <stddef.h>
#include <stdio.h>

#include "sme_ai_ops.h"
#include "smeai_q2k.h"

int main(void) {
    __fp16 input[4] = {1, 2, 3, 4};
    sme_ai_workspace ws;
    sme_ai_packed_linear_weight pw;
    printf("sizeof_ws=%zu sizeof_packed=%zu sizeof_fp16=%zu\n", sizeof(ws), sizeof(pw), sizeof(input[0]));
    printf("off_a_pairs=%zu off_tmp_f16=%zu off_attn=%zu off_packed=%zu\n", offsetof(sme_ai_workspace, a_pairs),
           offsetof(sme_ai_workspace, tmp_f16), offsetof(sme_ai_workspace, attn_scores),
           offsetof(sme_ai_packed_linear_weight, packed_weight));
    printf("cntb=%llu cntw=%llu\n", (unsigned long long)sme_ai_cntb(), (unsigned long long)sme_ai_cntw());
    printf("bad_ws=%d\n", (int)sme_ai_workspace_init(NULL, 1, 1, 1));
    printf("bad_zero=%d\n", (int)sme_ai_workspace_init(&ws, 0, 1, 1));
    printf("bad_ref=%d\n", (int)sme_ai_linear_ref_f16f32(NULL, 1, 1, input, 1, NULL, NULL));
    printf("bad_packed=%d\n", (int)sme_ai_linear_sme_packed_f16f32(&ws, input, 1, NULL, NULL, NULL));
    printf("bad_repack=%d\n", smeai_q2k_repack(NULL, 1, 256, NULL));
    printf("bad_mulmat=%d\n", smeai_q2k_mul_mat(NULL, 1, 256, NULL, 1, NULL, 1, NULL));
    printf("block_bytes=%d,%d\n", SMEAI_BLOCK_Q2_K_BYTES, SMEAI_BLOCK_Q8_K_BYTES);
    return 0;
}
