/*
 * smeai_oracle.h -- CPU restatement of the reference's hot-path arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links, loads or
 * calls this code.  It exists so that tests, the smoke check and the CPU
 * baseline leg of the benchmark have an independent, readable statement of
 * what every GPU kernel must compute.
 *
 * Two reference paths are restated:
 *
 *  Path A -- sme_ai_library fp16-in / fp32-accumulate operators
 *            (sme_ai_library/src/sme_ai_ops.c).  Each function cites the
 *            reference lines it follows.
 *
 *  Path B -- the ggml Q2_K x Q8_K mul_mat path grafted into llama.cpp
 *            (llama.cpp/doc/SME_Q2K_OPTIMIZATION.md:82-136).  Its source is
 *            third-party ggml 0.9.8 (ggml-quants.c / ggml-cpu/quants.c),
 *            absent from the reference tree; the functions here restate the
 *            published generic-C algorithms of that version.  The Q2_K block
 *            decoding is pinned against gguf-py 0.19.0
 *            (gguf/quants.py Q2_K.dequantize_blocks); Q8_K quantization and the
 *            super-block dot have no reference outputs anywhere, so their
 *            parity against ggml itself is unpinned (known-answer tests only).
 */
#ifndef SMEAI_ORACLE_H
#define SMEAI_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_QK_K 256

/* ggml block_q2_K: 84 bytes per 256 weights (gguf/constants.py:4241). */
typedef struct {
    uint8_t scales[16]; /* low nibble: 4-bit scale, high nibble: 4-bit min */
    uint8_t qs[64];     /* 2-bit quants, 4 per byte                        */
    uint16_t d;         /* fp16 super-block scale for scales               */
    uint16_t dmin;      /* fp16 super-block scale for mins                 */
} orc_block_q2_K;

/* ggml block_q3_K: 110 bytes per 256 weights (gguf/constants.py, Q3_K). */
typedef struct {
    uint8_t hmask[32];  /* high bit of each 3-bit quant                   */
    uint8_t qs[64];     /* low 2 bits, 4 per byte (the Q2_K bit order)     */
    uint8_t scales[12]; /* 16 6-bit scales                                 */
    uint16_t d;         /* fp16 super-block scale                          */
} orc_block_q3_K;

/* ggml block_q6_K: 210 bytes per 256 weights (gguf/constants.py, Q6_K). */
typedef struct {
    uint8_t ql[128];    /* low 4 bits of each 6-bit quant                  */
    uint8_t qh[64];     /* high 2 bits, 4 per byte                         */
    int8_t scales[16];  /* 8-bit sub-block scales                          */
    uint16_t d;         /* fp16 super-block scale                          */
} orc_block_q6_K;

/* ggml block_q8_K: 292 bytes per 256 activations (gguf/constants.py:4246). */
typedef struct {
    float d;
    int8_t qs[256];
    int16_t bsums[16];
} orc_block_q8_K;

/* Rounding of iscale*x in quantize_row_q8_K (see smeai_oracle.c). */
enum { ORC_Q8K_ROUND_FUSED = 0, ORC_Q8K_ROUND_SEPARATE = 1 };
/* Evaluation of the per-super-block float combine in the Q2_K dot. */
enum { ORC_COMBINE_FUSED = 0, ORC_COMBINE_SEPARATE = 1 };

/* ---------------- fp16 helpers ---------------- */
float orc_half_to_float(uint16_t h);
uint16_t orc_float_to_half(float f);
void orc_halves_to_floats(const uint16_t *src, float *dst, uint64_t n);
void orc_floats_to_halves(const float *src, uint16_t *dst, uint64_t n);

/* ---------------- reference test-bench data generators ---------------- */
void orc_lcg_fill_f16(uint16_t *dst, uint64_t count, uint32_t seed);
void orc_lcg_fill_f32(float *dst, uint64_t count, uint32_t seed);

/* ---------------- Path A ---------------- */
enum { ORC_ACT_NONE = 0, ORC_ACT_RELU = 1, ORC_ACT_GELU = 2, ORC_ACT_SILU = 3 };

int orc_linear_f16f32(const uint16_t *input, uint64_t batch, uint64_t in_features,
                      const uint16_t *weight, uint64_t out_features,
                      const float *bias, float *output, int act);
int orc_linear_f32f32(const float *input, uint64_t batch, uint64_t in_features,
                      const float *weight, uint64_t out_features,
                      const float *bias, float *output, int act);
int orc_mlp_f16f32(const uint16_t *input, uint64_t batch, uint64_t in_features,
                   const uint16_t *fc1_weight, uint64_t hidden_features, const float *fc1_bias,
                   const uint16_t *fc2_weight, uint64_t out_features, const float *fc2_bias,
                   float *output, int act);
int orc_swiglu_f16f32(const uint16_t *input, uint64_t batch, uint64_t in_features,
                      const uint16_t *gate_weight, uint64_t hidden_features, const float *gate_bias,
                      const uint16_t *up_weight, const float *up_bias,
                      const uint16_t *down_weight, uint64_t out_features, const float *down_bias,
                      float *output);
void orc_pack_weight_f16_tiles(const uint16_t *weight, float *packed,
                               uint64_t in_features, uint64_t out_features);
/* Self-attention (sme_ai_self_attention_ref_f16f32).  Weights are
 * [model_dim][model_dim] fp16, biases may be NULL.  context16 (optional,
 * seq_len * model_dim halves) receives the fp16 context fed to the output
 * projection. */
int orc_self_attention_f16f32(const uint16_t *input, uint64_t seq_len, uint64_t model_dim, uint64_t num_heads,
                              const uint16_t *q_weight, const float *q_bias,
                              const uint16_t *k_weight, const float *k_bias,
                              const uint16_t *v_weight, const float *v_bias,
                              const uint16_t *out_weight, const float *out_bias,
                              int causal, float *output, uint16_t *context16);

/* ---------------- Path B ---------------- */
void orc_quantize_row_q8_K(const float *x, orc_block_q8_K *y, int64_t k, int rounding);
void orc_quantize_row_q2_K(const float *x, orc_block_q2_K *y, int64_t k);
void orc_dequantize_row_q2_K(const orc_block_q2_K *x, float *y, int64_t k);
void orc_q2k_block_sums(int n, const orc_block_q2_K *x, const orc_block_q8_K *y,
                        int32_t *isum, int32_t *summs);
float orc_vec_dot_q2_K_q8_K(int n, const orc_block_q2_K *x, const orc_block_q8_K *y, int combine);
void orc_q2k_mul_mat(const orc_block_q2_K *w, int64_t n_rows, int64_t k,
                     const orc_block_q8_K *xq, int64_t n_cols, float *y, int64_t ldy,
                     int combine, int n_threads);

/* Q3_K: ggml's generic decode and dot (8 float lanes over positions mod 8),
 * the per-super-block integer sum, and the block-order combine of the GPU. */
enum { ORC_Q3K_GGML = 0, ORC_Q3K_BLOCK_ORDER = 1 };
void orc_q3k_scales(const orc_block_q3_K *x, int8_t sc[16]);      /* scale - 32 */
void orc_dequantize_row_q3_K(const orc_block_q3_K *x, float *y, int64_t k);
void orc_q3k_block_sums(int n, const orc_block_q3_K *x, const orc_block_q8_K *y, int32_t *isum);
float orc_vec_dot_q3_K_q8_K(int n, const orc_block_q3_K *x, const orc_block_q8_K *y, int order);
void orc_q3k_mul_mat(const orc_block_q3_K *w, int64_t n_rows, int64_t k,
                     const orc_block_q8_K *xq, int64_t n_cols, float *y, int64_t ldy,
                     int order, int n_threads);

/* Q6_K: the same three forms (ggml's 8-lane generic dot; the GPU's
 * block-order combine of the same per-block integer). */
void orc_dequantize_row_q6_K(const orc_block_q6_K *x, float *y, int64_t k);
void orc_q6k_block_sums(int n, const orc_block_q6_K *x, const orc_block_q8_K *y, int32_t *isum);
float orc_vec_dot_q6_K_q8_K(int n, const orc_block_q6_K *x, const orc_block_q8_K *y, int order);
void orc_q6k_mul_mat(const orc_block_q6_K *w, int64_t n_rows, int64_t k,
                     const orc_block_q8_K *xq, int64_t n_cols, float *y, int64_t ldy,
                     int order, int n_threads);

/* ---------------- decode-stack helpers ---------------- */
float orc_rms_group_sumsq(const float *x);      /* one 32-value group */
float orc_rms_sumsq(const float *x, int64_t k);  /* k a multiple of 32 */
float orc_rms_inv(const float *x, int64_t k, float eps);
void orc_rmsnorm_quantize_q8_K(const float *x, orc_block_q8_K *y, int64_t k, float eps, int rounding);
void orc_rmsnorm_w_quantize_q8_K(const float *x, const float *weight, orc_block_q8_K *y, int64_t k, float eps,
                                 int rounding);
void orc_silu_mul(const float *g, const float *u, float *h, int64_t n);

#ifdef __cplusplus
}
#endif
#endif
