/*
 * sme_ai_ops.h -- sm_100a drop-in for the reference's packed Linear / MLP /
 * SwiGLU operator API (sme_ai_library/include/sme_ai_ops.h).
 *
 * Same symbols, argument order, struct layouts and status codes as the
 * reference for every function on the Linear path; the work runs on a
 * compute-capability-10.x GPU instead of the SME1 FMOPA tile.  Functions of
 * the reference header that are not on the Linear path (attention, Conv2D,
 * pooling, softmax, norms, embedding, sigmoid/tanh) are not provided.
 *
 * Memory: every data pointer may be host memory (as in the reference; the
 * call copies through device staging buffers held by the workspace) or
 * device memory (used in place, no copies).  Calls are synchronous, like the
 * reference's.  Accumulation and outputs are fp32; inputs and weights are
 * IEEE binary16.
 *
 * fp16 type: on Arm the reference's __fp16 is used.  Elsewhere C code gets
 * _Float16 (and, unless SME_AI_NO_FP16_ALIAS is defined, `__fp16` is made a
 * name for it so unmodified reference callers compile); C++ gets uint16_t
 * holding the binary16 bit pattern.  All three are the same 2-byte layout.
 */
#ifndef SME_AI_OPS_H
#define SME_AI_OPS_H

#include <stdint.h>

#if defined(__ARM_FP16_FORMAT_IEEE)
typedef __fp16 sme_ai_fp16;
#elif !defined(__cplusplus) && defined(__FLT16_MAX__)
typedef _Float16 sme_ai_fp16;
#if !defined(SME_AI_NO_FP16_ALIAS) && !defined(__fp16)
#define __fp16 _Float16
#endif
#else
typedef uint16_t sme_ai_fp16;
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes; identical values to the reference (sme_ai_ops.h:39-45). */
typedef enum {
    SME_AI_OK = 0,
    SME_AI_BAD_ARGUMENT = -1,        /* NULL pointer, zero size, shape mismatch */
    SME_AI_ALLOC_FAILED = -2,        /* host or device allocation failed */
    SME_AI_UNSUPPORTED = -3,         /* no compute-capability-10.x GPU */
    SME_AI_WORKSPACE_TOO_SMALL = -4, /* batch / feature size beyond the workspace */
} sme_ai_status;

/*
 * Caller-owned workspace (layout of sme_ai_ops.h:61-79).  The max_* fields
 * bound every later call exactly as in the reference; cntb/cntw report 64/16
 * so benches written for the reference accept the device.  The pointer
 * fields hold DEVICE scratch (tmp_f32, tmp2_f32, tmp_f16) or library
 * bookkeeping (a_pairs); callers must not dereference them.  Not thread-safe:
 * one workspace serves one thread at a time, as in the reference.
 */
typedef struct {
    uint64_t max_batch;
    uint64_t max_in_features;
    uint64_t max_out_features;
    uint64_t cntb;
    uint64_t cntw;
    uint64_t max_h;
    uint64_t max_m_pad;
    uint64_t max_k_pad;
    uint64_t max_n_pad;
    float *a_pairs;
    float *a_mod;
    float *b_pack;
    float *tmp_f32;
    float *tmp2_f32;
    sme_ai_fp16 *tmp_f16;
    float *gemm_c_tile;
    float *attn_scores;
} sme_ai_workspace;

/*
 * Pre-packed Linear weight (layout of sme_ai_ops.h:92-98).  k_pad / n_pad are
 * in_features / out_features rounded up to 16, as in the reference.
 * packed_weight is an opaque, non-NULL token for the device-resident copy:
 * do not dereference it.
 */
typedef struct {
    uint64_t in_features;
    uint64_t out_features;
    uint64_t k_pad;
    uint64_t n_pad;
    float *packed_weight;
} sme_ai_packed_linear_weight;

/* ---- environment (sme_ai_ops.h:100-112) ---------------------------------- */
int sme_ai_has_sme(void);        /* 1 when a compute-capability-10.x GPU is usable */
int sme_ai_has_sme2(void);       /* always 0: no SME2 path exists or is needed */
uint64_t sme_ai_cntb(void);      /* 64: the 512-bit vector length the API implies */
uint64_t sme_ai_cntw(void);      /* 16: the reference tile width */

/* ---- lifecycle (sme_ai_ops.h:122-139) ------------------------------------ */
sme_ai_status sme_ai_workspace_init(sme_ai_workspace *ws, uint64_t max_batch, uint64_t max_in_features,
                                    uint64_t max_out_features);
void sme_ai_workspace_destroy(sme_ai_workspace *ws);

/* weight: [in_features][out_features] fp16, host or device. */
sme_ai_status sme_ai_packed_linear_weight_init(sme_ai_packed_linear_weight *packed, const sme_ai_fp16 *weight,
                                               uint64_t in_features, uint64_t out_features);
void sme_ai_packed_linear_weight_destroy(sme_ai_packed_linear_weight *packed);

/* ---- Linear (sme_ai_ops.h:150-206) ----------------------------------------
 * output[b][o] = sum_k input[b][k] * weight[k][o] (+ bias[o]); bias may be
 * NULL.  input [batch][in], output [batch][out]. */
sme_ai_status sme_ai_linear_ref_f16f32(const sme_ai_fp16 *input, uint64_t batch, uint64_t in_features,
                                       const sme_ai_fp16 *weight, uint64_t out_features, const float *bias,
                                       float *output);
sme_ai_status sme_ai_linear_sme_simple_f16f32(sme_ai_workspace *ws, const sme_ai_fp16 *input, uint64_t batch,
                                              uint64_t in_features, const sme_ai_fp16 *weight,
                                              uint64_t out_features, const float *bias, float *output);
sme_ai_status sme_ai_linear_sme_packed_f16f32(sme_ai_workspace *ws, const sme_ai_fp16 *input, uint64_t batch,
                                              const sme_ai_packed_linear_weight *packed_weight,
                                              const float *bias, float *output);

/* Linear + activation (ReLU max(x,0); GELU tanh form; SiLU x/(1+e^-x)). */
sme_ai_status sme_ai_linear_relu_ref_f16f32(const sme_ai_fp16 *input, uint64_t batch, uint64_t in_features,
                                            const sme_ai_fp16 *weight, uint64_t out_features, const float *bias,
                                            float *output);
sme_ai_status sme_ai_linear_relu_sme_packed_f16f32(sme_ai_workspace *ws, const sme_ai_fp16 *input,
                                                   uint64_t batch, const sme_ai_packed_linear_weight *packed_weight,
                                                   const float *bias, float *output);
sme_ai_status sme_ai_linear_gelu_ref_f16f32(const sme_ai_fp16 *input, uint64_t batch, uint64_t in_features,
                                            const sme_ai_fp16 *weight, uint64_t out_features, const float *bias,
                                            float *output);
sme_ai_status sme_ai_linear_gelu_sme_packed_f16f32(sme_ai_workspace *ws, const sme_ai_fp16 *input,
                                                   uint64_t batch, const sme_ai_packed_linear_weight *packed_weight,
                                                   const float *bias, float *output);
sme_ai_status sme_ai_linear_silu_ref_f16f32(const sme_ai_fp16 *input, uint64_t batch, uint64_t in_features,
                                            const sme_ai_fp16 *weight, uint64_t out_features, const float *bias,
                                            float *output);
sme_ai_status sme_ai_linear_silu_sme_packed_f16f32(sme_ai_workspace *ws, const sme_ai_fp16 *input,
                                                   uint64_t batch, const sme_ai_packed_linear_weight *packed_weight,
                                                   const float *bias, float *output);

/* ---- MLP (sme_ai_ops.h:215-237, 359-380) -----------------------------------
 * hidden = fp16(act(input*fc1 + b1)); output = hidden*fc2 + b2. */
sme_ai_status sme_ai_mlp_relu_ref_f16f32(sme_ai_workspace *ws, const sme_ai_fp16 *input, uint64_t batch,
                                         uint64_t in_features, const sme_ai_fp16 *fc1_weight,
                                         uint64_t hidden_features, const float *fc1_bias,
                                         const sme_ai_fp16 *fc2_weight, uint64_t out_features,
                                         const float *fc2_bias, float *output);
sme_ai_status sme_ai_mlp_relu_sme_packed_f16f32(sme_ai_workspace *ws, const sme_ai_fp16 *input, uint64_t batch,
                                                const sme_ai_packed_linear_weight *fc1_weight,
                                                const float *fc1_bias,
                                                const sme_ai_packed_linear_weight *fc2_weight,
                                                const float *fc2_bias, float *output);
sme_ai_status sme_ai_mlp_gelu_ref_f16f32(sme_ai_workspace *ws, const sme_ai_fp16 *input, uint64_t batch,
                                         uint64_t in_features, const sme_ai_fp16 *fc1_weight,
                                         uint64_t hidden_features, const float *fc1_bias,
                                         const sme_ai_fp16 *fc2_weight, uint64_t out_features,
                                         const float *fc2_bias, float *output);
sme_ai_status sme_ai_mlp_gelu_sme_packed_f16f32(sme_ai_workspace *ws, const sme_ai_fp16 *input, uint64_t batch,
                                                const sme_ai_packed_linear_weight *fc1_weight,
                                                const float *fc1_bias,
                                                const sme_ai_packed_linear_weight *fc2_weight,
                                                const float *fc2_bias, float *output);

/* ---- SwiGLU (sme_ai_ops.h:382-408) ------------------------------------------
 * hidden = fp16(silu(input*gate + bg) * (input*up + bu));
 * output = hidden*down + bd.  gate/up out == down in. */
sme_ai_status sme_ai_swiglu_ref_f16f32(sme_ai_workspace *ws, const sme_ai_fp16 *input, uint64_t batch,
                                       uint64_t in_features, const sme_ai_fp16 *gate_weight,
                                       uint64_t hidden_features, const float *gate_bias,
                                       const sme_ai_fp16 *up_weight, const float *up_bias,
                                       const sme_ai_fp16 *down_weight, uint64_t out_features,
                                       const float *down_bias, float *output);
sme_ai_status sme_ai_swiglu_sme_packed_f16f32(sme_ai_workspace *ws, const sme_ai_fp16 *input, uint64_t batch,
                                              const sme_ai_packed_linear_weight *gate_weight,
                                              const float *gate_bias,
                                              const sme_ai_packed_linear_weight *up_weight, const float *up_bias,
                                              const sme_ai_packed_linear_weight *down_weight,
                                              const float *down_bias, float *output);

/* ---- self-attention (sme_ai_ops.h:410-455) ----------------------------------
 * Q, K, V = input * {q,k,v}_weight + bias   (input [seq_len][model_dim])
 * per head (model_dim / num_heads columns):
 *   p = softmax(Q K^T / sqrtf(head_dim)), causal when `causal` is non-zero
 *   context = p V
 * output = fp16(context) * out_weight + out_bias.
 * Weights are [model_dim][model_dim]; biases may be NULL.  seq_len must not
 * exceed ws->max_batch, model_dim neither max_in_features nor
 * max_out_features (else WORKSPACE_TOO_SMALL); model_dim % num_heads != 0 is
 * BAD_ARGUMENT.  head_dim above 512, or a seq_len whose score rows do not fit
 * the GPU's shared memory (about 50k keys), reports UNSUPPORTED.  The packed
 * variant requires every weight to be model_dim x model_dim. */
sme_ai_status sme_ai_self_attention_ref_f16f32(sme_ai_workspace *ws, const sme_ai_fp16 *input, uint64_t seq_len,
                                               uint64_t model_dim, uint64_t num_heads,
                                               const sme_ai_fp16 *q_weight, const float *q_bias,
                                               const sme_ai_fp16 *k_weight, const float *k_bias,
                                               const sme_ai_fp16 *v_weight, const float *v_bias,
                                               const sme_ai_fp16 *out_weight, const float *out_bias, int causal,
                                               float *output);
sme_ai_status sme_ai_self_attention_sme_packed_f16f32(sme_ai_workspace *ws, const sme_ai_fp16 *input,
                                                      uint64_t seq_len, uint64_t model_dim, uint64_t num_heads,
                                                      const sme_ai_packed_linear_weight *q_weight,
                                                      const float *q_bias,
                                                      const sme_ai_packed_linear_weight *k_weight,
                                                      const float *k_bias,
                                                      const sme_ai_packed_linear_weight *v_weight,
                                                      const float *v_bias,
                                                      const sme_ai_packed_linear_weight *out_weight,
                                                      const float *out_bias, int causal, float *output);

/* ---- elementwise helpers of the Linear path (sme_ai_ops.h:241-270) --------
 * void, silently ignore NULL like the reference; host or device pointers. */
void sme_ai_add_f32(float *output, const float *lhs, const float *rhs, uint64_t count);
void sme_ai_mul_f32(float *output, const float *lhs, const float *rhs, uint64_t count);
void sme_ai_residual_add_f32(float *output, const float *input, const float *residual, uint64_t count);
void sme_ai_add_bias_rowwise_f32(float *output, const float *input, const float *bias, uint64_t rows,
                                 uint64_t cols);
void sme_ai_relu_inplace_f32(float *data, uint64_t count);
void sme_ai_gelu_inplace_f32(float *data, uint64_t count);
void sme_ai_silu_inplace_f32(float *data, uint64_t count);

/* ---- additions with no reference counterpart ------------------------------- */

/* True-fp32 Linear: a packed weight built from fp32 data and an fp32 input.
 * Same loop order as the fp16 operator; the multiply-add is fused. */
sme_ai_status sme_ai_packed_linear_weight_init_f32(sme_ai_packed_linear_weight *packed, const float *weight,
                                                   uint64_t in_features, uint64_t out_features);
sme_ai_status sme_ai_linear_sme_packed_f32f32(sme_ai_workspace *ws, const float *input, uint64_t batch,
                                              const sme_ai_packed_linear_weight *packed_weight,
                                              const float *bias, float *output);

/* Asynchronous device-pointer form of the packed Linear: every pointer is
 * device memory, work is queued on `stream` (a cudaStream_t, NULL = legacy
 * default) and the call returns without waiting.  act: 0 none, 1 ReLU,
 * 2 GELU, 3 SiLU. */
sme_ai_status sme_ai_linear_packed_f16f32_device(const sme_ai_fp16 *input, uint64_t batch,
                                                 const sme_ai_packed_linear_weight *packed_weight,
                                                 const float *bias, int act, float *output, void *stream);

/* Asynchronous device-pointer form of sme_ai_self_attention_sme_packed_f16f32:
 * same checks and results; input, biases and output are device memory, work
 * is queued on `stream` (a cudaStream_t, NULL = legacy default) and the call
 * returns without waiting.  Q, K, the fp16 context and the score matrix
 * live in the workspace's device scratch, so calls sharing a workspace must
 * be ordered on one stream.  For head_dim 32, 64 or 128 and 256 <= seq_len
 * <= 16384 the scores of a chunk of heads (at most 1 GiB, or one head) are
 * kept in a workspace-owned device buffer that the first call needing it
 * allocates (a cudaMalloc, which may synchronize the device). */
sme_ai_status sme_ai_self_attention_packed_f16f32_device(sme_ai_workspace *ws, const sme_ai_fp16 *input,
                                                         uint64_t seq_len, uint64_t model_dim, uint64_t num_heads,
                                                         const sme_ai_packed_linear_weight *q_weight,
                                                         const float *q_bias,
                                                         const sme_ai_packed_linear_weight *k_weight,
                                                         const float *k_bias,
                                                         const sme_ai_packed_linear_weight *v_weight,
                                                         const float *v_bias,
                                                         const sme_ai_packed_linear_weight *out_weight,
                                                         const float *out_bias, int causal, float *output,
                                                         void *stream);

/* The per-head core alone (scores, softmax, weighted sum; the reference's
 * sme_ai_ops.c:1383-1402 loop): q, k, v [seq_len][model_dim] fp32 device
 * arrays, context [seq_len][model_dim] fp16, queued on `stream`.  The score
 * buffer of the tiled shapes (see above) belongs to the calling thread: calls
 * from one thread must be ordered on one stream. */
sme_ai_status sme_ai_self_attention_core_f32_device(const float *q, const float *k, const float *v,
                                                    uint64_t seq_len, uint64_t model_dim, uint64_t num_heads,
                                                    int causal, sme_ai_fp16 *context, void *stream);

/* SwiGLU on packed weights for callers that cannot allocate device memory.
 * No counterpart in the reference.  Some callers may not call cudaMalloc at
 * all: code running under a framework that owns the whole device heap
 * through its own pool allocator, or a steady-state loop that must never make
 * an allocation (which may synchronize the device).  This entry point
 * allocates nothing: every pointer is device memory supplied by the caller
 * (input [batch][in], biases, output [batch][out]); the fp16 hidden state
 * lives in a fixed device array built into the library, 1 MiB
 * (batch * hidden_features <= 524288; larger requests return
 * SME_AI_WORKSPACE_TOO_SMALL with the reason in smeai_last_error()), held on
 * every GPU that loads the library until the process exits.  Work is queued
 * on `stream` (a cudaStream_t, NULL = legacy default) and the call returns
 * without waiting; results equal sme_ai_swiglu_sme_packed_f16f32's.
 * The first call on each device looks up the array's device address (a
 * one-time set-up), so make that first call before any stream capture.  All
 * calls share the one array: calls whose work overlaps on the GPU (different
 * streams, or different host threads on one device) race on it and must be
 * serialized by the caller.  Nothing in the array needs to start at zero:
 * each call writes every hidden value before reading it.  The looked-up
 * address is kept for the life of the process: after a cudaDeviceReset the
 * library's module (and the array with it) is loaded anew, so this entry
 * point must not be called on a device that was reset after its first call. */
sme_ai_status sme_ai_swiglu_packed_f16f32_noalloc(const sme_ai_fp16 *input, uint64_t batch,
                                                  const sme_ai_packed_linear_weight *gate_weight,
                                                  const float *gate_bias,
                                                  const sme_ai_packed_linear_weight *up_weight, const float *up_bias,
                                                  const sme_ai_packed_linear_weight *down_weight,
                                                  const float *down_bias, float *output, void *stream);

#ifdef __cplusplus
}
#endif

#endif
