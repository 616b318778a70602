// linear.h -- host launchers of the fp16 packed-Linear kernels (internal).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace smeai {

// Activation kinds, in the reference's order (sme_ai_ops.c:60-65).
enum Act : int { kActNone = 0, kActRelu = 1, kActGelu = 2, kActSilu = 3 };
enum LinearEpi : int { kEpiF32 = 0, kEpiF16 = 1, kEpiSwiGLU = 2 };

// C[M,N] = act(A[M,K] * B[K,N] + bias), B row-major with leading dim ldb.
int linear_f16(const __half* A, int64_t M, int64_t K, const __half* B, int64_t ldb, int64_t N, const float* bias,
               int act, float* C, cudaStream_t s);
int linear_f16_to_f16(const __half* A, int64_t M, int64_t K, const __half* B, int64_t ldb, int64_t N,
                      const float* bias, int act, __half* C16, cudaStream_t s);
int swiglu_gate_up_f16(const __half* A, int64_t M, int64_t K, const __half* Bg, const __half* Bu, int64_t ldb,
                       int64_t N, const float* bg, const float* bu, __half* H16, cudaStream_t s);
int linear_f32(const float* A, int64_t M, int64_t K, const float* B, int64_t ldb, int64_t N, const float* bias,
               int act, float* C, cudaStream_t s);
int linear_ref_f16(const __half* A, int64_t M, int64_t K, const __half* W, int64_t N, const float* bias, int act,
                   float* C, cudaStream_t s);
int f32_to_f16(const float* x, __half* y, int64_t n, cudaStream_t s);
int silu_mul_f16(const float* g, const float* u, __half* h, int64_t n, cudaStream_t s);
int act_inplace(float* x, int64_t n, int act, cudaStream_t s);
// Per-head scores, softmax and weighted sum of the reference's self-attention:
// Q, K, V [S][D] fp32 (heads of D / heads columns), ctx16 [S][D] fp16.
// `scores` (device, scores_bytes) backs the tiled kernels' score matrix;
// attention_scratch_bytes() gives the size they need (0 when the fused
// one-kernel path serves the shape).  Without it the fused path runs.
size_t attention_scratch_bytes(int64_t S, int64_t D, int64_t heads);
int attention_core(const float* Q, const float* K, const float* V, int64_t S, int64_t D, int64_t heads, int causal,
                   __half* ctx16, float* scores, size_t scores_bytes, cudaStream_t s);
int pack_weight_f16(const __half* w, int64_t K, int64_t N, __half* out, int64_t k_pad, int64_t n_pad,
                    cudaStream_t s);

}  // namespace smeai
