// q8k_quant.cu -- standalone activation quantizer (fp32 -> ggml block_q8_K),
// optionally preceded by an RMSNorm of the whole row
// (sme_ai_library/src/sme_ai_ops.c:1060-1092: x / sqrt(mean(x^2) + eps), then
// times weight[j] when a weight is given -- two roundings, as there).
// The arithmetic lives in q8k_device.cuh; one warp quantizes one block.
#include "common.cuh"
#include "kernels.h"
#include "q8k_device.cuh"

namespace smeai {

// Plain quantization: warp per block over rows x blocks.
__global__ void q8k_quantize_kernel(const float* __restrict__ x, int64_t ld_x, int nb, int64_t total_blocks,
                                    uint8_t* __restrict__ y) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t blk = warp; blk < total_blocks; blk += nwarps) {
    const int64_t row = blk / nb, b = blk % nb;
    float v[8];
    load8(x + row * ld_x + b * QK_K + lane * 8, v);
    q8k_store_global(q8k_quantize_lane(v), y + blk * Q8K_BLOCK_BYTES);
  }
}

// RMSNorm + quantization, one CTA per row.
__global__ void rms_q8k_quantize_kernel(const float* __restrict__ x, int64_t ld_x, int nb, float eps,
                                        const float* __restrict__ norm_w, uint8_t* __restrict__ y) {
  extern __shared__ float sm_gsum[];  // 8 group sums per block, then 1/rms
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int64_t row = blockIdx.x;
  const float* xr = x + row * ld_x;
  for (int b = warp; b < nb; b += nwarps) {
    float v[8];
    load8(xr + b * QK_K + lane * 8, v);
    const float s = group_sumsq_load8(v);
    if ((lane & 3) == 0) sm_gsum[b * 8 + (lane >> 2)] = s;
  }
  __syncthreads();
  if (warp == 0) {
    const float total = rms_fold_groups(sm_gsum, nb * 8);
    if (lane == 0) sm_gsum[nb * 8] = rms_inv_from_sum(total, nb * QK_K, eps);
  }
  __syncthreads();
  const float inv = sm_gsum[nb * 8];
  for (int b = warp; b < nb; b += nwarps) {
    float v[8];
    load8(xr + b * QK_K + lane * 8, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(v[i], inv);
    if (norm_w) {
      float g[8];
      load8(norm_w + b * QK_K + lane * 8, g);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(v[i], g[i]);
    }
    q8k_store_global(q8k_quantize_lane(v), y + (row * nb + b) * Q8K_BLOCK_BYTES);
  }
}

int q8k_quantize(const float* x, int64_t ld_x, int64_t n_rows, int64_t k, void* y, cudaStream_t stream) {
  if (k <= 0 || k % QK_K != 0 || n_rows <= 0 || ld_x < k) {
    set_last_error("q8k_quantize: k must be a positive multiple of 256 (k=%lld rows=%lld ld=%lld)",
                   (long long)k, (long long)n_rows, (long long)ld_x);
    return kBadArgument;
  }
  const int nb = (int)(k / QK_K);
  const int64_t total = n_rows * nb;
  const int warps_per_cta = 4;
  int64_t ctas = (total + warps_per_cta - 1) / warps_per_cta;
  if (ctas > 148 * 32) ctas = 148 * 32;
  SMEAI_CUDA_TRY(launch(q8k_quantize_kernel, dim3((unsigned)ctas), dim3(32 * warps_per_cta), 0, stream, x, ld_x,
                        nb, total, static_cast<uint8_t*>(y)));
  return kOk;
}

int rms_q8k_quantize(const float* x, int64_t ld_x, int64_t n_rows, int64_t k, float eps, void* y,
                     cudaStream_t stream, const float* norm_w) {
  if (k <= 0 || k % QK_K != 0 || n_rows <= 0 || ld_x < k || n_rows > 0x7fffffff) {
    set_last_error("rms_q8k_quantize: k must be a positive multiple of 256");
    return kBadArgument;
  }
  const int nb = (int)(k / QK_K);
  const int threads = nb >= 16 ? 512 : (nb >= 8 ? 256 : 128);
  SMEAI_CUDA_TRY(launch(rms_q8k_quantize_kernel, dim3((unsigned)n_rows), dim3(threads), (size_t)(8 * nb + 1) * 4,
                        stream, x, ld_x, nb, eps, norm_w, static_cast<uint8_t*>(y)));
  return kOk;
}

}  // namespace smeai
