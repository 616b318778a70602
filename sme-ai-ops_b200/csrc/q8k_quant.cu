// q8k_quant.cu -- activation quantizer (fp32 -> ggml block_q8_K), optionally
// preceded by an RMSNorm of the whole row.
//
// Restates ggml's quantize_row_q8_K (generic C, ggml 0.9.8), the quantizer the
// reference's Q2_K mul_mat applies to every activation row
// (llama.cpp/doc/SME_Q2K_OPTIMIZATION.md:127-131):
//   max   = the value of largest magnitude in the 256-block (first on ties)
//   iscale= -127/max,  q = nearest(iscale*x) capped at 127,  d = 1/iscale
//   bsums = sums of 16 consecutive q.
// nearest() is ggml's nearest_int evaluated as one fused multiply-add with
// the 1.5*2^23 constant, as GCC's default contraction compiles it on an FMA
// target.  An all-zero block gives d = 0 and zero quants and sums.
//
// One warp quantizes one 256-value block; lane l holds values 8l..8l+7.
#include "common.cuh"
#include "kernels.h"

namespace smeai {

// Quantize the 8 values v[] held by this lane as part of one warp-wide block,
// writing the 292-byte ggml block at `out` (4-byte aligned).
__device__ __forceinline__ void quantize_block_warp(const float (&v)[8], uint8_t* out) {
  const int lane = threadIdx.x & 31;
  // largest magnitude, first index on ties
  float amax = 0.f, vmax = 0.f;
  int idx = 0x7fffffff;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float a = fabsf(v[i]);
    if (a > amax) { amax = a; vmax = v[i]; idx = lane * 8 + i; }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    float a2 = __shfl_xor_sync(0xffffffffu, amax, off);
    float v2 = __shfl_xor_sync(0xffffffffu, vmax, off);
    int i2 = __shfl_xor_sync(0xffffffffu, idx, off);
    if (a2 > amax || (a2 == amax && i2 < idx)) { amax = a2; vmax = v2; idx = i2; }
  }
  uint32_t* ow = reinterpret_cast<uint32_t*>(out);
  if (amax == 0.f) {
    ow[1 + 2 * lane] = 0u;
    ow[2 + 2 * lane] = 0u;
    if (lane == 0) ow[0] = 0u;
    if (lane < 8) ow[65 + lane] = 0u;
    return;
  }
  const float iscale = __fdiv_rn(-127.f, vmax);
  int q[8];
  int part = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int r = magic_round_bits(__fmaf_rn(iscale, v[i], kMagic));
    q[i] = r > 127 ? 127 : r;
    part += q[i];
  }
  uint32_t w0 = (q[0] & 0xff) | ((q[1] & 0xff) << 8) | ((q[2] & 0xff) << 16) | ((uint32_t)(q[3] & 0xff) << 24);
  uint32_t w1 = (q[4] & 0xff) | ((q[5] & 0xff) << 8) | ((q[6] & 0xff) << 16) | ((uint32_t)(q[7] & 0xff) << 24);
  ow[1 + 2 * lane] = w0;
  ow[2 + 2 * lane] = w1;
  // bsums: group g = lanes 2g, 2g+1; lanes 4m.. write the pair (2m, 2m+1)
  int gsum = part + __shfl_xor_sync(0xffffffffu, part, 1);
  int other = __shfl_down_sync(0xffffffffu, gsum, 2);
  if ((lane & 3) == 0) ow[65 + (lane >> 2)] = (uint32_t)(gsum & 0xffff) | ((uint32_t)other << 16);
  if (lane == 0) {
    float d = __fdiv_rn(1.f, iscale);
    ow[0] = __float_as_uint(d);
  }
}

__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
    float4 a = *reinterpret_cast<const float4*>(p);
    float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = p[i];
  }
}

// Plain quantization: warp per block over rows x blocks.
__global__ void q8k_quantize_kernel(const float* __restrict__ x, int64_t ld_x, int nb, int64_t total_blocks,
                                    uint8_t* __restrict__ y) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t blk = warp; blk < total_blocks; blk += nwarps) {
    int64_t row = blk / nb, b = blk % nb;
    float v[8];
    load8(x + row * ld_x + b * QK_K + lane * 8, v);
    quantize_block_warp(v, y + blk * Q8K_BLOCK_BYTES);
  }
}

// RMSNorm + quantization, one CTA per row.  The sum of squares is taken in a
// fixed order: per block, lane partials of 8 fused squares, folded at
// distances 16..1; then block sums added in ascending order by one thread.
__global__ void rms_q8k_quantize_kernel(const float* __restrict__ x, int64_t ld_x, int nb, float eps,
                                        uint8_t* __restrict__ y) {
  extern __shared__ float sm_bsum[];  // nb floats + 1
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int64_t row = blockIdx.x;
  const float* xr = x + row * ld_x;
  for (int b = warp; b < nb; b += nwarps) {
    float v[8];
    load8(xr + b * QK_K + lane * 8, v);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s = __fmaf_rn(v[i], v[i], s);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
    if (lane == 0) sm_bsum[b] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float total = 0.f;
    for (int b = 0; b < nb; ++b) total = __fadd_rn(total, sm_bsum[b]);
    float mean = __fdiv_rn(total, (float)(nb * QK_K));
    sm_bsum[nb] = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(mean, eps)));
  }
  __syncthreads();
  const float inv = sm_bsum[nb];
  for (int b = warp; b < nb; b += nwarps) {
    float v[8];
    load8(xr + b * QK_K + lane * 8, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(v[i], inv);
    quantize_block_warp(v, y + (row * nb + b) * Q8K_BLOCK_BYTES);
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
                     cudaStream_t stream) {
  if (k <= 0 || k % QK_K != 0 || n_rows <= 0 || ld_x < k || n_rows > 0x7fffffff) {
    set_last_error("rms_q8k_quantize: k must be a positive multiple of 256");
    return kBadArgument;
  }
  const int nb = (int)(k / QK_K);
  const int threads = nb >= 16 ? 512 : (nb >= 8 ? 256 : 128);
  SMEAI_CUDA_TRY(launch(rms_q8k_quantize_kernel, dim3((unsigned)n_rows), dim3(threads), (size_t)(nb + 1) * 4,
                        stream, x, ld_x, nb, eps, static_cast<uint8_t*>(y)));
  return kOk;
}

}  // namespace smeai
