// elementwise.cu -- the elementwise helpers of the Linear path
// (sme_ai_library/src/sme_ai_ops.c:780-887): add, mul, row-wise bias add.
#include "common.cuh"
#include "elementwise.h"

namespace smeai {

namespace {

__global__ void add_kernel(float* __restrict__ out, const float* __restrict__ a, const float* __restrict__ b,
                           int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = a[i] + b[i];
}

__global__ void mul_kernel(float* __restrict__ out, const float* __restrict__ a, const float* __restrict__ b,
                           int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = a[i] * b[i];
}

__global__ void bias_rows_kernel(float* out, const float* in, const float* __restrict__ bias, int64_t rows,
                                 int64_t cols) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < rows * cols) {
    const float v = in[i];
    out[i] = bias ? v + bias[i % cols] : v;
  }
}

unsigned nblk(int64_t n) { return (unsigned)((n + 255) / 256); }

}  // namespace

int ew_add(float* out, const float* a, const float* b, int64_t n, cudaStream_t s) {
  SMEAI_CUDA_TRY(launch(add_kernel, dim3(nblk(n)), dim3(256), 0, s, out, a, b, n));
  return kOk;
}

int ew_mul(float* out, const float* a, const float* b, int64_t n, cudaStream_t s) {
  SMEAI_CUDA_TRY(launch(mul_kernel, dim3(nblk(n)), dim3(256), 0, s, out, a, b, n));
  return kOk;
}

int ew_bias_rows(float* out, const float* in, const float* bias, int64_t rows, int64_t cols, cudaStream_t s) {
  SMEAI_CUDA_TRY(launch(bias_rows_kernel, dim3(nblk(rows * cols)), dim3(256), 0, s, out, in, bias, rows, cols));
  return kOk;
}

}  // namespace smeai
