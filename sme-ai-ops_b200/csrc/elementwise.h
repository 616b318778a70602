// elementwise.h -- host launchers of the elementwise helpers (internal).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace smeai {

int ew_add(float* out, const float* a, const float* b, int64_t n, cudaStream_t s);
int ew_mul(float* out, const float* a, const float* b, int64_t n, cudaStream_t s);
int ew_bias_rows(float* out, const float* in, const float* bias, int64_t rows, int64_t cols, cudaStream_t s);

}  // namespace smeai
