// q6k_quant.cu -- Q6_K weights: ggml block_q6_K rows into the device tile
// layout of q6k_core.cuh, and the block decoder (ggml dequantize_row_q6_K).
#include "common.cuh"
#include "kernels.h"
#include "runtime.h"
#include "q6k_core.cuh"

namespace smeai {

namespace {

// One thread per (group, super-block, lane = row of the group).  A 210-byte
// block is 2-byte aligned in a row-major ggml tensor: read as 105 halfwords.
// Rows past n_rows become zero blocks.
__global__ void q6k_repack_kernel(const uint8_t* __restrict__ src, int64_t n_rows, int nb, int64_t n_groups,
                                  uint8_t* __restrict__ tiles) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_groups * nb * 32) return;
  const int lane = (int)(i & 31);
  const int64_t gb = i >> 5;
  const int64_t group = gb / nb;
  const int b = (int)(gb % nb);
  const int64_t row = group * 32 + lane;
  uint32_t w[53];  // block bytes 0..211 as words (bytes 210, 211 zero)
  if (row < n_rows) {
    const uint16_t* s = reinterpret_cast<const uint16_t*>(src + (row * nb + b) * (int64_t)kQ6KBlockBytes);
#pragma unroll
    for (int k = 0; k < 52; ++k) w[k] = (uint32_t)s[2 * k] | ((uint32_t)s[2 * k + 1] << 16);
    w[52] = (uint32_t)s[104];
  } else {
#pragma unroll
    for (int k = 0; k < 53; ++k) w[k] = 0u;
  }
  // block words: 0..31 ql, 32..47 qh, 48..51 scales, 52 d
  uint4* t4 = reinterpret_cast<uint4*>(tiles + gb * (int64_t)kQ6KTileBytes);
#pragma unroll
  for (int c = 0; c < 13; ++c) t4[c * 32 + lane] = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
  reinterpret_cast<uint32_t*>(tiles + gb * (int64_t)kQ6KTileBytes + 13 * 512)[lane] = w[52];
}

// Weight i of a block: d * scale_j * (u - 32), two roundings (d * scale, then
// * q) as ggml's dequantize_row_q6_K.  One thread per weight.
__global__ void q6k_dequantize_kernel(const uint8_t* __restrict__ w, int64_t k_total, float* __restrict__ y) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= k_total) return;
  const uint8_t* blk = w + (i / QK_K) * kQ6KBlockBytes;
  const int e = (int)(i % QK_K);
  const int half = e / 128, within = e % 128, g = within / 32, l = within % 32;
  const int ql = blk[64 * half + l + 32 * (g & 1)];
  const int lo = g < 2 ? (ql & 0xF) : (ql >> 4);
  const int hi = (blk[128 + 32 * half + l] >> (2 * g)) & 3;
  const int q = (lo | (hi << 4)) - 32;
  const int sc = (int)(int8_t)blk[192 + e / 16];
  const float d = __half2float(__ushort_as_half((unsigned short)(blk[208] | (blk[209] << 8))));
  y[i] = __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
}

}  // namespace

size_t q6k_tile_bytes(int64_t n_rows, int64_t k) {
  const int64_t groups = (n_rows + kRowsPerGroup - 1) / kRowsPerGroup;
  return (size_t)groups * (size_t)(k / QK_K) * kQ6KTileBytes;
}

int q6k_repack_into(const void* w_blocks_dev, int64_t n_rows, int64_t k, uint8_t* tiles, Q2KWeight* out,
                    cudaStream_t stream) {
  if (!w_blocks_dev || !tiles || !out || n_rows <= 0 || k <= 0 || k % QK_K) {
    set_last_error("q6k_repack: bad arguments (rows=%lld k=%lld)", (long long)n_rows, (long long)k);
    return kBadArgument;
  }
  if ((reinterpret_cast<uintptr_t>(w_blocks_dev) & 1) || (reinterpret_cast<uintptr_t>(tiles) & 15)) {
    set_last_error("q6k_repack: blocks must be 2-byte and tiles 16-byte aligned");
    return kBadArgument;
  }
  Q2KWeight w;
  w.fmt = kFmtQ6K;
  w.n_rows = n_rows;
  w.k = k;
  w.nb = (int)(k / QK_K);
  w.n_groups = (n_rows + kRowsPerGroup - 1) / kRowsPerGroup;
  w.bytes = q6k_tile_bytes(n_rows, k);
  w.tiles = tiles;
  SMEAI_CUDA_TRY(cudaGetDevice(&w.device));
  const int64_t threads = w.n_groups * w.nb * 32;
  SMEAI_CUDA_TRY(launch(q6k_repack_kernel, dim3((unsigned)((threads + 255) / 256)), dim3(256), 0, stream,
                        static_cast<const uint8_t*>(w_blocks_dev), n_rows, w.nb, w.n_groups, tiles));
  *out = w;
  return kOk;
}

int q6k_repack(const void* w_blocks_dev, int64_t n_rows, int64_t k, Q2KWeight* out, cudaStream_t stream) {
  if (n_rows <= 0 || k <= 0 || k % QK_K) {
    set_last_error("q6k_repack: bad arguments (rows=%lld k=%lld)", (long long)n_rows, (long long)k);
    return kBadArgument;
  }
  const size_t bytes = q6k_tile_bytes(n_rows, k);
  uint8_t* tiles = nullptr;
  if (device_malloc((void**)&tiles, bytes) != cudaSuccess) {
    cudaGetLastError();
    set_last_error("q6k_repack: cudaMalloc of %zu bytes failed", bytes);
    return kAllocFailed;
  }
  const int st = q6k_repack_into(w_blocks_dev, n_rows, k, tiles, out, stream);
  if (st != kOk) cudaFree(tiles);
  return st;
}

int q6k_dequantize(const void* w, int64_t k_total, float* y, cudaStream_t stream) {
  if (!w || !y || k_total <= 0 || k_total % QK_K) {
    set_last_error("q6k_dequantize: bad arguments");
    return kBadArgument;
  }
  SMEAI_CUDA_TRY(launch(q6k_dequantize_kernel, dim3((unsigned)((k_total + 255) / 256)), dim3(256), 0, stream,
                        static_cast<const uint8_t*>(w), k_total, y));
  return kOk;
}

}  // namespace smeai
