// q3k_quant.cu -- Q3_K weights: ggml block_q3_K rows into the device tile
// layout of q3k_core.cuh, and the block decoder (ggml dequantize_row_q3_K).
#include "common.cuh"
#include "kernels.h"
#include "runtime.h"
#include "q3k_core.cuh"

namespace smeai {

namespace {

// One thread per (group, super-block, lane = row of the group).  A 110-byte
// block is 2-byte aligned in a row-major ggml tensor, so it is read as 55
// halfwords.  Rows past n_rows become zero blocks.
__global__ void q3k_repack_kernel(const uint8_t* __restrict__ src, int64_t n_rows, int nb, int64_t n_groups,
                                  uint8_t* __restrict__ tiles) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_groups * nb * 32) return;
  const int lane = (int)(i & 31);
  const int64_t gb = i >> 5;
  const int64_t group = gb / nb;
  const int b = (int)(gb % nb);
  const int64_t row = group * 32 + lane;
  uint32_t w[28];  // block bytes 0..111 as words (bytes 110, 111 zero)
  if (row < n_rows) {
    const uint16_t* s = reinterpret_cast<const uint16_t*>(src + (row * nb + b) * (int64_t)kQ3KBlockBytes);
#pragma unroll
    for (int k = 0; k < 27; ++k) w[k] = (uint32_t)s[2 * k] | ((uint32_t)s[2 * k + 1] << 16);
    w[27] = (uint32_t)s[54];
  } else {
#pragma unroll
    for (int k = 0; k < 28; ++k) w[k] = 0u;
  }
  // block words: 0..7 hmask, 8..23 qs, 24..26 scales, 27 d
  uint4* t4 = reinterpret_cast<uint4*>(tiles + gb * (int64_t)kQ3KTileBytes);
#pragma unroll
  for (int c = 0; c < 4; ++c) t4[c * 32 + lane] = make_uint4(w[8 + 4 * c], w[9 + 4 * c], w[10 + 4 * c], w[11 + 4 * c]);
  t4[4 * 32 + lane] = make_uint4(w[0], w[1], w[2], w[3]);
  t4[5 * 32 + lane] = make_uint4(w[4], w[5], w[6], w[7]);
  t4[6 * 32 + lane] = make_uint4(w[24], w[25], w[26], w[27]);
}

// Weight i of a block: d * (scale_j - 32) * q_i, two roundings (d * scale,
// then * q) as ggml's dequantize_row_q3_K.  One thread per weight.
__global__ void q3k_dequantize_kernel(const uint8_t* __restrict__ w, int64_t k_total, float* __restrict__ y) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= k_total) return;
  const uint8_t* blk = w + (i / QK_K) * kQ3KBlockBytes;
  const int e = (int)(i % QK_K);
  const int half = e / 128, within = e % 128, plane = within / 32, l = within % 32, j = e / 16;
  const int q = ((blk[32 + half * 32 + l] >> (2 * plane)) & 3) - (((blk[l] >> (4 * half + plane)) & 1) ? 0 : 4);
  const int lo = j < 8 ? (blk[96 + j] & 0xF) : (blk[96 + j - 8] >> 4);
  const int hi = (blk[104 + (j & 3)] >> (2 * (j >> 2))) & 3;
  const int sc = (lo | (hi << 4)) - 32;
  const float d = __half2float(__ushort_as_half((unsigned short)(blk[108] | (blk[109] << 8))));
  y[i] = __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
}

}  // namespace

size_t q3k_tile_bytes(int64_t n_rows, int64_t k) {
  const int64_t groups = (n_rows + kRowsPerGroup - 1) / kRowsPerGroup;
  return (size_t)groups * (size_t)(k / QK_K) * kQ3KTileBytes;
}

int q3k_repack_into(const void* w_blocks_dev, int64_t n_rows, int64_t k, uint8_t* tiles, Q2KWeight* out,
                    cudaStream_t stream) {
  if (!w_blocks_dev || !tiles || !out || n_rows <= 0 || k <= 0 || k % QK_K) {
    set_last_error("q3k_repack: bad arguments (rows=%lld k=%lld)", (long long)n_rows, (long long)k);
    return kBadArgument;
  }
  if ((reinterpret_cast<uintptr_t>(w_blocks_dev) & 1) || (reinterpret_cast<uintptr_t>(tiles) & 15)) {
    set_last_error("q3k_repack: blocks must be 2-byte and tiles 16-byte aligned");
    return kBadArgument;
  }
  Q2KWeight w;
  w.fmt = kFmtQ3K;
  w.n_rows = n_rows;
  w.k = k;
  w.nb = (int)(k / QK_K);
  w.n_groups = (n_rows + kRowsPerGroup - 1) / kRowsPerGroup;
  w.bytes = q3k_tile_bytes(n_rows, k);
  w.tiles = tiles;
  SMEAI_CUDA_TRY(cudaGetDevice(&w.device));
  const int64_t threads = w.n_groups * w.nb * 32;
  SMEAI_CUDA_TRY(launch(q3k_repack_kernel, dim3((unsigned)((threads + 255) / 256)), dim3(256), 0, stream,
                        static_cast<const uint8_t*>(w_blocks_dev), n_rows, w.nb, w.n_groups, tiles));
  *out = w;
  return kOk;
}

int q3k_repack(const void* w_blocks_dev, int64_t n_rows, int64_t k, Q2KWeight* out, cudaStream_t stream) {
  if (n_rows <= 0 || k <= 0 || k % QK_K) {
    set_last_error("q3k_repack: bad arguments (rows=%lld k=%lld)", (long long)n_rows, (long long)k);
    return kBadArgument;
  }
  const size_t bytes = q3k_tile_bytes(n_rows, k);
  uint8_t* tiles = nullptr;
  if (device_malloc((void**)&tiles, bytes) != cudaSuccess) {
    cudaGetLastError();
    set_last_error("q3k_repack: cudaMalloc of %zu bytes failed", bytes);
    return kAllocFailed;
  }
  const int st = q3k_repack_into(w_blocks_dev, n_rows, k, tiles, out, stream);
  if (st != kOk) cudaFree(tiles);
  return st;
}

int q3k_dequantize(const void* w, int64_t k_total, float* y, cudaStream_t stream) {
  if (!w || !y || k_total <= 0 || k_total % QK_K) {
    set_last_error("q3k_dequantize: bad arguments");
    return kBadArgument;
  }
  SMEAI_CUDA_TRY(launch(q3k_dequantize_kernel, dim3((unsigned)((k_total + 255) / 256)), dim3(256), 0, stream,
                        static_cast<const uint8_t*>(w), k_total, y));
  return kOk;
}

}  // namespace smeai
