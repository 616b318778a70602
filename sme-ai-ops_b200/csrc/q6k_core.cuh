// q6k_core.cuh -- Q6_K weights for the persistent GEMV (q2k_gemv.cu).
//
// ggml block_q6_K (210 bytes per 256 weights): ql[128], qh[64], scales[16]
// (int8), d (fp16).  In each 128-weight half (ql + 64h, qh + 32h), weight
// 32g + l (g = 0..3, l = 0..31) is d * scale_j * (u - 32) with
//   u = (g < 2 ? low : high nibble of ql[l + 32 (g & 1)]) | (qh[l] >> 2g & 3) << 4
// and j = its index / 16 (ggml dequantize_row_q6_K / gguf-py
// Q6_K.dequantize_blocks).
//
// Tile of one (group, super-block): 13 chunks of [32 rows][16 B] -- ql bytes
// 16c..16c+15 (c = 0..7), qh bytes 16(c-8).. (c = 8..11), the 16 scales
// (c = 12) -- then d as [32 rows][4 B] (fp16 + 2 bytes of padding): 6784
// bytes, 212 per row-super-block against ggml's 210.
#pragma once

#include "common.cuh"
#include "q2k_core.cuh"
#include "q3k_core.cuh"

namespace smeai {

constexpr int kQ6KBlockBytes = 210;
constexpr int kQ6KTileBytes = 32 * (13 * 16 + 4);

struct WBlock6 {
  uint4 ql[8];
  uint4 qh[4];
  uint4 sc;
  unsigned d;
};

__device__ __forceinline__ WBlock6 load_wblock6(const uint8_t* tile, int lane) {
  const uint4* t4 = reinterpret_cast<const uint4*>(tile);
  WBlock6 wb;
#pragma unroll
  for (int c = 0; c < 8; ++c) wb.ql[c] = t4[c * 32 + lane];
#pragma unroll
  for (int c = 0; c < 4; ++c) wb.qh[c] = t4[(8 + c) * 32 + lane];
  wb.sc = t4[12 * 32 + lane];
  wb.d = reinterpret_cast<const unsigned*>(tile + 13 * 512)[lane];
  return wb;
}

__device__ __forceinline__ unsigned wblock6_dep(const WBlock6& wb) {
  unsigned d = wb.sc.x ^ wb.sc.y ^ wb.sc.z ^ wb.sc.w ^ wb.d;
#pragma unroll
  for (int c = 0; c < 8; ++c) d ^= wb.ql[c].x ^ wb.ql[c].y ^ wb.ql[c].z ^ wb.ql[c].w;
#pragma unroll
  for (int c = 0; c < 4; ++c) d ^= wb.qh[c].x ^ wb.qh[c].y ^ wb.qh[c].z ^ wb.qh[c].w;
  return d;
}

__device__ __forceinline__ unsigned u4w(const uint4& v, int w) { return w == 0 ? v.x : w == 1 ? v.y : w == 2 ? v.z : v.w; }

// Integer core + float term of super-block b for this lane's row (T tokens):
//   S_j  = sum_{i in j} u_i * q8_i              (dp4a, u in [0, 63])
//   isum = sum_j scale_j * (S_j - 32 * bsums_j) -- ggml's integer total
//   term = (fp32(d) * d_x) * fp32(isum)         (summed in ascending order)
// SUMS: isum_out = isum, summs_out = sum_j scale_j * bsums_j.
template <int T, bool SUMS>
__device__ __forceinline__ void block_terms6(const WBlock6& wb, const ActSmem& m, int aslot, int astride, int nb,
                                             int b, float* terms, int lane, int64_t row, int64_t n_rows,
                                             int32_t* isum_out, int32_t* summs_out) {
  const unsigned scw[4] = {wb.sc.x, wb.sc.y, wb.sc.z, wb.sc.w};
  int acc[T];
#pragma unroll
  for (int t = 0; t < T; ++t) acc[t] = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
#pragma unroll
    for (int p = 0; p < 2; ++p) {  // bytes l = 16p .. 16p + 15 of the half
      const uint4 A = wb.ql[4 * h + p], B = wb.ql[4 * h + 2 + p], H = wb.qh[2 * h + p];
      unsigned u[4][4];  // [g][word]
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const unsigned a = u4w(A, w), bb = u4w(B, w), hh = u4w(H, w);
        u[0][w] = (a & 0x0F0F0F0Fu) | ((hh << 4) & 0x30303030u);
        u[1][w] = (bb & 0x0F0F0F0Fu) | ((hh << 2) & 0x30303030u);
        u[2][w] = ((a >> 4) & 0x0F0F0F0Fu) | (hh & 0x30303030u);
        u[3][w] = ((bb >> 4) & 0x0F0F0F0Fu) | ((hh >> 2) & 0x30303030u);
      }
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const int j = 8 * h + 2 * g + p;  // sub-block = 16-byte activation chunk
        const int sc = sbyte(scw[j >> 2], j & 3);
#pragma unroll
        for (int t = 0; t < T; ++t) {
          const int4 av = m.qs[(aslot + t * astride) * 16 + j];
          int sj = dp4a_us(u[g][0], av.x, 0);
          sj = dp4a_us(u[g][1], av.y, sj);
          sj = dp4a_us(u[g][2], av.z, sj);
          sj = dp4a_us(u[g][3], av.w, sj);
          acc[t] += sc * sj;
        }
      }
    }
  }
  const float dw = __half2float(__ushort_as_half((unsigned short)(wb.d & 0xffffu)));
#pragma unroll
  for (int t = 0; t < T; ++t) {
    const int* bsp = m.bs + (aslot + t * astride) * 8;
    const int4 bs0 = *reinterpret_cast<const int4*>(bsp);
    const int4 bs1 = *reinterpret_cast<const int4*>(bsp + 4);
    int mm = dp2a_lo_ss(bs0.x, scw[0], 0);
    mm = dp2a_hi_ss(bs0.y, scw[0], mm);
    mm = dp2a_lo_ss(bs0.z, scw[1], mm);
    mm = dp2a_hi_ss(bs0.w, scw[1], mm);
    mm = dp2a_lo_ss(bs1.x, scw[2], mm);
    mm = dp2a_hi_ss(bs1.y, scw[2], mm);
    mm = dp2a_lo_ss(bs1.z, scw[3], mm);
    mm = dp2a_hi_ss(bs1.w, scw[3], mm);
    const int isum = acc[t] - 32 * mm;
    if constexpr (SUMS) {
      if (row < n_rows) {
        isum_out[row * nb + b] = isum;
        summs_out[row * nb + b] = mm;
      }
    } else {
      const float dd = __fmul_rn(dw, m.d[aslot + t * astride]);
      terms[(t * nb + b) * 32 + lane] = __fmul_rn(dd, __int2float_rn(isum));
    }
  }
}

struct FmtQ6K {
  static constexpr int kTile = kQ6KTileBytes;
  using Block = WBlock6;
  __device__ static Block load(const uint8_t* tile, int lane) { return load_wblock6(tile, lane); }
  __device__ static unsigned dep(const Block& b) { return wblock6_dep(b); }
  template <int T, bool SUMS>
  __device__ static void terms(const Block& wb, const ActSmem& m, int aslot, int astride, int nb, int b,
                               float* terms, int lane, int64_t row, int64_t n_rows, int32_t* isum_out,
                               int32_t* summs_out) {
    block_terms6<T, SUMS>(wb, m, aslot, astride, nb, b, terms, lane, row, n_rows, isum_out, summs_out);
  }
};

}  // namespace smeai
