// q3k_core.cuh -- Q3_K weights for the persistent GEMV (q2k_gemv.cu): the
// device tile layout, the per-(32-row group, super-block) integer core and the
// float term, with the same ring / terms / ordered-sum machinery as Q2_K.
//
// ggml block_q3_K (110 bytes per 256 weights): hmask[32], qs[64], scales[12],
// d (fp16).  Weight i = d * (scale_j - 32) * q_i with q_i = u_i - 4,
// u_i = low 2 bits (the Q2_K plane order of qs) | high bit << 2, where the
// high bit of quant (half h, plane s, byte l) is bit 4h+s of hmask[l]
// (ggml dequantize_row_q3_K / gguf-py Q3_K.dequantize_blocks).
//
// Tile of one (group, super-block): 7 chunks of [32 rows][16 B] = 3584 bytes
//   chunks 0..3  qs bytes 16c..16c+15         (as the Q2_K tile)
//   chunks 4..5  hmask bytes 16(c-4)..+15
//   chunk  6     scales[12], d (fp16), 2 bytes of padding
#pragma once

#include "common.cuh"
#include "q2k_core.cuh"

namespace smeai {

constexpr int kQ3KBlockBytes = 110;
constexpr int kQ3KTileBytes = 32 * 112;

struct WBlock3 {
  uint4 q[4];
  uint4 hm[2];
  uint4 sd;
};

__device__ __forceinline__ WBlock3 load_wblock3(const uint8_t* tile, int lane) {
  const uint4* t4 = reinterpret_cast<const uint4*>(tile);
  WBlock3 wb;
#pragma unroll
  for (int c = 0; c < 4; ++c) wb.q[c] = t4[c * 32 + lane];
  wb.hm[0] = t4[4 * 32 + lane];
  wb.hm[1] = t4[5 * 32 + lane];
  wb.sd = t4[6 * 32 + lane];
  return wb;
}

__device__ __forceinline__ unsigned wblock3_dep(const WBlock3& wb) {
  unsigned d = wb.sd.x ^ wb.sd.y ^ wb.sd.z ^ wb.sd.w;
#pragma unroll
  for (int c = 0; c < 4; ++c) d ^= wb.q[c].x ^ wb.q[c].y ^ wb.q[c].z ^ wb.q[c].w;
#pragma unroll
  for (int c = 0; c < 2; ++c) d ^= wb.hm[c].x ^ wb.hm[c].y ^ wb.hm[c].z ^ wb.hm[c].w;
  return d;
}

// Two signed 16-bit lanes of a times signed bytes 0,1 (lo) or 2,3 (hi) of b.
__device__ __forceinline__ int dp2a_lo_ss(int a, unsigned b, int c) {
  int d;
  asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp2a_hi_ss(int a, unsigned b, int c) {
  int d;
  asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Byte k of w sign-extended to 32 bits (PTX prmt: a selector nibble with its
// top bit set replicates the sign bit of the byte it names).
__device__ __forceinline__ int sbyte(unsigned w, int k) {
  const unsigned sel = 0x8880u | ((unsigned)k * 0x1111u);
  int d;
  asm("prmt.b32 %0, %1, 0, %2;" : "=r"(d) : "r"(w), "r"(sel));
  return d;
}

// The 16 scales as signed bytes 4*(scale - 32), scale j in byte j%4 of word
// j/4.  ggml's unpacking (low 4 bits from the nibbles of bytes 0..7, top 2
// bits from bytes 8..11) gives 6-bit values v; (v ^ 32) << 2 is 4*(v - 32)
// as a signed byte (flipping bit 5 maps v to v - 32 mod 64, the shift puts
// that bit in the sign), with no carry between bytes.
__device__ __forceinline__ void q3k_scales4(const uint4& sd, unsigned (&s4)[4]) {
  const unsigned a0 = sd.x, a1 = sd.y, t = sd.z;
  const unsigned v0 = (a0 & 0x0F0F0F0Fu) | ((t & 0x03030303u) << 4);
  const unsigned v1 = (a1 & 0x0F0F0F0Fu) | (((t >> 2) & 0x03030303u) << 4);
  const unsigned v2 = ((a0 >> 4) & 0x0F0F0F0Fu) | (((t >> 4) & 0x03030303u) << 4);
  const unsigned v3 = ((a1 >> 4) & 0x0F0F0F0Fu) | (((t >> 6) & 0x03030303u) << 4);
  s4[0] = (v0 ^ 0x20202020u) << 2;
  s4[1] = (v1 ^ 0x20202020u) << 2;
  s4[2] = (v2 ^ 0x20202020u) << 2;
  s4[3] = (v3 ^ 0x20202020u) << 2;
}

// Integer core + float term of super-block b for this lane's row (T tokens):
//   S_j   = sum_{i in j} u_i * q8_i        (dp4a, u in [0, 7])
//   isum  = sum_j (scale_j - 32) * (S_j - 4 * bsums_j)
//         = (sum_j 4(scale_j-32) S_j) / 4 - sum_j 4(scale_j-32) bsums_j
// -- ggml's per-super-block integer total, exactly -- and the term
//   fp32(d) * d_x * isum     (summed over super-blocks in ascending order).
// SUMS: isum_out = isum, summs_out = sum_j (scale_j - 32) * bsums_j.
template <int T, bool SUMS>
__device__ __forceinline__ void block_terms3(const WBlock3& wb, const ActSmem& m, int aslot, int astride, int nb,
                                             int b, float* terms, int lane, int64_t row, int64_t n_rows,
                                             int32_t* isum_out, int32_t* summs_out) {
  unsigned s4[4];
  q3k_scales4(wb.sd, s4);
  int acc[T];
#pragma unroll
  for (int t = 0; t < T; ++t) acc[t] = 0;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int h = c >> 1, hf = c & 1;
    const unsigned q0 = wb.q[c].x, q1 = wb.q[c].y, q2 = wb.q[c].z, q3 = wb.q[c].w;
    const unsigned h0 = wb.hm[hf].x, h1 = wb.hm[hf].y, h2 = wb.hm[hf].z, h3 = wb.hm[hf].w;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const int hb = 4 * h + s;  // hmask bit of this plane
      const unsigned u0 = ((q0 >> (2 * s)) & 0x03030303u) | (((h0 >> hb) & 0x01010101u) << 2);
      const unsigned u1 = ((q1 >> (2 * s)) & 0x03030303u) | (((h1 >> hb) & 0x01010101u) << 2);
      const unsigned u2 = ((q2 >> (2 * s)) & 0x03030303u) | (((h2 >> hb) & 0x01010101u) << 2);
      const unsigned u3 = ((q3 >> (2 * s)) & 0x03030303u) | (((h3 >> hb) & 0x01010101u) << 2);
      const int j = 8 * h + 2 * s + hf;
      const int sc4 = sbyte(s4[j >> 2], j & 3);
      const int chunk = h * 8 + s * 2 + hf;
#pragma unroll
      for (int t = 0; t < T; ++t) {
        const int4 av = m.qs[(aslot + t * astride) * 16 + chunk];
        int sj = dp4a_us(u0, av.x, 0);
        sj = dp4a_us(u1, av.y, sj);
        sj = dp4a_us(u2, av.z, sj);
        sj = dp4a_us(u3, av.w, sj);
        acc[t] += sc4 * sj;
      }
    }
  }
  const float dw = __half2float(__ushort_as_half((unsigned short)(wb.sd.w & 0xffffu)));
#pragma unroll
  for (int t = 0; t < T; ++t) {
    const int* bsp = m.bs + (aslot + t * astride) * 8;
    const int4 bs0 = *reinterpret_cast<const int4*>(bsp);
    const int4 bs1 = *reinterpret_cast<const int4*>(bsp + 4);
    int mm = dp2a_lo_ss(bs0.x, s4[0], 0);
    mm = dp2a_hi_ss(bs0.y, s4[0], mm);
    mm = dp2a_lo_ss(bs0.z, s4[1], mm);
    mm = dp2a_hi_ss(bs0.w, s4[1], mm);
    mm = dp2a_lo_ss(bs1.x, s4[2], mm);
    mm = dp2a_hi_ss(bs1.y, s4[2], mm);
    mm = dp2a_lo_ss(bs1.z, s4[3], mm);
    mm = dp2a_hi_ss(bs1.w, s4[3], mm);
    const int isum = (acc[t] >> 2) - mm;  // acc[t] is a multiple of 4
    if constexpr (SUMS) {
      if (row < n_rows) {
        isum_out[row * nb + b] = isum;
        summs_out[row * nb + b] = mm >> 2;
      }
    } else {
      const float dd = __fmul_rn(dw, m.d[aslot + t * astride]);
      terms[(t * nb + b) * 32 + lane] = __fmul_rn(dd, __int2float_rn(isum));
    }
  }
}

// Weight formats of the persistent GEMV: tile size, per-lane block, core.
struct FmtQ2K {
  static constexpr int kTile = kTileBytes;
  using Block = WBlock;
  __device__ static Block load(const uint8_t* tile, int lane) { return load_wblock(tile, lane); }
  __device__ static unsigned dep(const Block& b) { return wblock_dep(b); }
  template <int T, bool SUMS>
  __device__ static void terms(const Block& wb, const ActSmem& m, int aslot, int astride, int nb, int b,
                               float* terms, int lane, int64_t row, int64_t n_rows, int32_t* isum_out,
                               int32_t* summs_out) {
    block_terms<T, SUMS>(wb, m, aslot, astride, nb, b, terms, lane, row, n_rows, isum_out, summs_out);
  }
};

struct FmtQ3K {
  static constexpr int kTile = kQ3KTileBytes;
  using Block = WBlock3;
  __device__ static Block load(const uint8_t* tile, int lane) { return load_wblock3(tile, lane); }
  __device__ static unsigned dep(const Block& b) { return wblock3_dep(b); }
  template <int T, bool SUMS>
  __device__ static void terms(const Block& wb, const ActSmem& m, int aslot, int astride, int nb, int b,
                               float* terms, int lane, int64_t row, int64_t n_rows, int32_t* isum_out,
                               int32_t* summs_out) {
    block_terms3<T, SUMS>(wb, m, aslot, astride, nb, b, terms, lane, row, n_rows, isum_out, summs_out);
  }
};

}  // namespace smeai
