// q2k_core.cuh -- the per-(32-row group, super-block) arithmetic shared by
// the Q2_K GEMV (q2k_gemv.cu) and the persistent decode program
// (q2k_program.cu): the tile of one super-block for 32 rows, the Q8_K
// activation planes in shared memory, and the exact integer core.
#pragma once

#include "common.cuh"
#include "q8k_device.cuh"

namespace smeai {

// One row's Q2_K super-block as a lane holds it: 64 bytes of 2-bit quants
// (4 chunks of 16), 16 scale/min bytes, d|dmin.
struct WBlock {
  uint4 q[4];
  uint4 s;
  unsigned dm;
};

// Read this lane's row from a 2688-byte tile (layout of q2k_repack_kernel).
__device__ __forceinline__ WBlock load_wblock(const uint8_t* tile, int lane) {
  const uint4* t4 = reinterpret_cast<const uint4*>(tile);
  WBlock wb;
  wb.q[0] = t4[0 * 32 + lane];
  wb.q[1] = t4[1 * 32 + lane];
  wb.q[2] = t4[2 * 32 + lane];
  wb.q[3] = t4[3 * 32 + lane];
  wb.s = t4[4 * 32 + lane];
  wb.dm = reinterpret_cast<const unsigned*>(tile + 5 * 512)[lane];
  return wb;
}

// A value that depends on every register of the block: arriving on the ring
// slot's barrier with it (mbar_arrive_warp) waits for the lane's loads.
__device__ __forceinline__ unsigned wblock_dep(const WBlock& wb) {
  unsigned d = wb.s.x ^ wb.s.y ^ wb.s.z ^ wb.s.w ^ wb.dm;
#pragma unroll
  for (int c = 0; c < 4; ++c) d ^= wb.q[c].x ^ wb.q[c].y ^ wb.q[c].z ^ wb.q[c].w;
  return d;
}

// Q8_K activation blocks in shared memory, slot = token * nb + block:
// qs 256 int8 (16-byte chunks), bsums as 8 int32 pairs, d.
struct ActSmem {
  int4* qs;
  int* bs;
  float* d;
};

// Stage one ggml block_q8_K (73 words: d, 64 words of qs, 8 words of bsums)
// from global memory into slot `slot`; one warp.
__device__ __forceinline__ void copy_q8k_smem(const uint32_t* blk, const ActSmem& m, int slot, int lane) {
  const uint32_t w0 = __ldcg(blk + lane), w1 = __ldcg(blk + lane + 32);
  const uint32_t w2 = lane + 64 < Q8K_BLOCK_WORDS ? __ldcg(blk + lane + 64) : 0u;
  uint32_t* q = reinterpret_cast<uint32_t*>(m.qs) + (size_t)slot * 64;
  if (lane == 0) m.d[slot] = __uint_as_float(w0);
  else q[lane - 1] = w0;
  q[lane + 31] = w1;
  if (lane + 64 < Q8K_BLOCK_WORDS) {
    if (lane == 0) q[63] = w2;
    else m.bs[slot * 8 + (lane - 1)] = (int)w2;
  }
}

__device__ __forceinline__ void store_q8k_smem(const Q8KLane& r, const ActSmem& m, int slot) {
  const int lane = threadIdx.x & 31;
  uint32_t* q = reinterpret_cast<uint32_t*>(m.qs) + (size_t)slot * 64;
  q[2 * lane] = r.w0;
  q[2 * lane + 1] = r.w1;
  if ((lane & 3) == 0) m.bs[slot * 8 + (lane >> 2)] = (int)r.bsum_pair;
  if (lane == 0) m.d[slot] = r.d;
}

// Integer core + float term of super-block b for this lane's row.
template <int T, bool SUMS>
// The activation of token t sits in slot aslot + t * astride; the term goes
// to terms[(t * nb + b) * 32 + lane].
__device__ __forceinline__ void block_terms(const WBlock& wb, const ActSmem& m, int aslot, int astride, int nb,
                                            int b, float* terms,
                                            int lane, int64_t row, int64_t n_rows, int32_t* isum_out,
                                            int32_t* summs_out) {
  const unsigned sl[4] = {wb.s.x & 0x0F0F0F0Fu, wb.s.y & 0x0F0F0F0Fu, wb.s.z & 0x0F0F0F0Fu, wb.s.w & 0x0F0F0F0Fu};
  const unsigned mh[4] = {(wb.s.x >> 4) & 0x0F0F0F0Fu, (wb.s.y >> 4) & 0x0F0F0F0Fu, (wb.s.z >> 4) & 0x0F0F0F0Fu,
                          (wb.s.w >> 4) & 0x0F0F0F0Fu};
  int plane[T][4];
#pragma unroll
  for (int t = 0; t < T; ++t)
#pragma unroll
    for (int s = 0; s < 4; ++s) plane[t][s] = 0;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const unsigned q0 = wb.q[c].x, q1 = wb.q[c].y, q2 = wb.q[c].z, q3 = wb.q[c].w;
    const int h = c >> 1, hf = c & 1;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const unsigned mask = 0x03030303u << (2 * s);
      const unsigned m0 = q0 & mask, m1 = q1 & mask, m2 = q2 & mask, m3 = q3 & mask;
      const int j = 8 * h + 2 * s + hf;  // sub-block of these 16 quants
      const int sc = (int)__byte_perm(sl[j >> 2], 0u, 0x4440u | (unsigned)(j & 3));
      const int chunk = h * 8 + s * 2 + hf;  // 16-byte activation chunk within the block
#pragma unroll
      for (int t = 0; t < T; ++t) {
        const int4 av = m.qs[(aslot + t * astride) * 16 + chunk];
        int acc = dp4a_us(m0, av.x, 0);
        acc = dp4a_us(m1, av.y, acc);
        acc = dp4a_us(m2, av.z, acc);
        acc = dp4a_us(m3, av.w, acc);
        plane[t][s] += sc * acc;
      }
    }
  }
  const float dw = __half2float(__ushort_as_half((unsigned short)(wb.dm & 0xffffu)));
  const float dmw = __half2float(__ushort_as_half((unsigned short)(wb.dm >> 16)));
#pragma unroll
  for (int t = 0; t < T; ++t) {
    const int isum = plane[t][0] + (plane[t][1] >> 2) + (plane[t][2] >> 4) + (plane[t][3] >> 6);
    const int* bsp = m.bs + (aslot + t * astride) * 8;
    const int4 bs0 = *reinterpret_cast<const int4*>(bsp);
    const int4 bs1 = *reinterpret_cast<const int4*>(bsp + 4);
    int mm = dp2a_lo_su(bs0.x, mh[0], 0);
    mm = dp2a_hi_su(bs0.y, mh[0], mm);
    mm = dp2a_lo_su(bs0.z, mh[1], mm);
    mm = dp2a_hi_su(bs0.w, mh[1], mm);
    mm = dp2a_lo_su(bs1.x, mh[2], mm);
    mm = dp2a_hi_su(bs1.y, mh[2], mm);
    mm = dp2a_lo_su(bs1.z, mh[3], mm);
    mm = dp2a_hi_su(bs1.w, mh[3], mm);
    if constexpr (SUMS) {
      if (row < n_rows) {
        isum_out[row * nb + b] = isum;
        summs_out[row * nb + b] = mm;
      }
    } else {
      const float dx = m.d[aslot + t * astride];
      const float dall = __fmul_rn(dx, dw);
      const float dmn = __fmul_rn(dx, dmw);
      terms[(t * nb + b) * 32 + lane] =
          __fmaf_rn(dall, __int2float_rn(isum), -__fmul_rn(dmn, __int2float_rn(mm)));
    }
  }
}

// ---- 8 tokens on the warp-level tensor core ---------------------------------
// One 32-row x 256-weight tile for 8 tokens as 16 mma.sync.m16n8k32 (u8 x s8
// -> s32): N = the 8 tokens, M = 16 weight rows, K = 32 weights.  K block
// (n, s) holds weights n*128 + s*32 + k (k < 32): qs bytes n*32 + k, plane s,
// and activations n*128 + s*32 + k.  A = scale * q (at most 45, so the four
// byte products of one 32-bit multiply never carry); the sub-block of k is
// n*8 + 2s + (k >= 16), so one fragment register never straddles two scales.
// The s32 sums are the integers of the dp4a core (and of ggml's dot), and the
// min term and the float combine are block_terms', so the terms are the same
// bits.  Fragment layout (m16n8k32, 8-bit): lane = 4 * g + t; a0/a2 rows g,
// a1/a3 rows g + 8; a0/a1 k = 4t..4t+3, a2/a3 k = 16 + 4t..; b0 k = 4t.., b1
// k = 16 + 4t.., column n = g; c0/c1 row g, columns 2t, 2t+1; c2/c3 row g + 8.
__device__ __forceinline__ void mma_u8s8_16832(int (&c)[4], unsigned a0, unsigned a1, unsigned a2, unsigned a3,
                                               unsigned b0, unsigned b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The activation fragments of one block for the 8 tokens (token t in slot
// aslot + t * astride): b[kb][0..1] for K block kb = 4n + s.
struct Act8Frag {
  unsigned b[8][2];
};
__device__ __forceinline__ void load_act8_frag(const ActSmem& m, int aslot, int astride, int lane, Act8Frag& f) {
  const int g = lane >> 2, t = lane & 3;
  const unsigned* q = reinterpret_cast<const unsigned*>(m.qs) + (size_t)(aslot + g * astride) * 64;
#pragma unroll
  for (int n = 0; n < 2; ++n)
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      f.b[4 * n + s][0] = q[n * 32 + s * 8 + t];
      f.b[4 * n + s][1] = q[n * 32 + s * 8 + 4 + t];
    }
}

// Terms of super-block b for the tile's 32 rows and 8 tokens:
// terms[(tok * nb + b) * 32 + row], the layout block_terms<8> writes.
__device__ __forceinline__ void block_terms_mma8(const uint8_t* tile, const Act8Frag& f, const ActSmem& m,
                                                 int aslot, int astride, int nb, int b, float* terms, int lane) {
  const int g = lane >> 2, t = lane & 3;
  // the min term's activation side for tokens 2t and 2t + 1: bsums pairs and d
  int4 bsa[2][2];
  float dx[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int sl = aslot + (2 * t + j) * astride;
    bsa[j][0] = *reinterpret_cast<const int4*>(m.bs + sl * 8);
    bsa[j][1] = *reinterpret_cast<const int4*>(m.bs + sl * 8 + 4);
    dx[j] = m.d[sl];
  }
  const unsigned* qs = reinterpret_cast<const unsigned*>(tile);
#pragma unroll
  for (int mb = 0; mb < 2; ++mb) {
    const int r0 = 16 * mb + g, r1 = r0 + 8;
    const uint4 s0 = reinterpret_cast<const uint4*>(tile + 2048)[r0];
    const uint4 s1 = reinterpret_cast<const uint4*>(tile + 2048)[r1];
    const unsigned sw0[4] = {s0.x, s0.y, s0.z, s0.w}, sw1[4] = {s1.x, s1.y, s1.z, s1.w};
    int acc[4] = {0, 0, 0, 0};
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      // qs word t of rows r0 / r1 in chunks 2n (k < 16) and 2n + 1 (k >= 16)
      const unsigned w0 = qs[(2 * n) * 128 + r0 * 4 + t], w1 = qs[(2 * n) * 128 + r1 * 4 + t];
      const unsigned w2 = qs[(2 * n + 1) * 128 + r0 * 4 + t], w3 = qs[(2 * n + 1) * 128 + r1 * 4 + t];
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const int sw = 2 * n + (s >> 1), sh = 16 * (s & 1);   // sub-block n*8 + 2s: word sw, byte (2s) & 3
        const unsigned c00 = (sw0[sw] >> sh) & 0xFu, c01 = (sw0[sw] >> (sh + 8)) & 0xFu;
        const unsigned c10 = (sw1[sw] >> sh) & 0xFu, c11 = (sw1[sw] >> (sh + 8)) & 0xFu;
        const unsigned mask = 0x03030303u;
        mma_u8s8_16832(acc, ((w0 >> (2 * s)) & mask) * c00, ((w1 >> (2 * s)) & mask) * c10,
                       ((w2 >> (2 * s)) & mask) * c01, ((w3 >> (2 * s)) & mask) * c11, f.b[4 * n + s][0],
                       f.b[4 * n + s][1]);
      }
    }
    // min term and combine for rows r0, r1 x tokens 2t, 2t + 1
    const unsigned* dmp = reinterpret_cast<const unsigned*>(tile + 2560);
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const unsigned* sw = rr ? sw1 : sw0;
      const unsigned mh0 = (sw[0] >> 4) & 0x0F0F0F0Fu, mh1 = (sw[1] >> 4) & 0x0F0F0F0Fu;
      const unsigned mh2 = (sw[2] >> 4) & 0x0F0F0F0Fu, mh3 = (sw[3] >> 4) & 0x0F0F0F0Fu;
      const int row = rr ? r1 : r0;
      const unsigned dm = dmp[row];
      const float dw = __half2float(__ushort_as_half((unsigned short)(dm & 0xffffu)));
      const float dmw = __half2float(__ushort_as_half((unsigned short)(dm >> 16)));
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int4 bs0 = bsa[j][0], bs1 = bsa[j][1];
        int mm = dp2a_lo_su(bs0.x, mh0, 0);
        mm = dp2a_hi_su(bs0.y, mh0, mm);
        mm = dp2a_lo_su(bs0.z, mh1, mm);
        mm = dp2a_hi_su(bs0.w, mh1, mm);
        mm = dp2a_lo_su(bs1.x, mh2, mm);
        mm = dp2a_hi_su(bs1.y, mh2, mm);
        mm = dp2a_lo_su(bs1.z, mh3, mm);
        mm = dp2a_hi_su(bs1.w, mh3, mm);
        const int isum = acc[2 * rr + j];
        const float dall = __fmul_rn(dx[j], dw);
        const float dmn = __fmul_rn(dx[j], dmw);
        terms[((2 * t + j) * nb + b) * 32 + row] =
            __fmaf_rn(dall, __int2float_rn(isum), -__fmul_rn(dmn, __int2float_rn(mm)));
      }
    }
  }
}

}  // namespace smeai
