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


}  // namespace smeai
