// q8k_device.cuh -- warp-level Q8_K quantization core shared by the standalone
// quantizer (q8k_quant.cu) and the GEMV prologue (q2k_gemv.cu), so both
// produce identical blocks.
//
// Restates ggml's quantize_row_q8_K (generic C, ggml 0.9.8): per 256 values,
// the value of largest magnitude (first on ties) gives iscale = -127/max;
// q = nearest(iscale*x) capped at 127 (ggml's nearest_int as one fused
// multiply-add with 1.5*2^23, the form GCC's default contraction produces on
// an FMA target); d = 1/iscale; bsums = sums of 16 consecutive q.  An
// all-zero block gives d = 0 and zero quants and sums.
#pragma once

#include "common.cuh"

namespace smeai {

// What one lane contributes to its block: qs bytes 8l..8l+7 as two words;
// on lanes with l % 4 == 0, the bsums pair (2*(l/4), 2*(l/4)+1) as one word;
// d (same on every lane).
struct Q8KLane {
  uint32_t w0, w1;
  uint32_t bsum_pair;
  float d;
};

// RMSNorm sum of squares, in the fixed order of the CPU restatement:
//   1. per 32-value group: the squares (each rounded) folded pairwise at
//      distances 16, 8, 4, 2, 1;
//   2. the group sums: lane l adds groups l, l+32, l+64, ... in ascending
//      order from 0, then the lanes are folded at distances 16, 8, 4, 2, 1.
// Group sum from the load8 layout (8 consecutive values per lane; lanes
// 4q..4q+3 hold group q of the 256-value block): distances 16 and 8 are
// lanes xor 2 and xor 1, distances 4, 2, 1 are within the lane.  All four
// lanes of the group return the sum.
__device__ __forceinline__ float group_sumsq_load8(const float (&v)[8]) {
  float a[8];
#pragma unroll
  for (int b = 0; b < 8; ++b) a[b] = __fmul_rn(v[b], v[b]);
#pragma unroll
  for (int b = 0; b < 8; ++b) a[b] = __fadd_rn(a[b], __shfl_xor_sync(0xffffffffu, a[b], 2));
#pragma unroll
  for (int b = 0; b < 8; ++b) a[b] = __fadd_rn(a[b], __shfl_xor_sync(0xffffffffu, a[b], 1));
#pragma unroll
  for (int b = 0; b < 4; ++b) a[b] = __fadd_rn(a[b], a[b + 4]);
  a[0] = __fadd_rn(a[0], a[2]);
  a[1] = __fadd_rn(a[1], a[3]);
  return __fadd_rn(a[0], a[1]);
}
// Group sum with one value per lane (lane i holds value i of the group); all
// lanes return it.
__device__ __forceinline__ float group_sumsq_lane(float v) {
  float a = __fmul_rn(v, v);
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, off));
  return a;
}
// Step 2 over G group sums at p (shared or global memory); all lanes return
// the total.
// The same over group sums other CTAs of the running grid wrote (read
// through L2; each lane's loads go out together).
__device__ __forceinline__ float rms_fold_groups_cg(const float* p, int G) {
  const int lane = threadIdx.x & 31;
  float acc = 0.f;
  for (int g0 = 0; g0 < G; g0 += 32 * 8) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int g = g0 + lane + 32 * j;
      v[j] = g < G ? __ldcg(p + g) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (g0 + lane + 32 * j < G) acc = __fadd_rn(acc, v[j]);
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
  return acc;
}
__device__ __forceinline__ float rms_fold_groups(const float* p, int G) {
  const int lane = threadIdx.x & 31;
  float acc = 0.f;
  for (int g = lane; g < G; g += 32) acc = __fadd_rn(acc, p[g]);
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
  return acc;
}

// inv = 1/sqrt(sum/k + eps), each step rounded once.
__device__ __forceinline__ float rms_inv_from_sum(float total, int k, float eps) {
  const float mean = __fdiv_rn(total, (float)k);
  return __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(mean, eps)));
}

// The block's value of largest magnitude, the first one on ties (ggml scans
// the block in order with a strict '>'), NaNs never chosen: two warp
// reductions on the magnitudes' bit patterns (which order like the values
// for non-negative floats) and one shuffle of the winner's signed value.
__device__ __forceinline__ Q8KLane q8k_quantize_lane(const float (&v)[8]) {
  const int lane = threadIdx.x & 31;
  unsigned mag[8], m = 0u;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    mag[i] = __float_as_uint(v[i]) & 0x7fffffffu;
    if (mag[i] <= 0x7f800000u && mag[i] > m) m = mag[i];   // NaN (> 0x7f800000) skipped
  }
  const unsigned abits = __reduce_max_sync(0xffffffffu, m);
  unsigned first = 0xffffffffu;
#pragma unroll
  for (int i = 7; i >= 0; --i)
    if (mag[i] == abits) first = (unsigned)(lane * 8 + i);
  const unsigned idx = __reduce_min_sync(0xffffffffu, first);
  float mine = v[0];
#pragma unroll
  for (int i = 1; i < 8; ++i)
    if ((int)(idx & 7u) == i) mine = v[i];
  const float vmax = __shfl_sync(0xffffffffu, mine, (int)(idx >> 3) & 31);
  const float amax = __uint_as_float(abits);
  Q8KLane r;
  if (amax == 0.f) {
    r.w0 = r.w1 = r.bsum_pair = 0u;
    r.d = 0.f;
    return r;
  }
  const float iscale = __fdiv_rn(-127.f, vmax);
  int part = 0;
  uint32_t w[2] = {0u, 0u};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int q = magic_round_bits(__fmaf_rn(iscale, v[i], kMagic));
    q = q > 127 ? 127 : q;
    part += q;
    w[i >> 2] |= (uint32_t)(q & 0xff) << (8 * (i & 3));
  }
  r.w0 = w[0];
  r.w1 = w[1];
  const int gsum = part + __shfl_xor_sync(0xffffffffu, part, 1);      // group l/2
  const int other = __shfl_down_sync(0xffffffffu, gsum, 2);          // group l/2 + 1
  r.bsum_pair = (uint32_t)(gsum & 0xffff) | ((uint32_t)other << 16);
  r.d = __fdiv_rn(1.f, iscale);
  return r;
}

// Write one lane's share as a ggml block_q8_K (292 bytes, 4-byte aligned).
__device__ __forceinline__ void q8k_store_global(const Q8KLane& r, uint8_t* out) {
  const int lane = threadIdx.x & 31;
  uint32_t* ow = reinterpret_cast<uint32_t*>(out);
  ow[1 + 2 * lane] = r.w0;
  ow[2 + 2 * lane] = r.w1;
  if ((lane & 3) == 0) ow[65 + (lane >> 2)] = r.bsum_pair;
  if (lane == 0) ow[0] = __float_as_uint(r.d);
}

__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = p[i];
  }
}

// load8 through L2 only (ld.global.cg): for data other CTAs of the running
// grid wrote, which this SM's L1 may hold stale.
__device__ __forceinline__ void load8_cg(const float* p, float (&v)[8]) {
  if ((reinterpret_cast<uintptr_t>(p) & 15) == 0) {
    const float4 a = __ldcg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldcg(reinterpret_cast<const float4*>(p + 4));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __ldcg(p + i);
  }
}

}  // namespace smeai
