// attention.cu -- the per-head core of the reference's self-attention
// (sme_ai_self_attention_{ref,sme_packed}_f16f32, sme_ai_ops.c:1320-1499):
// scores, softmax and the weighted sum of V in one kernel, writing the fp16
// context that the output projection reads.
//
// One warp per (head, query row); a CTA holds up to 8 consecutive query rows
// of one head, so key / value rows staged in shared memory serve 8 queries.
// Numerics follow the reference step by step:
//   s_ij  = dot(Q_i, K_j) * scale   -- 16 fused-multiply-add lanes (d mod 16),
//           reduced pairwise (dot_f32_sve, :1268-1279, with svaddv's
//           implementation-defined order fixed as lane l + lane l+w, w=8..1)
//   e_ij  = expf(s_ij - max_j s_ij); sum_j e_ij summed sequentially, j
//           ascending (:893-973); p_ij = e_ij / sum (IEEE division)
//   ctx_i = sum_j V_j * p_ij, j ascending, multiply then add, two roundings
//           (attention_weighted_sum_f32, :1287-1318)
//   fp16(ctx_i) rounded to nearest even (convert_fp32_to_fp16, :175-179).
// Causal rows skip keys j > i: the reference gives them -1e30, whose
// exponential is exactly 0, so their terms add +-0 to sums that are never -0
// and leave every value unchanged.  Only expf differs from glibc's (by at most
// 2 ulp), so results agree with the CPU restatement to a few ulp.
#include <math.h>

#include "common.cuh"
#include "linear.h"

namespace smeai {

namespace {

constexpr int kMaxRows = 8;  // query rows (warps) per CTA
constexpr int kKeys = 32;    // key / value rows per shared-memory tile
constexpr int kSmemLimit = 227 * 1024;

// Shared memory: tile [kKeys][ldt] floats (K rows in the score pass, V rows
// in the sum pass; ldt = hd | 1 is odd, so lane l reading element d of row l
// hits bank (l * ldt + d) % 32, distinct over the warp), q [rows][hd],
// p [rows][S] (score / probability row of each warp).
size_t attn_smem_bytes(int rows, int64_t S, int hd) {
  return ((size_t)kKeys * (size_t)(hd | 1) + (size_t)rows * (size_t)hd + (size_t)rows * (size_t)S) * sizeof(float);
}

template <int E>  // E >= ceil(hd / 32): context elements per lane
__global__ void __launch_bounds__(kMaxRows * 32) attention_kernel(const float* __restrict__ Q,
                                                                  const float* __restrict__ K,
                                                                  const float* __restrict__ V, int64_t S, int64_t D,
                                                                  int hd, float scale, int causal,
                                                                  __half* __restrict__ ctx16) {
  extern __shared__ float smem[];
  const int rows = blockDim.x >> 5;
  const int ldt = hd | 1;
  float* tile = smem;
  float* qs = tile + kKeys * ldt;
  float* ps = qs + rows * hd;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t i0 = (int64_t)blockIdx.x * rows, i = i0 + w;
  const bool active = i < S;
  const int64_t off = (int64_t)blockIdx.y * hd;
  float* p = ps + (size_t)w * (size_t)S;
  float* q = qs + w * hd;
  // keys this CTA visits, and this warp's
  const int64_t i_last = (i0 + rows < S ? i0 + rows : S) - 1;
  const int64_t n_keys = causal ? i_last + 1 : S;
  const int64_t my_keys = !active ? 0 : causal ? i + 1 : S;

  pdl_trigger();
  pdl_wait();  // Q, K, V come from the projection kernels
  if (active)
    for (int d = lane; d < hd; d += 32) q[d] = Q[i * D + off + d];

  // ---- scores: lane l takes key j0 + l of each tile --------------------------
  float mx = -INFINITY;
  for (int64_t j0 = 0; j0 < n_keys; j0 += kKeys) {
    const int kt = (int)(n_keys - j0 < kKeys ? n_keys - j0 : kKeys);
    __syncthreads();  // the previous tile is consumed (and q is written)
    for (int e = threadIdx.x; e < kt * hd; e += blockDim.x) {
      const int r = e / hd, d = e - r * hd;
      tile[r * ldt + d] = K[(j0 + r) * D + off + d];
    }
    __syncthreads();
    const int64_t j = j0 + lane;
    if (j < my_keys) {
      const float* kr = tile + lane * ldt;
      float acc[16];
#pragma unroll
      for (int l = 0; l < 16; ++l) acc[l] = 0.f;
      int d0 = 0;
      for (; d0 + 16 <= hd; d0 += 16) {
#pragma unroll
        for (int l = 0; l < 16; ++l) acc[l] = __fmaf_rn(q[d0 + l], kr[d0 + l], acc[l]);
      }
#pragma unroll
      for (int l = 0; l < 16; ++l)
        if (d0 + l < hd) acc[l] = __fmaf_rn(q[d0 + l], kr[d0 + l], acc[l]);
#pragma unroll
      for (int wd = 8; wd >= 1; wd >>= 1) {
#pragma unroll
        for (int l = 0; l < wd; ++l) acc[l] = __fadd_rn(acc[l], acc[l + wd]);
      }
      const float s = __fmul_rn(acc[0], scale);
      p[j] = s;
      mx = fmaxf(mx, s);
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  __syncwarp();

  // ---- softmax: exponentials, the sequential sum, the division ---------------
  for (int64_t j = lane; j < my_keys; j += 32) p[j] = expf(__fsub_rn(p[j], mx));
  __syncwarp();
  float sum = 0.f;
  if (lane == 0) {
    int64_t j = 0;
    for (; j + 4 <= my_keys; j += 4) {
      const float a = p[j], b = p[j + 1], c = p[j + 2], e = p[j + 3];
      sum = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(sum, a), b), c), e);
    }
    for (; j < my_keys; ++j) sum = __fadd_rn(sum, p[j]);
  }
  sum = __shfl_sync(0xffffffffu, sum, 0);
  for (int64_t j = lane; j < my_keys; j += 32) p[j] = sum == 0.f ? 0.f : __fdiv_rn(p[j], sum);
  __syncwarp();

  // ---- context: lanes over d, keys in order ----------------------------------
  float acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.f;
  for (int64_t j0 = 0; j0 < n_keys; j0 += kKeys) {
    const int kt = (int)(n_keys - j0 < kKeys ? n_keys - j0 : kKeys);
    __syncthreads();
    for (int e = threadIdx.x; e < kt * hd; e += blockDim.x) {
      const int r = e / hd, d = e - r * hd;
      tile[r * ldt + d] = V[(j0 + r) * D + off + d];
    }
    __syncthreads();
    const int64_t left = my_keys - j0;
    const int jn = (int)(left < kt ? (left > 0 ? left : 0) : kt);
    for (int r = 0; r < jn; ++r) {
      const float pj = p[j0 + r];
      const float* vr = tile + r * ldt;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int d = lane + 32 * e;
        if (d < hd) acc[e] = __fadd_rn(acc[e], __fmul_rn(vr[d], pj));
      }
    }
  }
  if (active) {
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int d = lane + 32 * e;
      if (d < hd) ctx16[i * D + off + d] = __float2half_rn(acc[e]);
    }
  }
}

template <int E>
int launch_attention(const float* Q, const float* K, const float* V, int64_t S, int64_t D, int64_t heads, int hd,
                     float scale, int causal, __half* ctx16, cudaStream_t s) {
  int rows = kMaxRows;
  while (rows > 1 && attn_smem_bytes(rows, S, hd) > (size_t)kSmemLimit) --rows;
  const size_t smem = attn_smem_bytes(rows, S, hd);
  if (smem > (size_t)kSmemLimit) {
    set_last_error("self_attention: seq_len %lld with head_dim %d needs %zu bytes of shared memory (limit %d)",
                   (long long)S, hd, smem, kSmemLimit);
    return kUnsupported;
  }
  SMEAI_CUDA_TRY(cudaFuncSetAttribute(attention_kernel<E>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((unsigned)((S + rows - 1) / rows), (unsigned)heads);
  SMEAI_CUDA_TRY(launch(attention_kernel<E>, grid, dim3(rows * 32), smem, s, Q, K, V, S, D, hd, scale, causal, ctx16));
  return kOk;
}

}  // namespace

int attention_core(const float* Q, const float* K, const float* V, int64_t S, int64_t D, int64_t heads, int causal,
                   __half* ctx16, cudaStream_t s) {
  if (!Q || !K || !V || !ctx16 || S <= 0 || D <= 0 || heads <= 0 || D % heads) {
    set_last_error("self_attention: bad arguments");
    return kBadArgument;
  }
  if (S > 0x7fffffff || heads > 65535) {
    set_last_error("self_attention: seq_len %lld / heads %lld beyond the launch grid", (long long)S,
                   (long long)heads);
    return kUnsupported;
  }
  const int64_t hd64 = D / heads;
  if (hd64 > 512) {
    set_last_error("self_attention: head_dim %lld > 512 is not supported", (long long)hd64);
    return kUnsupported;
  }
  const int hd = (int)hd64;
  // 1 / sqrtf(hd), both IEEE-rounded on the host as in the reference (:1388)
  const float scale = 1.0f / sqrtf((float)hd);
  if (hd <= 32) return launch_attention<1>(Q, K, V, S, D, heads, hd, scale, causal, ctx16, s);
  if (hd <= 64) return launch_attention<2>(Q, K, V, S, D, heads, hd, scale, causal, ctx16, s);
  if (hd <= 128) return launch_attention<4>(Q, K, V, S, D, heads, hd, scale, causal, ctx16, s);
  if (hd <= 256) return launch_attention<8>(Q, K, V, S, D, heads, hd, scale, causal, ctx16, s);
  return launch_attention<16>(Q, K, V, S, D, heads, hd, scale, causal, ctx16, s);
}

}  // namespace smeai
