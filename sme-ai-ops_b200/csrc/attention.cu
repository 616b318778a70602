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
// Two implementations compute these same values:
//   tiled (head_dim 32, 64 or 128, 256 <= S <= 16384): three kernels per chunk
//     of heads -- attn_scores_kernel (64 x 64 score tiles, 4 x 4 per thread,
//     the 16 dot-product lanes evaluated in the order of their pairwise tree,
//     so only four partial sums per score are live), attn_softmax_kernel (one
//     warp per score row, held in registers up to 2048 keys) and attn_pv_kernel (64 query rows x head_dim per
//     CTA, keys in order) -- through a score buffer of heads x S x S floats;
//   fused (everything else): attention_kernel, one warp per query row.
// Causal rows skip keys j > i: the reference gives them -1e30, whose
// exponential is exactly 0, so their terms add +-0 to sums that are never -0
// and leave every value unchanged.  Only expf differs from glibc's (by at most
// 2 ulp), so results agree with the CPU restatement to a few ulp.
#include <math.h>
#include <stdlib.h>

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

// ---- tiled path ----------------------------------------------------------------------
constexpr int kTQ = 64;                         // query / key rows per score tile
constexpr int kTJ = 32;                         // keys per weighted-sum step
constexpr size_t kScoreBudget = 1ull << 30;     // score buffer per chunk of heads

// The budget, overridable with SMEAI_ATTN_SCORE_BUDGET (bytes; tests use a
// small one to run several chunks of heads).
size_t score_budget() {
  const char* e = getenv("SMEAI_ATTN_SCORE_BUDGET");
  if (e && *e) {
    const long long v = atoll(e);
    if (v > 0) return (size_t)v;
  }
  return kScoreBudget;
}

__host__ __device__ constexpr int bitrev4(int s) {
  return ((s & 1) << 3) | ((s & 2) << 1) | ((s & 4) >> 1) | ((s & 8) >> 3);
}

// Tile pair t of a head: all (ib, jb) pairs, or jb <= ib when causal.
__device__ __forceinline__ void tile_pair(int t, int tiles, int causal, int& ib, int& jb) {
  if (!causal) {
    ib = t / tiles;
    jb = t - ib * tiles;
    return;
  }
  int r = (int)((sqrtf(8.f * (float)t + 1.f) - 1.f) * 0.5f);
  while ((r + 1) * (r + 2) / 2 <= t) ++r;
  while (r * (r + 1) / 2 > t) --r;
  ib = r;
  jb = t - r * (r + 1) / 2;
}

// sc[hh][i][j] = dot(Q_i, K_j) * scale for the 64 x 64 tile pair of blockIdx.x,
// head h0 + blockIdx.y.  Shared memory: Qt [hd][64], Kt [hd][64] (transposed,
// so a thread's 4 rows / 4 keys are one float4).  The dot of each (i, j)
// follows the reference order: lane l (l = 0..15) accumulates d = l, l+16, ..
// with fused multiply-adds, and the lanes are summed pairwise (l + l+8, then
// +4, +2, +1).  Lanes are evaluated in bit-reversed order (0, 8, 4, 12, ..),
// the post-order of that tree, so each pair is added as soon as both exist.
template <int HD>
__global__ void __launch_bounds__(256, 2) attn_scores_kernel(const float* __restrict__ Q,
                                                             const float* __restrict__ K, int64_t S, int64_t D,
                                                             int h0, float scale, int causal, int tiles,
                                                             float* __restrict__ sc, int64_t ldsc) {
  constexpr int hd = HD;
  extern __shared__ __align__(16) float smem[];
  float* Qt = smem;
  float* Kt = smem + hd * kTQ;
  int ib, jb;
  tile_pair((int)blockIdx.x, tiles, causal, ib, jb);
  const int64_t i0 = (int64_t)ib * kTQ, j0 = (int64_t)jb * kTQ;
  const int64_t off = (int64_t)(h0 + (int)blockIdx.y) * hd;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;

  pdl_trigger();
  pdl_wait();
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  // all of the thread's tile loads in flight at once, then the transposed stores
  constexpr int kIt = kTQ * hd / 4 / 256;
  float4 qv[kIt], kv[kIt];
#pragma unroll
  for (int it = 0; it < kIt; ++it) {
    const int e = tid + 256 * it, r = e % kTQ, c = (e / kTQ) * 4;
    qv[it] = i0 + r < S ? *reinterpret_cast<const float4*>(Q + (i0 + r) * D + off + c) : z4;
    kv[it] = j0 + r < S ? *reinterpret_cast<const float4*>(K + (j0 + r) * D + off + c) : z4;
  }
#pragma unroll
  for (int it = 0; it < kIt; ++it) {
    const int e = tid + 256 * it, r = e % kTQ, c = (e / kTQ) * 4;
    Qt[(c + 0) * kTQ + r] = qv[it].x;
    Qt[(c + 1) * kTQ + r] = qv[it].y;
    Qt[(c + 2) * kTQ + r] = qv[it].z;
    Qt[(c + 3) * kTQ + r] = qv[it].w;
    Kt[(c + 0) * kTQ + r] = kv[it].x;
    Kt[(c + 1) * kTQ + r] = kv[it].y;
    Kt[(c + 2) * kTQ + r] = kv[it].z;
    Kt[(c + 3) * kTQ + r] = kv[it].w;
  }
  __syncthreads();

  float p0[4][4], p1[4][4], p2[4][4], p3[4][4];  // pending sums of tree levels 0..3
#pragma unroll
  for (int s = 0; s < 16; ++s) {
    const int l = bitrev4(s);
    float a[4][4];
#pragma unroll
    for (int ii = 0; ii < 4; ++ii)
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) a[ii][jj] = 0.f;
#pragma unroll
    for (int d = l; d < hd; d += 16) {
      const float4 q4 = *reinterpret_cast<const float4*>(Qt + d * kTQ + ty * 4);
      const float4 k4 = *reinterpret_cast<const float4*>(Kt + d * kTQ + tx * 4);
      const float qv[4] = {q4.x, q4.y, q4.z, q4.w}, kv[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
      for (int ii = 0; ii < 4; ++ii)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) a[ii][jj] = __fmaf_rn(qv[ii], kv[jj], a[ii][jj]);
    }
#pragma unroll
    for (int ii = 0; ii < 4; ++ii)
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        float v = a[ii][jj];
        if ((s & 1) == 0) { p0[ii][jj] = v; continue; }
        v = __fadd_rn(p0[ii][jj], v);                 // lane l + lane l+8
        if ((s & 2) == 0) { p1[ii][jj] = v; continue; }
        v = __fadd_rn(p1[ii][jj], v);                 // + the pair 4 lanes on
        if ((s & 4) == 0) { p2[ii][jj] = v; continue; }
        v = __fadd_rn(p2[ii][jj], v);                 // + the quad 2 lanes on
        if ((s & 8) == 0) { p3[ii][jj] = v; continue; }
        p3[ii][jj] = __fadd_rn(p3[ii][jj], v);        // the total
      }
  }
  float* out = sc + (int64_t)blockIdx.y * S * ldsc;
#pragma unroll
  for (int ii = 0; ii < 4; ++ii) {
    const int64_t i = i0 + ty * 4 + ii;
    if (i >= S) continue;
    *reinterpret_cast<float4*>(out + i * ldsc + j0 + tx * 4) =
        make_float4(__fmul_rn(p3[ii][0], scale), __fmul_rn(p3[ii][1], scale), __fmul_rn(p3[ii][2], scale),
                    __fmul_rn(p3[ii][3], scale));
  }
}

// Softmax of score rows in place, one warp per row (head blockIdx.y; CTAs
// take row blocks from the last one down): max, expf(s - max), the sequential sum (lane 0,
// j ascending), e / sum; causal rows then zero their entries up to the end
// of the diagonal 64-key tile, which the weighted-sum kernel reads.
template <int R>  // R > 0: the row held in registers, R values per lane (S <= 32 R); 0: staged only
__global__ void __launch_bounds__(256) attn_softmax_kernel(float* __restrict__ sc, int64_t S, int64_t ldsc,
                                                           int causal) {
  extern __shared__ __align__(16) float smem[];
  const int warps = blockDim.x >> 5, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t i = (int64_t)(gridDim.x - 1 - blockIdx.x) * warps + w;  // longest causal rows first
  float* e = smem + (size_t)w * (size_t)ldsc;
  pdl_trigger();
  pdl_wait();
  if (i >= S) return;
  float* row = sc + ((int64_t)blockIdx.y * S + i) * ldsc;
  const int64_t n = causal ? i + 1 : S;
  float mx = -INFINITY;
  float v[R > 0 ? R : 1];
  if constexpr (R > 0) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t j = lane + 32 * r;
      v[r] = j < n ? row[j] : -INFINITY;
      mx = fmaxf(mx, v[r]);
    }
  } else {
    for (int64_t j = lane; j < n; j += 32) {
      const float x = row[j];
      e[j] = x;
      mx = fmaxf(mx, x);
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if constexpr (R > 0) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t j = lane + 32 * r;
      if (j < n) {
        v[r] = expf(__fsub_rn(v[r], mx));
        e[j] = v[r];
      }
    }
  } else {
    for (int64_t j = lane; j < n; j += 32) e[j] = expf(__fsub_rn(e[j], mx));
  }
  __syncwarp();
  float sum = 0.f;
  if (lane == 0) {  // in key order, four at a time from shared memory
    int64_t j = 0;
    for (; j + 4 <= n; j += 4) {
      const float4 q = *reinterpret_cast<const float4*>(e + j);
      sum = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(sum, q.x), q.y), q.z), q.w);
    }
    for (; j < n; ++j) sum = __fadd_rn(sum, e[j]);
  }
  sum = __shfl_sync(0xffffffffu, sum, 0);
  if constexpr (R > 0) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t j = lane + 32 * r;
      if (j < n) row[j] = sum == 0.f ? 0.f : __fdiv_rn(v[r], sum);
    }
  } else {
    for (int64_t j = lane; j < n; j += 32) row[j] = sum == 0.f ? 0.f : __fdiv_rn(e[j], sum);
  }
  if (causal) {
    const int64_t tile_end = (i / kTQ + 1) * kTQ;
    const int64_t jend = tile_end < S ? tile_end : S;
    for (int64_t j = n + lane; j < jend; j += 32) row[j] = 0.f;
  }
}

// ctx16[i][off + d] = fp16(sum_j p_ij * V_j[d]) for 64 query rows (query
// tiles from the last one down) of head h0 + blockIdx.y; keys in ascending order, 32 per
// step, each term a multiply then an add (two roundings).  256 threads as
// 16 x 16: rows ty*4 .. ty*4+3, columns tx*CW/2 + .. and HD/2 + tx*CW/2 + ..
// (CW = HD/16 columns per thread).  Shared memory: Pt [32][64] (P transposed),
// Vs [32][HD].
template <int HD>
__global__ void __launch_bounds__(256) attn_pv_kernel(const float* __restrict__ sc, int64_t ldsc,
                                                      const float* __restrict__ V, int64_t S, int64_t D, int h0,
                                                      int causal, __half* __restrict__ ctx16) {
  constexpr int CW = HD / 16, HW = CW / 2;
  __shared__ __align__(16) float Pt[kTJ][kTQ];
  __shared__ __align__(16) float Vs[kTJ][HD];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  // last query tile first: causal tiles' work grows with the tile index
  const int64_t i0 = (int64_t)(gridDim.x - 1 - blockIdx.x) * kTQ;
  const int64_t off = (int64_t)(h0 + (int)blockIdx.y) * HD;
  const float* P = sc + (int64_t)blockIdx.y * S * ldsc;
  const int64_t jmax = causal ? (i0 + kTQ < S ? i0 + kTQ : S) : S;
  float acc[4][CW];
#pragma unroll
  for (int ii = 0; ii < 4; ++ii)
#pragma unroll
    for (int c = 0; c < CW; ++c) acc[ii][c] = 0.f;
  pdl_trigger();
  pdl_wait();
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  // the next step's P and V are fetched into registers while the current
  // step's products run, then stored over the shared tiles
  constexpr int kPIt = kTQ * kTJ / 4 / 256, kVIt = kTJ * HD / 4 / 256;
  float4 pr[kPIt], vr[kVIt];
  auto fetch = [&](int64_t j0) {
#pragma unroll
    for (int it = 0; it < kPIt; ++it) {  // P rows i0 + r, keys j0 + c .. c+3
      const int e = tid + 256 * it, r = e % kTQ, c = (e / kTQ) * 4;
      pr[it] = (i0 + r < S && j0 + c < jmax) ? *reinterpret_cast<const float4*>(P + (i0 + r) * ldsc + j0 + c) : z4;
    }
#pragma unroll
    for (int it = 0; it < kVIt; ++it) {
      const int e = tid + 256 * it, r = e / (HD / 4), c = (e % (HD / 4)) * 4;
      vr[it] = j0 + r < jmax ? *reinterpret_cast<const float4*>(V + (j0 + r) * D + off + c) : z4;
    }
  };
  auto stash = [&]() {
#pragma unroll
    for (int it = 0; it < kPIt; ++it) {
      const int e = tid + 256 * it, r = e % kTQ, c = (e / kTQ) * 4;
      Pt[c + 0][r] = pr[it].x;
      Pt[c + 1][r] = pr[it].y;
      Pt[c + 2][r] = pr[it].z;
      Pt[c + 3][r] = pr[it].w;
    }
#pragma unroll
    for (int it = 0; it < kVIt; ++it) {
      const int e = tid + 256 * it, r = e / (HD / 4), c = (e % (HD / 4)) * 4;
      *reinterpret_cast<float4*>(&Vs[r][c]) = vr[it];
    }
  };
  fetch(0);
  for (int64_t j0 = 0; j0 < jmax; j0 += kTJ) {
    __syncthreads();  // the previous step's products are done with the tiles
    stash();
    __syncthreads();
    if (j0 + kTJ < jmax) fetch(j0 + kTJ);
#pragma unroll 4
    for (int jj = 0; jj < kTJ; ++jj) {
      const float4 p4 = *reinterpret_cast<const float4*>(&Pt[jj][ty * 4]);
      const float pv[4] = {p4.x, p4.y, p4.z, p4.w};
      float vv[CW];
      if constexpr (HW == 4) {
        const float4 v0 = *reinterpret_cast<const float4*>(&Vs[jj][tx * 4]);
        const float4 v1 = *reinterpret_cast<const float4*>(&Vs[jj][HD / 2 + tx * 4]);
        vv[0] = v0.x; vv[1] = v0.y; vv[2] = v0.z; vv[3] = v0.w;
        vv[4] = v1.x; vv[5] = v1.y; vv[6] = v1.z; vv[7] = v1.w;
      } else if constexpr (HW == 2) {
        const float2 v0 = *reinterpret_cast<const float2*>(&Vs[jj][tx * 2]);
        const float2 v1 = *reinterpret_cast<const float2*>(&Vs[jj][HD / 2 + tx * 2]);
        vv[0] = v0.x; vv[1] = v0.y; vv[2] = v1.x; vv[3] = v1.y;
      } else {
        vv[0] = Vs[jj][tx];
        vv[1] = Vs[jj][HD / 2 + tx];
      }
#pragma unroll
      for (int ii = 0; ii < 4; ++ii)
#pragma unroll
        for (int c = 0; c < CW; ++c) acc[ii][c] = __fadd_rn(acc[ii][c], __fmul_rn(vv[c], pv[ii]));
    }
  }
#pragma unroll
  for (int ii = 0; ii < 4; ++ii) {
    const int64_t i = i0 + ty * 4 + ii;
    if (i >= S) continue;
#pragma unroll
    for (int c = 0; c < CW; ++c) {
      const int d = c < HW ? tx * HW + c : HD / 2 + tx * HW + c - HW;
      ctx16[i * D + off + d] = __float2half_rn(acc[ii][c]);
    }
  }
}

bool tiled_ok(int64_t S, int hd) { return (hd == 32 || hd == 64 || hd == 128) && S >= 256 && S <= 16384; }

int64_t score_ld(int64_t S) { return (S + kTQ - 1) / kTQ * kTQ; }

int64_t heads_per_chunk(int64_t S, int64_t heads) {
  const size_t per = (size_t)S * (size_t)score_ld(S) * sizeof(float);
  int64_t hc = (int64_t)(score_budget() / per);
  if (hc < 1) hc = 1;
  return hc < heads ? hc : heads;
}

int attention_tiled(const float* Q, const float* K, const float* V, int64_t S, int64_t D, int64_t heads, int hd,
                    float scale, int causal, __half* ctx16, float* scores, cudaStream_t s) {
  const int64_t ldsc = score_ld(S), hc_max = heads_per_chunk(S, heads);
  const int tiles = (int)(ldsc / kTQ);
  const int64_t pairs = causal ? (int64_t)tiles * (tiles + 1) / 2 : (int64_t)tiles * tiles;
  const size_t sc_smem = (size_t)2 * hd * kTQ * sizeof(float);
  int warps = 8;
  while (warps > 1 && (size_t)warps * ldsc * sizeof(float) > (size_t)kSmemLimit) --warps;
  const size_t sm_smem = (size_t)warps * ldsc * sizeof(float);
  auto scores_k = hd == 32 ? attn_scores_kernel<32> : hd == 64 ? attn_scores_kernel<64> : attn_scores_kernel<128>;
  SMEAI_CUDA_TRY(cudaFuncSetAttribute(scores_k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sc_smem));
  auto softmax_k = S <= 512    ? attn_softmax_kernel<16>
                   : S <= 1024 ? attn_softmax_kernel<32>
                   : S <= 2048 ? attn_softmax_kernel<64>
                               : attn_softmax_kernel<0>;
  SMEAI_CUDA_TRY(cudaFuncSetAttribute(softmax_k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm_smem));
  for (int64_t h0 = 0; h0 < heads; h0 += hc_max) {
    const int64_t hc = heads - h0 < hc_max ? heads - h0 : hc_max;
    SMEAI_CUDA_TRY(launch(scores_k, dim3((unsigned)pairs, (unsigned)hc), dim3(256), sc_smem, s, Q, K, S, D, (int)h0,
                          scale, causal, tiles, scores, ldsc));
    SMEAI_CUDA_TRY(launch(softmax_k, dim3((unsigned)((S + warps - 1) / warps), (unsigned)hc),
                          dim3(warps * 32), sm_smem, s, scores, S, ldsc, causal));
    const dim3 pv_grid((unsigned)((S + kTQ - 1) / kTQ), (unsigned)hc);
    if (hd == 32)
      SMEAI_CUDA_TRY(launch(attn_pv_kernel<32>, pv_grid, dim3(256), 0, s, (const float*)scores, ldsc, V, S, D, (int)h0,
                            causal, ctx16));
    else if (hd == 64)
      SMEAI_CUDA_TRY(launch(attn_pv_kernel<64>, pv_grid, dim3(256), 0, s, (const float*)scores, ldsc, V, S, D, (int)h0,
                            causal, ctx16));
    else
      SMEAI_CUDA_TRY(launch(attn_pv_kernel<128>, pv_grid, dim3(256), 0, s, (const float*)scores, ldsc, V, S, D,
                            (int)h0, causal, ctx16));
  }
  return kOk;
}

}  // namespace

size_t attention_scratch_bytes(int64_t S, int64_t D, int64_t heads) {
  if (S <= 0 || heads <= 0 || D % heads) return 0;
  if (!tiled_ok(S, (int)(D / heads))) return 0;
  return (size_t)heads_per_chunk(S, heads) * (size_t)S * (size_t)score_ld(S) * sizeof(float);
}

int attention_core(const float* Q, const float* K, const float* V, int64_t S, int64_t D, int64_t heads, int causal,
                   __half* ctx16, float* scores, size_t scores_bytes, cudaStream_t s) {
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
  const bool al = ((reinterpret_cast<uintptr_t>(Q) | reinterpret_cast<uintptr_t>(K) |
                    reinterpret_cast<uintptr_t>(V)) & 15) == 0;
  if (al && tiled_ok(S, hd) && scores && scores_bytes >= attention_scratch_bytes(S, D, heads))
    return attention_tiled(Q, K, V, S, D, heads, hd, scale, causal, ctx16, scores, s);
  if (hd <= 32) return launch_attention<1>(Q, K, V, S, D, heads, hd, scale, causal, ctx16, s);
  if (hd <= 64) return launch_attention<2>(Q, K, V, S, D, heads, hd, scale, causal, ctx16, s);
  if (hd <= 128) return launch_attention<4>(Q, K, V, S, D, heads, hd, scale, causal, ctx16, s);
  if (hd <= 256) return launch_attention<8>(Q, K, V, S, D, heads, hd, scale, causal, ctx16, s);
  return launch_attention<16>(Q, K, V, S, D, heads, hd, scale, causal, ctx16, s);
}

}  // namespace smeai
