// linear_f16.cu -- the sme_ai_library packed Linear / MLP / SwiGLU operators
// (sme_ai_library/src/sme_ai_ops.c:361-462, 504-557, 1227-1265) on sm_100a.
//
// Numerics follow the reference exactly: every output is a k-ascending fp32
// sum of fp16 x fp16 products (exact in fp32, so the fused FFMA used here
// rounds identically to the reference's acc += a*b and to its FMOPA tile,
// .S:56-68), then + bias (one rounding), then the activation.  The GEMM keeps
// one accumulator per output in registers (4x4 outputs per thread) and walks k
// in order, so the result is bit-identical to the scalar reference loop
// (scalar_matmul_f16f16_f32, :251-267) for fp16 inputs.
//
// Fused epilogues replace the reference's separate passes:
//   kEpiF32      y = act(acc + bias)                     (fp32 out)
//   kEpiF16      h = fp16(act(acc + bias))               (MLP hidden, :504-529)
//   kEpiSwiGLU   h = fp16(silu(acc_g + bg) * (acc_u + bu)) (gate and up in one
//                kernel: two accumulator sets over one A tile, :1227-1265)
#include <type_traits>

#include "common.cuh"
#include "linear.h"

namespace smeai {

namespace {

constexpr int BK = 16;

__device__ __forceinline__ float gelu_tanh(float x) {
  const float c0 = 0.7978845608f;
  const float c1 = 0.044715f;
  float cube = x * x * x;
  float inner = c0 * (x + c1 * cube);
  return 0.5f * x * (1.0f + tanhf(inner));
}

__device__ __forceinline__ float activate(float x, int act) {
  switch (act) {
    case kActRelu: return x > 0.0f ? x : 0.0f;
    case kActGelu: return gelu_tanh(x);
    case kActSilu: return x / (1.0f + expf(-x));
    default: return x;
  }
}

// Tile BM x BN, (BM/TM) x (BN/TN) threads, k step BK, register accumulators.
template <int BM, int BN, int TM, int TN, int EPI, typename TIn>
__global__ void __launch_bounds__((BM / TM) * (BN / TN)) linear_ffma_kernel(
    const TIn* __restrict__ A, int64_t M, int64_t K, int64_t lda, const TIn* __restrict__ B,
    const TIn* __restrict__ B2, int64_t ldb, int64_t N, const float* __restrict__ bias,
    const float* __restrict__ bias2, int act, float* __restrict__ C, __half* __restrict__ C16, int64_t ldc) {
  constexpr int NT = (BM / TM) * (BN / TN);
  constexpr bool kPair = EPI == kEpiSwiGLU;
  __shared__ __align__(16) float As[2][BK][BM];
  __shared__ __align__(16) float Bs[2][BK][BN];
  __shared__ __align__(16) float Bs2[kPair ? 2 : 1][BK][kPair ? BN : 4];

  const int tid = threadIdx.x;
  const int tx = tid % (BN / TN), ty = tid / (BN / TN);
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;

  float acc[TM][TN], acc2[kPair ? TM : 1][kPair ? TN : 1];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;
  if constexpr (kPair) {
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) acc2[i][j] = 0.f;
  }

  pdl_trigger();
  pdl_wait();

  auto load_tiles = [&](int buf, int64_t k0) {
    for (int e = tid; e < BM * BK; e += NT) {
      const int r = e / BK, c = e % BK;
      const int64_t gm = m0 + r, gk = k0 + c;
      float v = 0.f;
      if (gm < M && gk < K) v = (float)A[gm * lda + gk];
      As[buf][c][r] = v;
    }
    for (int e = tid; e < BK * BN; e += NT) {
      const int r = e / BN, c = e % BN;
      const int64_t gk = k0 + r, gn = n0 + c;
      float v = 0.f, v2 = 0.f;
      if (gk < K && gn < N) {
        v = (float)B[gk * ldb + gn];
        if constexpr (kPair) v2 = (float)B2[gk * ldb + gn];
      }
      Bs[buf][r][c] = v;
      if constexpr (kPair) Bs2[buf][r][c] = v2;
    }
  };

  int buf = 0;
  load_tiles(0, 0);
  __syncthreads();
  for (int64_t k0 = 0; k0 < K; k0 += BK) {
    if (k0 + BK < K) load_tiles(buf ^ 1, k0 + BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[TM], b[TN];
#pragma unroll
      for (int i = 0; i < TM; ++i) a[i] = As[buf][kk][ty * TM + i];
#pragma unroll
      for (int j = 0; j < TN; ++j) b[j] = Bs[buf][kk][tx * TN + j];
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
      if constexpr (kPair) {
        float b2[TN];
#pragma unroll
        for (int j = 0; j < TN; ++j) b2[j] = Bs2[buf][kk][tx * TN + j];
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
          for (int j = 0; j < TN; ++j) acc2[i][j] = __fmaf_rn(a[i], b2[j], acc2[i][j]);
      }
    }
    __syncthreads();
    buf ^= 1;
  }

#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int64_t gm = m0 + ty * TM + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int64_t gn = n0 + tx * TN + j;
      if (gn >= N) continue;
      float v = acc[i][j];
      if (bias) v = v + bias[gn];
      if constexpr (EPI == kEpiSwiGLU) {
        float u = acc2[i][j];
        if (bias2) u = u + bias2[gn];
        const float s = v / (1.0f + expf(-v));
        C16[gm * ldc + gn] = __float2half_rn(s * u);
      } else if constexpr (EPI == kEpiF16) {
        C16[gm * ldc + gn] = __float2half_rn(activate(v, act));
      } else {
        C[gm * ldc + gn] = activate(v, act);
      }
    }
  }
}

// Register-tiled FFMA GEMM for large fp16 problems.  CTA tile 128 x BN
// (BN = 16 * TN) of outputs, 256 threads as 16 x 16, each owning 8 x TN
// outputs: rows ty*4 + {0..3} and 64 + ty*4 + {0..3}, columns tx*TN/2 + ..
// and BN/2 + tx*TN/2 + .., so every shared-memory vector read of a warp is
// conflict-free.  k advances 16 at a time: the next step's operands are
// fetched into registers (one 16-byte load of A and one TN-half load of B
// per thread) while the current step's FFMAs run, then converted to fp32 and
// stored into the other shared buffer.  Each output still sums its products
// in k order with one accumulator, so results are those of linear_ffma_kernel
// bit for bit.  Requirements (checked by the launcher): K and lda multiples of
// 8, ldb a multiple of 16, 16-byte aligned A and B, B zero padded to
// round_up(K, 16) rows and ldb columns (the packed-weight layout).
template <int TN, int EPI>
__global__ void __launch_bounds__(256, 2) linear_tiled_kernel(
    const __half* __restrict__ A, int64_t M, int64_t K, int64_t lda, const __half* __restrict__ B,
    const __half* __restrict__ B2, int64_t ldb, int64_t N, const float* __restrict__ bias,
    const float* __restrict__ bias2, int act, float* __restrict__ C, __half* __restrict__ C16, int64_t ldc) {
  constexpr int BM = 128, BN = 16 * TN, HN = TN / 2;
  constexpr bool kPair = EPI == kEpiSwiGLU;
  using BVec = typename std::conditional<TN == 8, uint4, uint2>::type;
  __shared__ __align__(16) float As[2][BK][BM];
  __shared__ __align__(16) float Bs[2][BK][BN];
  __shared__ __align__(16) float Bs2[kPair ? 2 : 1][BK][kPair ? BN : 4];

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  // operand fetch coordinates: A row tid % 128, k half tid / 128; B row tid / 16, TN columns
  const int ra = tid & 127, ka = (tid >> 7) * 8;
  const int rb = tid >> 4, cb = (tid & 15) * TN;
  const bool a_row = m0 + ra < M;
  const bool b_col = n0 + cb + TN <= ldb;
  const __half* a_src = A + (a_row ? (m0 + ra) * lda : 0) + ka;
  const __half* b_src = B + (int64_t)rb * ldb + n0 + cb;
  const __half* b2_src = kPair ? B2 + (int64_t)rb * ldb + n0 + cb : nullptr;

  float acc[8][TN], acc2[kPair ? 8 : 1][kPair ? TN : 1];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;
  if constexpr (kPair) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) acc2[i][j] = 0.f;
  }

  pdl_trigger();
  pdl_wait();

  uint4 av;
  BVec bv, bv2;
  auto fetch = [&](int64_t k0) {
    av = (a_row && k0 + ka < K) ? *reinterpret_cast<const uint4*>(a_src + k0) : make_uint4(0, 0, 0, 0);
    if (b_col) {
      bv = *reinterpret_cast<const BVec*>(b_src + k0 * ldb);
      if constexpr (kPair) bv2 = *reinterpret_cast<const BVec*>(b2_src + k0 * ldb);
    } else {
      bv = BVec{};
      if constexpr (kPair) bv2 = BVec{};
    }
  };
  auto stash = [&](int buf) {
    const __half* ah = reinterpret_cast<const __half*>(&av);
#pragma unroll
    for (int i = 0; i < 8; ++i) As[buf][ka + i][ra] = __half2float(ah[i]);
    const __half* bh = reinterpret_cast<const __half*>(&bv);
#pragma unroll
    for (int j = 0; j < TN; j += 4)
      *reinterpret_cast<float4*>(&Bs[buf][rb][cb + j]) =
          make_float4(__half2float(bh[j]), __half2float(bh[j + 1]), __half2float(bh[j + 2]), __half2float(bh[j + 3]));
    if constexpr (kPair) {
      const __half* b2h = reinterpret_cast<const __half*>(&bv2);
#pragma unroll
      for (int j = 0; j < TN; j += 4)
        *reinterpret_cast<float4*>(&Bs2[buf][rb][cb + j]) = make_float4(
            __half2float(b2h[j]), __half2float(b2h[j + 1]), __half2float(b2h[j + 2]), __half2float(b2h[j + 3]));
    }
  };

  const int64_t nk = (K + BK - 1) / BK;
  fetch(0);
  stash(0);
  __syncthreads();
  int buf = 0;
  for (int64_t kt = 0; kt < nk; ++kt) {
    const bool more = kt + 1 < nk;
    if (more) fetch((kt + 1) * BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[8], b[TN];
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
      a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
      a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
      if constexpr (TN == 8) {
        const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
        const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
        b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
        b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
      } else {
        const float2 b0 = *reinterpret_cast<const float2*>(&Bs[buf][kk][tx * 2]);
        const float2 b1 = *reinterpret_cast<const float2*>(&Bs[buf][kk][32 + tx * 2]);
        b[0] = b0.x; b[1] = b0.y; b[2] = b1.x; b[3] = b1.y;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
      if constexpr (kPair) {
        float b2[TN];
        const float2 c0 = *reinterpret_cast<const float2*>(&Bs2[buf][kk][tx * 2]);
        const float2 c1 = *reinterpret_cast<const float2*>(&Bs2[buf][kk][32 + tx * 2]);
        b2[0] = c0.x; b2[1] = c0.y; b2[2] = c1.x; b2[3] = c1.y;
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < TN; ++j) acc2[i][j] = __fmaf_rn(a[i], b2[j], acc2[i][j]);
      }
    }
    if (more) stash(buf ^ 1);
    __syncthreads();
    buf ^= 1;
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t gm = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int64_t gn = n0 + (j < HN ? tx * HN + j : BN / 2 + tx * HN + j - HN);
      if (gn >= N) continue;
      float v = acc[i][j];
      if (bias) v = v + bias[gn];
      if constexpr (EPI == kEpiSwiGLU) {
        float u = acc2[i][j];
        if (bias2) u = u + bias2[gn];
        const float sv = v / (1.0f + expf(-v));
        C16[gm * ldc + gn] = __float2half_rn(sv * u);
      } else if constexpr (EPI == kEpiF16) {
        C16[gm * ldc + gn] = __float2half_rn(activate(v, act));
      } else {
        C[gm * ldc + gn] = activate(v, act);
      }
    }
  }
}

// FFMA GEMM for small and mid-sized fp16 problems (fewer than 120 tiles of
// the register-tiled kernel, e.g. the 128 x 512 x 512 Linear): CTA tile 16 x
// 32 outputs, 128 threads as 8 x 16, each owning a 2 x 2 block, so a small
// problem still spreads over many SMs.  Every output is a chain of K
// dependent FFMAs and a scheduler holds about one warp, so the products run in
// batches of 8 k: the batch's operands are read from shared memory into
// registers first (one latency per batch instead of one per k).  k advances
// in chunks of 256: the next chunk's fp16 operands are fetched into registers
// (12 16-byte loads per thread, all in flight together) while the current
// chunk's products run from shared memory (fp32, k-major), then converted and
// stored after a barrier.  Operands beyond K are zero: the accumulator starts
// at +0 and never becomes -0, so 0 * 0 leaves it unchanged.  One accumulator
// per output walked in k order: the results of linear_ffma_kernel bit for
// bit.  Requirements (checked by the launcher): K, lda and ldb multiples of 8,
// 16-byte aligned A and B, ldb >= N.
constexpr int kSmallBM = 16, kSmallBN = 32, kSmallKC = 256, kSmallNT = 128;
template <int EPI>
__global__ void __launch_bounds__(kSmallNT) linear_small_kernel(const __half* __restrict__ A, int64_t M, int64_t K,
                                                                int64_t lda, const __half* __restrict__ B,
                                                                int64_t ldb, int64_t N,
                                                                const float* __restrict__ bias, int act,
                                                                float* __restrict__ C, __half* __restrict__ C16,
                                                                int64_t ldc) {
  constexpr int BM = kSmallBM, BN = kSmallBN, KC = kSmallKC, NT = kSmallNT;
  constexpr int NA = BM * KC / 8 / NT, NB = KC * BN / 8 / NT;  // 16-byte loads per thread: 4 and 8
  __shared__ __align__(16) float As[KC][BM];
  __shared__ __align__(16) float Bs[KC][BN];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  float c00 = 0.f, c01 = 0.f, c10 = 0.f, c11 = 0.f;

  // dependents launch once the products are done: launched at the start,
  // their waiting CTAs share the SMs with this kernel's single warp per
  // scheduler (measured 20-40% slower)
  pdl_wait();

  uint4 ra[NA], rb[NB];
  // A load e = tid + NT i: row e % 16, k (e / 16) * 8; B load: k row e / 4, columns (e % 4) * 8
  auto fetch = [&](int64_t k0) {
#pragma unroll
    for (int i = 0; i < NA; ++i) {
      const int e = tid + NT * i, r = e % BM, kq = (e / BM) * 8;
      ra[i] = (m0 + r < M && k0 + kq < K) ? *reinterpret_cast<const uint4*>(A + (m0 + r) * lda + k0 + kq)
                                          : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < NB; ++i) {
      const int e = tid + NT * i, kr = e / 4, nq = (e % 4) * 8;
      rb[i] = (k0 + kr < K && n0 + nq + 8 <= ldb) ? *reinterpret_cast<const uint4*>(B + (k0 + kr) * ldb + n0 + nq)
                                                  : make_uint4(0, 0, 0, 0);
    }
  };
  auto stash = [&]() {
#pragma unroll
    for (int i = 0; i < NA; ++i) {
      const int e = tid + NT * i, r = e % BM, kq = (e / BM) * 8;
      const __half* h = reinterpret_cast<const __half*>(&ra[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) As[kq + j][r] = __half2float(h[j]);
    }
#pragma unroll
    for (int i = 0; i < NB; ++i) {
      const int e = tid + NT * i, kr = e / 4, nq = (e % 4) * 8;
      const __half* h = reinterpret_cast<const __half*>(&rb[i]);
      *reinterpret_cast<float4*>(&Bs[kr][nq]) =
          make_float4(__half2float(h[0]), __half2float(h[1]), __half2float(h[2]), __half2float(h[3]));
      *reinterpret_cast<float4*>(&Bs[kr][nq + 4]) =
          make_float4(__half2float(h[4]), __half2float(h[5]), __half2float(h[6]), __half2float(h[7]));
    }
  };

  fetch(0);
  for (int64_t k0 = 0; k0 < K; k0 += KC) {
    __syncthreads();  // the previous chunk's products are done with the shared tiles
    stash();
    __syncthreads();
    if (k0 + KC < K) fetch(k0 + KC);
#pragma unroll 1
    for (int kb = 0; kb < KC; kb += 8) {
      float2 a[8], b[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        a[u] = *reinterpret_cast<const float2*>(&As[kb + u][2 * ty]);
        b[u] = *reinterpret_cast<const float2*>(&Bs[kb + u][2 * tx]);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        c00 = __fmaf_rn(a[u].x, b[u].x, c00);
        c01 = __fmaf_rn(a[u].x, b[u].y, c01);
        c10 = __fmaf_rn(a[u].y, b[u].x, c10);
        c11 = __fmaf_rn(a[u].y, b[u].y, c11);
      }
    }
  }

  pdl_trigger();
  const float acc[2][2] = {{c00, c01}, {c10, c11}};
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int64_t gm = m0 + 2 * ty + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int64_t gn = n0 + 2 * tx + j;
      if (gn >= N) continue;
      float v = acc[i][j];
      if (bias) v = v + bias[gn];
      if constexpr (EPI == kEpiF16) {
        C16[gm * ldc + gn] = __float2half_rn(activate(v, act));
      } else {
        C[gm * ldc + gn] = activate(v, act);
      }
    }
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <int EPI, typename TIn>
int launch_linear(const TIn* A, int64_t M, int64_t K, int64_t lda, const TIn* B, const TIn* B2, int64_t ldb,
                  int64_t N, const float* bias, const float* bias2, int act, float* C, __half* C16, int64_t ldc,
                  cudaStream_t s) {
  // Large fp16 problems: the register-tiled kernel (128 x 128 tiles; 128 x 64
  // for the gate/up pair); mid-sized ones 64x64 tiles of 256 threads; small
  // ones 32x32 tiles of 64 threads so that more SMs take part.
  if constexpr (std::is_same<TIn, __half>::value) {
    constexpr int TN = EPI == kEpiSwiGLU ? 4 : 8;
    constexpr int BN = 16 * TN;
    const int64_t tiles = ((M + 127) / 128) * ((N + BN - 1) / BN);
    const bool ok = K % 8 == 0 && lda % 8 == 0 && ldb % 16 == 0 && ldb >= N && aligned16(A) && aligned16(B) &&
                    (EPI != kEpiSwiGLU || aligned16(B2));
    if (ok && tiles >= 120) {
      dim3 grid((unsigned)((N + BN - 1) / BN), (unsigned)((M + 127) / 128));
      SMEAI_CUDA_TRY(launch(linear_tiled_kernel<TN, EPI>, grid, dim3(256), 0, s, A, M, K, lda, B, B2, ldb, N, bias,
                            bias2, act, C, C16, ldc));
      return kOk;
    }
    if constexpr (EPI != kEpiSwiGLU) {
      if (K % 8 == 0 && lda % 8 == 0 && ldb % 8 == 0 && ldb >= N && aligned16(A) && aligned16(B)) {
        dim3 grid((unsigned)((N + kSmallBN - 1) / kSmallBN), (unsigned)((M + kSmallBM - 1) / kSmallBM));
        SMEAI_CUDA_TRY(launch(linear_small_kernel<EPI>, grid, dim3(kSmallNT), 0, s, A, M, K, lda, B, ldb, N, bias, act, C,
                              C16, ldc));
        return kOk;
      }
    }
  }
  const int64_t big_tiles = ((M + 63) / 64) * ((N + 63) / 64);
  if (big_tiles >= 148) {
    auto k = linear_ffma_kernel<64, 64, 4, 4, EPI, TIn>;
    dim3 grid((unsigned)((N + 63) / 64), (unsigned)((M + 63) / 64));
    SMEAI_CUDA_TRY(launch(k, grid, dim3(256), 0, s, A, M, K, lda, B, B2, ldb, N, bias, bias2, act, C, C16, ldc));
  } else {
    auto k = linear_ffma_kernel<32, 32, 4, 4, EPI, TIn>;
    dim3 grid((unsigned)((N + 31) / 32), (unsigned)((M + 31) / 32));
    SMEAI_CUDA_TRY(launch(k, grid, dim3(64), 0, s, A, M, K, lda, B, B2, ldb, N, bias, bias2, act, C, C16, ldc));
  }
  return kOk;
}

// ---- simple kernels backing the reference API's *_ref_* functions ----------
template <typename TIn>
__global__ void linear_ref_kernel(const TIn* __restrict__ A, int64_t M, int64_t K, const TIn* __restrict__ W,
                                  int64_t N, const float* __restrict__ bias, int act, float* __restrict__ C) {
  pdl_wait();  // A may be the previous kernel's output
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= M * N) return;
  const int64_t r = i / N, c = i % N;
  float acc = 0.f;
  for (int64_t k = 0; k < K; ++k) acc = __fmaf_rn((float)A[r * K + k], (float)W[k * N + c], acc);
  if (bias) acc = acc + bias[c];
  C[i] = activate(acc, act);
}

__global__ void f32_to_f16_kernel(const float* __restrict__ x, __half* __restrict__ y, int64_t n) {
  pdl_wait();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = __float2half_rn(x[i]);
}

__global__ void silu_mul_f16_kernel(const float* __restrict__ g, const float* __restrict__ u,
                                    __half* __restrict__ h, int64_t n) {
  pdl_wait();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const float x = g[i];
    const float s = x / (1.0f + expf(-x));
    h[i] = __float2half_rn(s * u[i]);
  }
}

__global__ void act_inplace_kernel(float* __restrict__ x, int64_t n, int act) {
  pdl_wait();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) x[i] = activate(x[i], act);
}

// Packed-weight layout on the device: fp16 [k_pad][n_pad], zero padded.
__global__ void pack_weight_kernel(const __half* __restrict__ w, int64_t K, int64_t N, __half* __restrict__ out,
                                   int64_t k_pad, int64_t n_pad) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= k_pad * n_pad) return;
  const int64_t k = i / n_pad, n = i % n_pad;
  out[i] = (k < K && n < N) ? w[k * N + n] : __float2half_rn(0.f);
}

unsigned blocks_for(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }

}  // namespace

int linear_f16(const __half* A, int64_t M, int64_t K, const __half* B, int64_t ldb, int64_t N, const float* bias,
               int act, float* C, cudaStream_t s) {
  return launch_linear<kEpiF32, __half>(A, M, K, K, B, nullptr, ldb, N, bias, nullptr, act, C, nullptr, N, s);
}

int linear_f16_to_f16(const __half* A, int64_t M, int64_t K, const __half* B, int64_t ldb, int64_t N,
                      const float* bias, int act, __half* C16, cudaStream_t s) {
  return launch_linear<kEpiF16, __half>(A, M, K, K, B, nullptr, ldb, N, bias, nullptr, act, nullptr, C16, N, s);
}

int swiglu_gate_up_f16(const __half* A, int64_t M, int64_t K, const __half* Bg, const __half* Bu, int64_t ldb,
                       int64_t N, const float* bg, const float* bu, __half* H16, cudaStream_t s) {
  return launch_linear<kEpiSwiGLU, __half>(A, M, K, K, Bg, Bu, ldb, N, bg, bu, kActNone, nullptr, H16, N, s);
}

int linear_f32(const float* A, int64_t M, int64_t K, const float* B, int64_t ldb, int64_t N, const float* bias,
               int act, float* C, cudaStream_t s) {
  return launch_linear<kEpiF32, float>(A, M, K, K, B, nullptr, ldb, N, bias, nullptr, act, C, nullptr, N, s);
}

int linear_ref_f16(const __half* A, int64_t M, int64_t K, const __half* W, int64_t N, const float* bias, int act,
                   float* C, cudaStream_t s) {
  SMEAI_CUDA_TRY(launch(linear_ref_kernel<__half>, dim3(blocks_for(M * N, 128)), dim3(128), 0, s, A, M, K, W, N,
                        bias, act, C));
  return kOk;
}

int f32_to_f16(const float* x, __half* y, int64_t n, cudaStream_t s) {
  SMEAI_CUDA_TRY(launch(f32_to_f16_kernel, dim3(blocks_for(n, 256)), dim3(256), 0, s, x, y, n));
  return kOk;
}

int silu_mul_f16(const float* g, const float* u, __half* h, int64_t n, cudaStream_t s) {
  SMEAI_CUDA_TRY(launch(silu_mul_f16_kernel, dim3(blocks_for(n, 256)), dim3(256), 0, s, g, u, h, n));
  return kOk;
}

int act_inplace(float* x, int64_t n, int act, cudaStream_t s) {
  if (act == kActNone) return kOk;
  SMEAI_CUDA_TRY(launch(act_inplace_kernel, dim3(blocks_for(n, 256)), dim3(256), 0, s, x, n, act));
  return kOk;
}

int pack_weight_f16(const __half* w, int64_t K, int64_t N, __half* out, int64_t k_pad, int64_t n_pad,
                    cudaStream_t s) {
  SMEAI_CUDA_TRY(launch(pack_weight_kernel, dim3(blocks_for(k_pad * n_pad, 256)), dim3(256), 0, s, w, K, N, out,
                        k_pad, n_pad));
  return kOk;
}

}  // namespace smeai
