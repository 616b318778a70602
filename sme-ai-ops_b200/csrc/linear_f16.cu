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

template <int EPI, typename TIn>
int launch_linear(const TIn* A, int64_t M, int64_t K, int64_t lda, const TIn* B, const TIn* B2, int64_t ldb,
                  int64_t N, const float* bias, const float* bias2, int act, float* C, __half* C16, int64_t ldc,
                  cudaStream_t s) {
  // Large problems: 64x64 tiles of 256 threads; small ones: 32x32 tiles of 64
  // threads so that more SMs take part.
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
