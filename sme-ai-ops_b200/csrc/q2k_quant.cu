// q2k_quant.cu -- fp32 -> ggml block_q2_K weight quantizer (ggml's from_float
// for Q2_K) and Q2_K -> fp32 decoding (to_float).
//
// Restates ggml-quants.c quantize_row_q2_K_ref / make_qkx2_quants (ggml 0.9.8):
// per 16-value group a (scale, min) fit with L in [0,3], |x| weights, 16
// perturbed inverse scales (rmin -0.5, step 0.1) and a weighted least-squares
// refit, best mean-absolute error kept; 16 scales and 16 mins quantized to 4
// bits against their maxima (d = max/15, dmin = max_min/15 as fp16); values
// requantized against the rounded (scale, min); four 2-bit values per byte.
// It is the weight generator for tests and benchmarks (weights normally
// arrive pre-quantized in GGUF files); hot-path parity is defined on
// identical blocks.  The file is compiled without contraction, so every
// expression rounds exactly like the CPU restatement built with
// -ffp-contract=off.
#include "common.cuh"
#include "kernels.h"

namespace smeai {

__device__ __forceinline__ int round_sep(float v) { return magic_round_bits(v + kMagic); }

// One thread fits one 16-value group.  Returns scale, writes -min and L[16].
__device__ float fit_group16(const float* x, const float* w, uint8_t* L, float* neg_min) {
  const int n = 16, nmax = 3;
  const float rmin = -0.5f, rdelta = 0.1f;
  const int nstep = 15;
  uint8_t trial[16];
  float lo = x[0], hi = x[0];
  float sw = w[0], swx = w[0] * x[0];
  for (int i = 1; i < n; ++i) {
    if (x[i] < lo) lo = x[i];
    if (x[i] > hi) hi = x[i];
    sw += w[i];
    swx += w[i] * x[i];
  }
  if (lo > 0.0f) lo = 0.0f;
  if (hi == lo) {
    for (int i = 0; i < n; ++i) L[i] = 0;
    *neg_min = -lo;
    return 0.0f;
  }
  float inv = (float)nmax / (hi - lo);
  float scale = 1.0f / inv;
  float best = 0.0f;
  for (int i = 0; i < n; ++i) {
    int l = round_sep(inv * (x[i] - lo));
    l = l < 0 ? 0 : (l > nmax ? nmax : l);
    L[i] = (uint8_t)l;
    float diff = scale * (float)l + lo - x[i];
    best += w[i] * fabsf(diff);
  }
  for (int step = 0; step <= nstep; ++step) {
    float inv_t = (rmin + rdelta * (float)step + (float)nmax) / (hi - lo);
    float sl = 0.0f, sl2 = 0.0f, sxl = 0.0f;
    for (int i = 0; i < n; ++i) {
      int l = round_sep(inv_t * (x[i] - lo));
      l = l < 0 ? 0 : (l > nmax ? nmax : l);
      trial[i] = (uint8_t)l;
      sl += w[i] * (float)l;
      sl2 += w[i] * (float)l * (float)l;
      sxl += w[i] * (float)l * x[i];
    }
    float det = sw * sl2 - sl * sl;
    if (det > 0.0f) {
      float s_t = (sw * sxl - swx * sl) / det;
      float m_t = (sl2 * swx - sl * sxl) / det;
      if (m_t > 0.0f) {
        m_t = 0.0f;
        s_t = sxl / sl2;
      }
      float err = 0.0f;
      for (int i = 0; i < n; ++i) {
        float diff = s_t * (float)trial[i] + m_t - x[i];
        err += w[i] * fabsf(diff);
      }
      if (err < best) {
        for (int i = 0; i < n; ++i) L[i] = trial[i];
        best = err;
        scale = s_t;
        lo = m_t;
      }
    }
  }
  *neg_min = -lo;
  return scale;
}

// 16 threads per 256-value block; blockDim.x = 256 -> 16 blocks per CTA.
__global__ void q2k_quantize_kernel(const float* __restrict__ x, int64_t nblocks, uint8_t* __restrict__ y) {
  __shared__ uint8_t sL[16][256];
  const int g = threadIdx.x & 15;          // group within block
  const int slot = threadIdx.x >> 4;       // block slot within CTA
  const int64_t blk = (int64_t)blockIdx.x * 16 + slot;
  const bool active = blk < nblocks;
  float xv[16], wv[16];
  uint8_t L[16];
  float scale = 0.f, nmin = 0.f;
  if (active) {
    const float* xb = x + blk * QK_K + g * 16;
    for (int i = 0; i < 16; ++i) { xv[i] = xb[i]; wv[i] = fabsf(xv[i]); }
    scale = fit_group16(xv, wv, L, &nmin);
  }
  // maxima over the 16 groups of the block (16-lane segments of the warp)
  float max_scale = scale > 0.f ? scale : 0.f, max_min = nmin > 0.f ? nmin : 0.f;
  for (int off = 8; off >= 1; off >>= 1) {
    max_scale = fmaxf(max_scale, __shfl_xor_sync(0xffffffffu, max_scale, off));
    max_min = fmaxf(max_min, __shfl_xor_sync(0xffffffffu, max_min, off));
  }
  uint8_t sc = 0;
  __half dh = __float2half_rn(0.f), dmh = __float2half_rn(0.f);
  if (max_scale > 0.f) {
    float inv = 15.0f / max_scale;
    sc = (uint8_t)round_sep(inv * scale);
    dh = __float2half_rn(max_scale / 15.0f);
  }
  if (max_min > 0.f) {
    float inv = 15.0f / max_min;
    sc |= (uint8_t)(round_sep(inv * nmin) << 4);
    dmh = __float2half_rn(max_min / 15.0f);
  }
  if (active) {
    float ds = __half2float(dh) * (float)(sc & 0xF);
    if (ds != 0.0f) {
      float ms = __half2float(dmh) * (float)(sc >> 4);
      for (int i = 0; i < 16; ++i) {
        int l = round_sep((xv[i] + ms) / ds);
        L[i] = (uint8_t)(l < 0 ? 0 : (l > 3 ? 3 : l));
      }
    }
    for (int i = 0; i < 16; ++i) sL[slot][g * 16 + i] = L[i];
  }
  __syncwarp();
  if (active) {
    uint8_t* out = y + blk * Q2K_BLOCK_BYTES;
    out[g] = sc;
    // bytes: thread g packs qs bytes 4g..4g+3
    for (int t = 0; t < 4; ++t) {
      int byte = g * 4 + t;
      int half = byte >> 5, l = byte & 31;
      const uint8_t* s = &sL[slot][half * 128 + l];
      out[16 + byte] = (uint8_t)(s[0] | (s[32] << 2) | (s[64] << 4) | (s[96] << 6));
    }
    if (g == 0) {
      *reinterpret_cast<__half*>(out + 80) = dh;
      *reinterpret_cast<__half*>(out + 82) = dmh;
    }
  }
}

__global__ void q2k_dequantize_kernel(const uint8_t* __restrict__ w, int64_t nblocks, float* __restrict__ y) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nblocks * QK_K) return;
  int64_t b = i / QK_K;
  int e = (int)(i % QK_K);
  const uint8_t* blk = w + b * Q2K_BLOCK_BYTES;
  int half = e >> 7, within = e & 127, shift = 2 * (within >> 5), l = within & 31;
  int q = (blk[16 + half * 32 + l] >> shift) & 3;
  int j = e >> 4;
  __half_raw dr, mr;
  dr.x = (unsigned short)(blk[80] | (blk[81] << 8));
  mr.x = (unsigned short)(blk[82] | (blk[83] << 8));
  float d = __half2float(__half(dr)), dmin = __half2float(__half(mr));
  float dl = d * (float)(blk[j] & 0xF);
  float ml = dmin * (float)(blk[j] >> 4);
  y[i] = dl * (float)q - ml;
}

int q2k_quantize(const float* x, int64_t k_total, void* y, cudaStream_t stream) {
  if (k_total <= 0 || k_total % QK_K) {
    set_last_error("q2k_quantize: element count must be a positive multiple of 256");
    return kBadArgument;
  }
  int64_t nb = k_total / QK_K;
  SMEAI_CUDA_TRY(launch(q2k_quantize_kernel, dim3((unsigned)((nb + 15) / 16)), dim3(256), 0, stream, x, nb,
                        static_cast<uint8_t*>(y)));
  return kOk;
}

int q2k_dequantize(const void* w, int64_t k_total, float* y, cudaStream_t stream) {
  if (k_total <= 0 || k_total % QK_K) {
    set_last_error("q2k_dequantize: element count must be a positive multiple of 256");
    return kBadArgument;
  }
  int64_t nb = k_total / QK_K;
  SMEAI_CUDA_TRY(launch(q2k_dequantize_kernel, dim3((unsigned)((k_total + 255) / 256)), dim3(256), 0, stream,
                        static_cast<const uint8_t*>(w), nb, y));
  return kOk;
}

}  // namespace smeai
