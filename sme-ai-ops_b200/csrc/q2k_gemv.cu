// q2k_gemv.cu -- Q2_K x Q8_K decode GEMV (1..8 activation rows), the
// HBM-bound core of the reference's Q2_K mul_mat (ggml_vec_dot_q2_K_q8_K /
// ggml_gemv_q2_K_8x8_q8_K, llama.cpp/doc/SME_Q2K_OPTIMIZATION.md:105-136).
//
// Work decomposition (one CTA = 32 weight rows, lane = row):
//   * weights arrive in the tile layout built by q2k_repack_kernel, so every
//     128-bit load of a warp covers 512 contiguous bytes;
//   * warp w of the CTA walks a contiguous range of super-blocks; the first
//     block's weights are loaded before griddepcontrol.wait, so they stream
//     while the kernel that produced the activations drains;
//   * the Q8_K activations of the CTA's tokens are staged once into shared
//     memory (16-byte aligned planes) and read by broadcast;
//   * the 2-bit quants are masked in place (no shift) and fed to
//     dp4a.u32.s32; each sub-block's sum is shifted back by 2*shift bits and
//     scaled by its 4-bit scale -- exact integer arithmetic, identical to
//     ggml's isum; the min term uses dp2a on the Q8_K bsums;
//   * per super-block the float term fmaf(d_x*d, isum, -(d_x*dmin*summs)) is
//     written to shared memory and summed over super-blocks in ascending order
//     by one thread per (row, token): the same rounding sequence as the CPU
//     restatement of ggml's generic dot;
//   * fused epilogues: plain store, residual add, or silu(gate)*up over
//     interleaved (gate, up) row pairs.
#include "common.cuh"
#include "kernels.h"

namespace smeai {

namespace {

struct WBlock {
  uint4 q[4];
  uint4 s;
  unsigned dm;
};

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

__device__ __forceinline__ void load_wblock(const uint8_t* tile, int lane, WBlock& wb) {
  const uint4* t4 = reinterpret_cast<const uint4*>(tile);
  wb.q[0] = ldg_stream(t4 + 0 * 32 + lane);
  wb.q[1] = ldg_stream(t4 + 1 * 32 + lane);
  wb.q[2] = ldg_stream(t4 + 2 * 32 + lane);
  wb.q[3] = ldg_stream(t4 + 3 * 32 + lane);
  wb.s = ldg_stream(t4 + 4 * 32 + lane);
  wb.dm = ldg_stream(reinterpret_cast<const unsigned*>(tile + 5 * 512) + lane);
}

// Shared-memory planes for T tokens x nb super-blocks.
struct ActSmem {
  int4* qs;      // [T*nb][16]  (256 int8 per block)
  int* bs;       // [T*nb][8]   (16 int16 bsums per block)
  float* d;      // [T*nb]
  float* terms;  // [T*nb][32]
};

__device__ __forceinline__ ActSmem carve(uint8_t* base, int tnb) {
  ActSmem a;
  a.qs = reinterpret_cast<int4*>(base);
  a.bs = reinterpret_cast<int*>(base + (size_t)tnb * 256);
  a.d = reinterpret_cast<float*>(base + (size_t)tnb * (256 + 32));
  a.terms = reinterpret_cast<float*>(base + (size_t)tnb * (256 + 32 + 4));
  return a;
}

// Copy T ggml Q8_K rows (contiguous, 292 B per block) into the planes.
__device__ __forceinline__ void stage_activations(const uint8_t* __restrict__ xq, int tnb, const ActSmem& a) {
  const uint32_t* src = reinterpret_cast<const uint32_t*>(xq);
  const int total = tnb * Q8K_BLOCK_WORDS;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int blk = i / Q8K_BLOCK_WORDS, w = i - blk * Q8K_BLOCK_WORDS;
    const uint32_t v = src[i];
    if (w == 0) {
      a.d[blk] = __uint_as_float(v);
    } else if (w <= 64) {
      reinterpret_cast<uint32_t*>(a.qs)[blk * 64 + (w - 1)] = v;
    } else {
      a.bs[blk * 8 + (w - 65)] = (int)v;
    }
  }
}

// Integer core for one super-block of this lane's row against T tokens.
template <int T>
__device__ __forceinline__ void block_isums(const WBlock& wb, const ActSmem& a, int nb, int b, int (&isum)[T],
                                            int (&summs)[T]) {
  const unsigned sw[4] = {wb.s.x, wb.s.y, wb.s.z, wb.s.w};
#pragma unroll
  for (int t = 0; t < T; ++t) isum[t] = 0;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const unsigned q0 = wb.q[c].x, q1 = wb.q[c].y, q2 = wb.q[c].z, q3 = wb.q[c].w;
    const int h = c >> 1, hf = c & 1;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const unsigned mask = 0x03030303u << (2 * s);
      const unsigned m0 = q0 & mask, m1 = q1 & mask, m2 = q2 & mask, m3 = q3 & mask;
      const int j = 8 * h + 2 * s + hf;  // sub-block of these 16 quants
      const int sc = (int)((sw[j >> 2] >> (8 * (j & 3))) & 0xFu);
      const int chunk = h * 8 + s * 2 + hf;  // 16-byte activation chunk within the block
#pragma unroll
      for (int t = 0; t < T; ++t) {
        const int4 av = a.qs[(t * nb + b) * 16 + chunk];
        int acc = dp4a_us(m0, av.x, 0);
        acc = dp4a_us(m1, av.y, acc);
        acc = dp4a_us(m2, av.z, acc);
        acc = dp4a_us(m3, av.w, acc);
        isum[t] += sc * (acc >> (2 * s));
      }
    }
  }
#pragma unroll
  for (int t = 0; t < T; ++t) {
    const int* bsp = a.bs + (t * nb + b) * 8;
    int mm = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const unsigned m4 = (sw[k] >> 4) & 0x0F0F0F0Fu;
      mm = dp2a_lo_su(bsp[2 * k], m4, mm);
      mm = dp2a_hi_su(bsp[2 * k + 1], m4, mm);
    }
    summs[t] = mm;
  }
}

__device__ __forceinline__ float half_lo(unsigned v) {
  __half_raw r;
  r.x = (unsigned short)(v & 0xffffu);
  return __half2float(__half(r));
}
__device__ __forceinline__ float half_hi(unsigned v) {
  __half_raw r;
  r.x = (unsigned short)(v >> 16);
  return __half2float(__half(r));
}

template <int T, int EPI, bool SUMS>
__global__ void __launch_bounds__(kThreads) q2k_gemv_kernel(const uint8_t* __restrict__ tiles, int nb,
                                                            int64_t n_rows, const uint8_t* __restrict__ xq,
                                                            float* y, int64_t ldy, const float* resid,
                                                            int64_t ld_resid, int32_t* __restrict__ isum_out,
                                                            int32_t* __restrict__ summs_out) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t group = blockIdx.x;
  const uint8_t* gtiles = tiles + group * (int64_t)nb * kTileBytes;
  const int b0 = (warp * nb) / kWarps, b1 = ((warp + 1) * nb) / kWarps;

  WBlock cur;
  if (b0 < b1) load_wblock(gtiles + (int64_t)b0 * kTileBytes, lane, cur);
  pdl_trigger();
  pdl_wait();

  const ActSmem a = carve(smem, T * nb);
  stage_activations(xq, T * nb, a);
  __syncthreads();

  for (int b = b0; b < b1; ++b) {
    WBlock nxt;
    if (b + 1 < b1) load_wblock(gtiles + (int64_t)(b + 1) * kTileBytes, lane, nxt);
    int isum[T], summs[T];
    block_isums<T>(cur, a, nb, b, isum, summs);
    if constexpr (SUMS) {
      const int64_t row = group * 32 + lane;
      if (row < n_rows) {
        isum_out[row * nb + b] = isum[0];
        summs_out[row * nb + b] = summs[0];
      }
    } else {
      const float dw = half_lo(cur.dm), dmw = half_hi(cur.dm);
#pragma unroll
      for (int t = 0; t < T; ++t) {
        const float dx = a.d[t * nb + b];
        const float dall = __fmul_rn(dx, dw);
        const float dmn = __fmul_rn(dx, dmw);
        const float term = __fmaf_rn(dall, __int2float_rn(isum[t]), -__fmul_rn(dmn, __int2float_rn(summs[t])));
        a.terms[(t * nb + b) * 32 + lane] = term;
      }
    }
    if (b + 1 < b1) cur = nxt;
  }
  if constexpr (SUMS) return;
  __syncthreads();

  if constexpr (EPI == kEpiSiluMul) {
    // 16 (gate, up) pairs per group and token
    for (int i = threadIdx.x; i < T * 16; i += blockDim.x) {
      const int t = i >> 4, p = i & 15;
      float g = 0.f, u = 0.f;
      for (int b = 0; b < nb; ++b) {
        g = __fadd_rn(g, a.terms[(t * nb + b) * 32 + 2 * p]);
        u = __fadd_rn(u, a.terms[(t * nb + b) * 32 + 2 * p + 1]);
      }
      const int64_t orow = group * 16 + p;
      if (2 * orow < n_rows) {
        const float sg = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
        y[t * ldy + orow] = __fmul_rn(sg, u);
      }
    }
  } else {
    for (int i = threadIdx.x; i < T * 32; i += blockDim.x) {
      const int t = i >> 5, r = i & 31;
      float s = 0.f;
      for (int b = 0; b < nb; ++b) s = __fadd_rn(s, a.terms[(t * nb + b) * 32 + r]);
      const int64_t row = group * 32 + r;
      if (row < n_rows) {
        if constexpr (EPI == kEpiResidual) s = __fadd_rn(resid[t * ld_resid + row], s);
        y[t * ldy + row] = s;
      }
    }
  }
}

// Scatter ggml blocks [n_rows][nb] (84 B each, 4-byte aligned) into tiles.
__global__ void q2k_repack_kernel(const uint8_t* __restrict__ src, int64_t n_rows, int nb, int64_t n_groups,
                                  uint8_t* __restrict__ tiles) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // (group, b, lane)
  if (i >= n_groups * nb * 32) return;
  const int lane = (int)(i & 31);
  const int64_t gb = i >> 5;
  const int64_t group = gb / nb;
  const int b = (int)(gb % nb);
  const int64_t row = group * 32 + lane;
  uint32_t w[21];
  if (row < n_rows) {
    const uint32_t* s = reinterpret_cast<const uint32_t*>(src + (row * nb + b) * (int64_t)Q2K_BLOCK_BYTES);
#pragma unroll
    for (int k = 0; k < 21; ++k) w[k] = s[k];
  } else {
#pragma unroll
    for (int k = 0; k < 21; ++k) w[k] = 0u;
  }
  uint8_t* tile = tiles + gb * kTileBytes;
  // ggml block words: 0..3 scales, 4..19 qs, 20 d|dmin
  uint4* t4 = reinterpret_cast<uint4*>(tile);
#pragma unroll
  for (int c = 0; c < 4; ++c) t4[c * 32 + lane] = make_uint4(w[4 + 4 * c], w[5 + 4 * c], w[6 + 4 * c], w[7 + 4 * c]);
  t4[4 * 32 + lane] = make_uint4(w[0], w[1], w[2], w[3]);
  reinterpret_cast<uint32_t*>(tile + 5 * 512)[lane] = w[20];
}

size_t gemv_smem_bytes(int T, int nb) { return (size_t)T * nb * (256 + 32 + 4 + 128); }

template <int T, int EPI, bool SUMS>
int launch_gemv(const Q2KWeight& w, const uint8_t* xq, float* y, int64_t ldy, const float* resid,
                int64_t ld_resid, int32_t* isum, int32_t* summs, cudaStream_t stream) {
  auto kern = q2k_gemv_kernel<T, EPI, SUMS>;
  const size_t smem = gemv_smem_bytes(T, w.nb);
  static unsigned configured = 0;  // per template instance, one bit per device
  int dev = 0;
  SMEAI_CUDA_TRY(cudaGetDevice(&dev));
  if (!(configured & (1u << (dev & 31)))) {
    SMEAI_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    configured |= 1u << (dev & 31);
  }
  SMEAI_CUDA_TRY(launch(kern, dim3((unsigned)w.n_groups), dim3(kThreads), smem, stream,
                        (const uint8_t*)w.tiles, w.nb, w.n_rows, xq, y, ldy, resid, ld_resid, isum, summs));
  return kOk;
}

template <int EPI>
int dispatch_t(int T, const Q2KWeight& w, const uint8_t* xq, float* y, int64_t ldy, const float* resid,
               int64_t ld_resid, cudaStream_t s) {
  switch (T) {
    case 1: return launch_gemv<1, EPI, false>(w, xq, y, ldy, resid, ld_resid, nullptr, nullptr, s);
    case 2: return launch_gemv<2, EPI, false>(w, xq, y, ldy, resid, ld_resid, nullptr, nullptr, s);
    case 3: return launch_gemv<3, EPI, false>(w, xq, y, ldy, resid, ld_resid, nullptr, nullptr, s);
    case 4: return launch_gemv<4, EPI, false>(w, xq, y, ldy, resid, ld_resid, nullptr, nullptr, s);
    case 5: return launch_gemv<5, EPI, false>(w, xq, y, ldy, resid, ld_resid, nullptr, nullptr, s);
    case 6: return launch_gemv<6, EPI, false>(w, xq, y, ldy, resid, ld_resid, nullptr, nullptr, s);
    case 7: return launch_gemv<7, EPI, false>(w, xq, y, ldy, resid, ld_resid, nullptr, nullptr, s);
    case 8: return launch_gemv<8, EPI, false>(w, xq, y, ldy, resid, ld_resid, nullptr, nullptr, s);
    default: return kBadArgument;
  }
}

}  // namespace

size_t q2k_tile_bytes(int64_t n_rows, int64_t k) {
  const int64_t groups = (n_rows + kRowsPerGroup - 1) / kRowsPerGroup;
  return (size_t)groups * (size_t)(k / QK_K) * kTileBytes;
}

int q2k_repack_into(const void* w_blocks_dev, int64_t n_rows, int64_t k, uint8_t* tiles, Q2KWeight* out,
                    cudaStream_t stream) {
  if (!w_blocks_dev || !tiles || !out || n_rows <= 0 || k <= 0 || k % QK_K) {
    set_last_error("q2k_repack: bad arguments (rows=%lld k=%lld)", (long long)n_rows, (long long)k);
    return kBadArgument;
  }
  if ((reinterpret_cast<uintptr_t>(w_blocks_dev) & 3) || (reinterpret_cast<uintptr_t>(tiles) & 15)) {
    set_last_error("q2k_repack: blocks must be 4-byte and tiles 16-byte aligned");
    return kBadArgument;
  }
  Q2KWeight w;
  w.n_rows = n_rows;
  w.k = k;
  w.nb = (int)(k / QK_K);
  w.n_groups = (n_rows + kRowsPerGroup - 1) / kRowsPerGroup;
  w.bytes = q2k_tile_bytes(n_rows, k);
  w.tiles = tiles;
  SMEAI_CUDA_TRY(cudaGetDevice(&w.device));
  const int64_t threads = w.n_groups * w.nb * 32;
  SMEAI_CUDA_TRY(launch(q2k_repack_kernel, dim3((unsigned)((threads + 255) / 256)), dim3(256), 0, stream,
                        static_cast<const uint8_t*>(w_blocks_dev), n_rows, w.nb, w.n_groups, tiles));
  *out = w;
  return kOk;
}

int q2k_repack(const void* w_blocks_dev, int64_t n_rows, int64_t k, Q2KWeight* out, cudaStream_t stream) {
  if (n_rows <= 0 || k <= 0 || k % QK_K) {
    set_last_error("q2k_repack: bad arguments (rows=%lld k=%lld)", (long long)n_rows, (long long)k);
    return kBadArgument;
  }
  const size_t bytes = q2k_tile_bytes(n_rows, k);
  uint8_t* tiles = nullptr;
  if (cudaMalloc(&tiles, bytes) != cudaSuccess) {
    cudaGetLastError();
    set_last_error("q2k_repack: cudaMalloc of %zu bytes failed", bytes);
    return kAllocFailed;
  }
  const int st = q2k_repack_into(w_blocks_dev, n_rows, k, tiles, out, stream);
  if (st != kOk) cudaFree(tiles);
  return st;
}

int q2k_gemv(const Q2KWeight& w, const void* xq, int64_t n_cols, float* y, int64_t ldy, int epilogue,
             const float* resid, int64_t ld_resid, cudaStream_t stream) {
  if (!w.tiles || !xq || !y || n_cols <= 0) {
    set_last_error("q2k_gemv: bad arguments");
    return kBadArgument;
  }
  if (reinterpret_cast<uintptr_t>(xq) & 3) {
    set_last_error("q2k_gemv: Q8_K activations must be 4-byte aligned");
    return kBadArgument;
  }
  if (epilogue == kEpiResidual && !resid) {
    set_last_error("q2k_gemv: residual epilogue needs a residual pointer");
    return kBadArgument;
  }
  if (epilogue == kEpiSiluMul && (w.n_rows & 1)) {
    set_last_error("q2k_gemv: silu*mul epilogue needs interleaved (gate, up) row pairs");
    return kBadArgument;
  }
  const int64_t out_rows = epilogue == kEpiSiluMul ? w.n_rows / 2 : w.n_rows;
  if (ldy < out_rows || (epilogue == kEpiResidual && ld_resid < out_rows)) {
    set_last_error("q2k_gemv: leading dimension smaller than the output rows");
    return kBadArgument;
  }
  const size_t q8_row_bytes = (size_t)w.nb * Q8K_BLOCK_BYTES;
  for (int64_t c0 = 0; c0 < n_cols;) {
    int T = (int)((n_cols - c0) > 8 ? 8 : (n_cols - c0));
    while (T > 1 && gemv_smem_bytes(T, w.nb) > 227 * 1024) --T;
    if (gemv_smem_bytes(T, w.nb) > 227 * 1024) {
      set_last_error("q2k_gemv: k=%lld too large for the shared-memory staging", (long long)w.k);
      return kBadArgument;
    }
    const uint8_t* xc = static_cast<const uint8_t*>(xq) + c0 * q8_row_bytes;
    float* yc = y + c0 * ldy;
    const float* rc = resid ? resid + c0 * ld_resid : nullptr;
    int st;
    switch (epilogue) {
      case kEpiStore: st = dispatch_t<kEpiStore>(T, w, xc, yc, ldy, rc, ld_resid, stream); break;
      case kEpiResidual: st = dispatch_t<kEpiResidual>(T, w, xc, yc, ldy, rc, ld_resid, stream); break;
      case kEpiSiluMul: st = dispatch_t<kEpiSiluMul>(T, w, xc, yc, ldy, rc, ld_resid, stream); break;
      default:
        set_last_error("q2k_gemv: unknown epilogue %d", epilogue);
        return kBadArgument;
    }
    if (st != kOk) return st;
    c0 += T;
  }
  return kOk;
}

int q2k_block_sums(const Q2KWeight& w, const void* xq, int32_t* isum, int32_t* summs, cudaStream_t stream) {
  if (!w.tiles || !xq || !isum || !summs) {
    set_last_error("q2k_block_sums: bad arguments");
    return kBadArgument;
  }
  return launch_gemv<1, kEpiStore, true>(w, static_cast<const uint8_t*>(xq), nullptr, 0, nullptr, 0, isum, summs,
                                          stream);
}

}  // namespace smeai
