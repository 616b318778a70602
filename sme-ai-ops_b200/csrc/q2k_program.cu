// q2k_program.cu -- a decode step (a chain of dependent Q2_K GEMVs) as ONE
// persistent cooperative kernel.
//
// Batch-1 decode of a Llama-shape stack is ~129 GEMVs (qkv, o, gate/up, down
// per layer, then lm_head), each reading the complete output of the one
// before it (after an RMSNorm, a silu*mul, or a plain re-quantization to
// Q8_K).  As separate launches every link costs a grid drain, a launch and a
// refill of the weight stream.  Here one CTA per SM runs the whole chain:
//   * warp 0, lane 0 (producer) streams this CTA's weight tiles of EVERY
//     phase, in program order, into a shared-memory ring with cp.async.bulk.
//     Weights do not depend on activations, so the stream runs ahead across
//     phase boundaries as far as the ring reaches;
//   * the consumer warps process the CTA's row groups of phase p exactly as
//     q2k_gemv_kernel does (q2k_core.cuh: same integer core, same ordered
//     float sum, same epilogues), so every output is bit-identical to the
//     separate launches; the finisher warp of each row group publishes it
//     with a release add on the phase's completion counter;
//   * before phase p+1, one consumer lane waits (acquire loads, bounded by
//     wall time and by the launch's abort word) until phase p's counter
//     reaches its group count; the CTA then quantizes its own activation
//     blocks from phase p's fp32 output (RMS-normalized when the phase asks)
//     with the standalone quantizer's helpers, so the Q8_K bits are the same;
//   * the last CTA to leave puts the counters back to zero for the next launch.
// All CTAs must be resident at once for the cross-CTA waits: the launch is
// cooperative (the runtime refuses a grid that cannot be co-resident).  Every
// wait is bounded; on expiry the kernel records kDevErrTimeout, sets the
// launch's abort word so the other CTAs stop waiting, and returns.
#include <stdio.h>

#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "q2k_core.cuh"
#include "q8k_device.cuh"
#include "runtime.h"

namespace smeai {

namespace {

constexpr uint64_t kTimeoutNs = 2000000000ull;  // 2 s
constexpr int kMaxWarps = 17;                    // producer + up to 16 consumers
constexpr uint32_t kProgramMagic = 0x51325047u;  // "Q2PG"

struct PhaseDev {
  const uint8_t* tiles;
  const void* x;       // Q8_K rows (contiguous) or fp32 rows
  float* y;
  const float* resid;
  int64_t n_rows;
  int64_t n_groups;
  int64_t ld_x;        // fp32 row stride (floats)
  int64_t ldy;
  int64_t ld_resid;
  int nb;
  int in_mode;
  int epi;
  int pad;
};

struct ProgParams {
  const PhaseDev* phases;
  int n_phases;
  int nb_max;
  float eps;
  int stages;
  int log2_stages;
  unsigned* ctr;    // [0, n_phases): row groups finished; [n_phases]: CTAs done; [n_phases + 1]: abort
  unsigned* err;
};

struct PSmem {
  uint8_t* ring;
  int4* qs;
  int* bs;
  float* d;
  float* rsum;
  float* terms;
  uint64_t* full;
  uint64_t* empty;
  uint64_t* grp;     // [2]
  uint64_t* tfree;   // [2]
  uint64_t* rms;     // [2]
  uint64_t* inready;
  uint64_t* done;
  unsigned* abort;
};

__host__ __device__ __forceinline__ size_t al16(size_t v) { return (v + 15) & ~(size_t)15; }

__host__ __device__ __forceinline__ size_t prog_fixed_bytes(int T, int nb_max) {
  return al16((size_t)T * nb_max * 256) + al16((size_t)T * nb_max * 32) + al16((size_t)T * nb_max * 4) +
         al16((size_t)T * (nb_max + 1) * 4) + al16((size_t)2 * T * nb_max * 128) + 8 * 8 + 16;
}
__host__ __device__ __forceinline__ size_t prog_smem_bytes(int T, int nb_max, int stages, int consumers) {
  return (size_t)stages * consumers * kTileBytes + prog_fixed_bytes(T, nb_max) + (size_t)stages * 16;
}

__device__ __forceinline__ PSmem pcarve(uint8_t* base, int T, int nb_max, int stages, int consumers) {
  PSmem m;
  size_t o = 0;
  m.ring = base;
  o += (size_t)stages * consumers * kTileBytes;
  m.qs = reinterpret_cast<int4*>(base + o);
  o += al16((size_t)T * nb_max * 256);
  m.bs = reinterpret_cast<int*>(base + o);
  o += al16((size_t)T * nb_max * 32);
  m.d = reinterpret_cast<float*>(base + o);
  o += al16((size_t)T * nb_max * 4);
  m.rsum = reinterpret_cast<float*>(base + o);
  o += al16((size_t)T * (nb_max + 1) * 4);
  m.terms = reinterpret_cast<float*>(base + o);
  o += al16((size_t)2 * T * nb_max * 128);
  m.full = reinterpret_cast<uint64_t*>(base + o);
  m.empty = m.full + stages;
  m.grp = m.empty + stages;
  m.tfree = m.grp + 2;
  m.rms = m.tfree + 2;
  m.inready = m.rms + 2;
  m.done = m.inready + 1;
  m.abort = reinterpret_cast<unsigned*>(m.done + 1);
  return m;
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_relaxed_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_gpu_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Wait until *ctr >= target; false on timeout or when the launch is aborted.
__device__ bool wait_count(const unsigned* ctr, unsigned target, const unsigned* abort_word) {
  if (ld_acquire_gpu(ctr) >= target) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    for (int k = 0; k < 32; ++k)
      if (ld_acquire_gpu(ctr) >= target) return true;
    if (ld_relaxed_gpu(abort_word)) return false;
    if (global_timer_ns() - t0 > kTimeoutNs) return false;
  }
}

__device__ __forceinline__ void fail(const ProgParams& P) {
  raise_device_error(P.err, kDevErrTimeout);
  atomicExch(P.ctr + P.n_phases + 1, 1u);
}

// Ordered sum of one row group's super-block terms and the phase's epilogue;
// the arithmetic of finish_group in q2k_gemv.cu.  Activations written earlier
// in this launch by other CTAs (the residual) are read through L2.
template <int T>
__device__ __forceinline__ void finish_group_prog(const float* terms, const PhaseDev& D, int64_t group, int lane) {
  const int nb = D.nb;
  if (D.epi == kEpiSiluMul) {
    if (lane < 16) {
      const int64_t orow = group * 16 + lane;
#pragma unroll 1
      for (int t = 0; t < T; ++t) {
        const float* tg = terms + (size_t)t * nb * 32 + 2 * lane;
        float g = 0.f, u = 0.f;
        for (int b = 0; b < nb; ++b) {
          g = __fadd_rn(g, tg[b * 32]);
          u = __fadd_rn(u, tg[b * 32 + 1]);
        }
        if (2 * orow < D.n_rows) {
          const float sg = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
          D.y[t * D.ldy + orow] = __fmul_rn(sg, u);
        }
      }
    }
  } else {
    const int64_t orow = group * 32 + lane;
#pragma unroll 1
    for (int t = 0; t < T; ++t) {
      const float* tr = terms + (size_t)t * nb * 32 + lane;
      float s = 0.f;
      int b = 0;
      for (; b + 8 <= nb; b += 8) {
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = tr[(b + k) * 32];
#pragma unroll
        for (int k = 0; k < 8; ++k) s = __fadd_rn(s, v[k]);
      }
      for (; b < nb; ++b) s = __fadd_rn(s, tr[b * 32]);
      if (orow < D.n_rows) {
        if (D.epi == kEpiResidual) s = __fadd_rn(__ldcg(D.resid + t * D.ld_resid + orow), s);
        D.y[t * D.ldy + orow] = s;
      }
    }
  }
}

// fp32 activation prologue: warp cw quantizes its super-blocks b = cw (mod W)
// of every token to Q8_K in shared memory (after an RMSNorm of each row for
// kInF32Rms), with the arithmetic of rms_q8k_quantize_kernel /
// q8k_quantize_kernel.  When the warp's blocks fit (T x blocks <= kRegItems)
// all its loads are issued at once and the values stay in registers between
// the RMS pass and the quantization.  Returns false after a timeout.
// (17 warps leave 96 registers a thread: 3 blocks of 8 values for one token,
// 2 for two, otherwise the values are re-read.)
template <int T>
__device__ __forceinline__ bool prologue_f32(const ProgParams& P, const PSmem& m, const ActSmem& act,
                                             const PhaseDev& D, int cw, int W, int lane, int& nrms) {
  const float* x = static_cast<const float*>(D.x);
  const int nb = D.nb;
  constexpr int kRegItems = T == 1 ? 3 : (T == 2 ? 2 : 1);
  const bool rms = D.in_mode == kInF32Rms;
  const int nbw = cw < nb ? (nb - cw + W - 1) / W : 0;  // blocks of this warp
  const int items = nbw * T;                            // item = i * T + t, block cw + i * W
  const bool inreg = items <= kRegItems;
  float v[kRegItems][8];
  if (inreg) {
#pragma unroll
    for (int it = 0; it < kRegItems; ++it)
      if (it < items) load8_cg(x + (it % T) * D.ld_x + (cw + (it / T) * W) * QK_K + lane * 8, v[it]);
  }
  if (rms) {
    if (inreg) {
#pragma unroll
      for (int it = 0; it < kRegItems; ++it)
        if (it < items) {
          const float s = block_sumsq_warp(v[it]);
          if (lane == 0) m.rsum[(it % T) * (nb + 1) + cw + (it / T) * W] = s;
        }
    } else {
      for (int it = 0; it < items; ++it) {
        float u[8];
        load8_cg(x + (it % T) * D.ld_x + (cw + (it / T) * W) * QK_K + lane * 8, u);
        const float s = block_sumsq_warp(u);
        if (lane == 0) m.rsum[(it % T) * (nb + 1) + cw + (it / T) * W] = s;
      }
    }
    mbar_arrive_warp(&m.rms[0]);
    if (cw == 0) {
      if (!mbar_wait_bounded(&m.rms[0], (unsigned)(nrms & 1), kTimeoutNs)) {
        fail(P);
        return false;
      }
      if (lane < T) {
        float* rs = m.rsum + lane * (nb + 1);
        float total = 0.f;
        for (int b = 0; b < nb; ++b) total = __fadd_rn(total, rs[b]);
        rs[nb] = rms_inv_from_sum(total, nb * QK_K, P.eps);
      }
      __syncwarp();
      mbar_arrive_warp(&m.rms[1]);
    }
    if (!mbar_wait_bounded(&m.rms[1], (unsigned)(nrms & 1), kTimeoutNs)) {
      fail(P);
      return false;
    }
    ++nrms;
  }
  if (inreg) {
#pragma unroll
    for (int it = 0; it < kRegItems; ++it)
      if (it < items) {
        const int t = it % T, b = cw + (it / T) * W;
        if (rms) {
          const float inv = m.rsum[t * (nb + 1) + nb];
#pragma unroll
          for (int k = 0; k < 8; ++k) v[it][k] = __fmul_rn(v[it][k], inv);
        }
        store_q8k_smem(q8k_quantize_lane(v[it]), act, t * nb + b);
      }
  } else {
    for (int it = 0; it < items; ++it) {
      const int t = it % T, b = cw + (it / T) * W;
      float u[8];
      load8_cg(x + t * D.ld_x + b * QK_K + lane * 8, u);
      if (rms) {
        const float inv = m.rsum[t * (nb + 1) + nb];
#pragma unroll
        for (int k = 0; k < 8; ++k) u[k] = __fmul_rn(u[k], inv);
      }
      store_q8k_smem(q8k_quantize_lane(u), act, t * nb + b);
    }
  }
  return true;
}

template <int T>
__global__ void __launch_bounds__(kMaxWarps * 32, 1) q2k_program_kernel(const ProgParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int W = (blockDim.x >> 5) - 1;
  const int S = P.stages, lgS = P.log2_stages, smask = S - 1;
  const int64_t C = gridDim.x, cta = blockIdx.x;
  const int stage_bytes = W * kTileBytes;
  const PSmem m = pcarve(smem, T, P.nb_max, S, W);
  unsigned* abort_word = P.ctr + P.n_phases + 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&m.full[s], 1);
      mbar_init(&m.empty[s], W);
    }
    mbar_init(&m.grp[0], W);
    mbar_init(&m.grp[1], W);
    mbar_init(&m.tfree[0], 1);
    mbar_init(&m.tfree[1], 1);
    mbar_init(&m.rms[0], W);
    mbar_init(&m.rms[1], 1);
    mbar_init(m.inready, 1);
    mbar_init(m.done, W);
    *m.abort = 0u;
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == 0) {
    // ---- producer: every phase's tiles of this CTA, in program order
    if (lane == 0) {
      int64_t i = 0;
      bool ok = true;
      for (int ph = 0; ph < P.n_phases && ok; ++ph) {
        const PhaseDev& D = P.phases[ph];
        const int nb = D.nb;
        const int64_t G = D.n_groups;
        const int64_t g0 = cta * G / C, g1 = (cta + 1) * G / C;
        const int nchunks = (nb + W - 1) / W;
        const uint8_t* src = D.tiles + g0 * nb * (int64_t)kTileBytes;
        for (int64_t j = 0; j < (g1 - g0) * nchunks; ++j, ++i) {
          const int s = (int)(i & smask);
          if (i >= S && !mbar_wait_bounded(&m.empty[s], (unsigned)(((i >> lgS) - 1) & 1), kTimeoutNs)) {
            ok = false;
            break;
          }
          const int64_t g = j / nchunks;
          const int c = (int)(j - g * nchunks);
          const int nblk = min(W, nb - c * W);
          mbar_arrive_expect_tx(&m.full[s], (unsigned)(nblk * kTileBytes));
          bulk_copy_g2s(m.ring + (size_t)s * stage_bytes, src + ((size_t)g * nb + (size_t)c * W) * kTileBytes,
                        (unsigned)(nblk * kTileBytes), &m.full[s]);
        }
      }
      if (!ok) {
        fail(P);
        for (int64_t j = (i > S ? i - S : 0); j < i; ++j)
          mbar_wait_bounded(&m.full[j & smask], (unsigned)((j >> lgS) & 1), kTimeoutNs);
      }
    }
    return;
  }

  // ---- consumers
  const int cw = warp - 1;
  const ActSmem act = {m.qs, m.bs, m.d};
  int64_t i = 0;  // ring stage, in step with the producer
  int jj = 0;     // row groups processed by this CTA (terms double buffer)
  int nwait = 0, nrms = 0;
  for (int ph = 0; ph < P.n_phases; ++ph) {
    const PhaseDev D = P.phases[ph];
    const int nb = D.nb;
    const int64_t g0 = cta * D.n_groups / C, g1 = (cta + 1) * D.n_groups / C;
    if (g0 == g1) continue;
    const int nchunks = (nb + W - 1) / W;

    // phase ph reads phase ph-1's complete output
    if (ph > 0) {
      if (cw == 0) {
        if (lane == 0 && !wait_count(P.ctr + ph - 1, (unsigned)P.phases[ph - 1].n_groups, abort_word)) {
          fail(P);
          *m.abort = 1u;
        }
        __syncwarp();
        mbar_arrive_warp(m.inready);
      }
      if (!mbar_wait_bounded(m.inready, (unsigned)(nwait & 1), kTimeoutNs)) {
        fail(P);
        return;
      }
      ++nwait;
      if (*reinterpret_cast<volatile unsigned*>(m.abort)) return;
    }

    // activation prologue: this warp's super-blocks b = cw (mod W)
    if (D.in_mode == kInQ8K) {
      const uint32_t* src = static_cast<const uint32_t*>(D.x);
      for (int b = cw; b < nb; b += W) {
#pragma unroll 1
        for (int t = 0; t < T; ++t)
          copy_q8k_smem(src + ((int64_t)t * nb + b) * Q8K_BLOCK_WORDS, act, t * nb + b, lane);
      }
    } else if (!prologue_f32<T>(P, m, act, D, cw, W, lane, nrms)) {
      return;
    }
    __syncwarp();

    // this CTA's row groups of the phase
    for (int64_t g = g0; g < g1; ++g, ++jj) {
      const int buf = jj & 1;
      float* terms = m.terms + (size_t)buf * T * P.nb_max * 32;
      if (jj >= 2 && !mbar_wait_bounded(&m.tfree[buf], (unsigned)(((jj >> 1) - 1) & 1), kTimeoutNs)) {
        fail(P);
        return;
      }
      const int64_t row = g * 32 + lane;
      for (int c = 0; c < nchunks; ++c, ++i) {
        const int s = (int)(i & smask);
        const int b = c * W + cw;
        if (!mbar_wait_bounded(&m.full[s], (unsigned)((i >> lgS) & 1), kTimeoutNs)) {
          fail(P);
          return;
        }
        if (b >= nb) {  // the group's last chunk is short
          mbar_arrive_warp(&m.empty[s]);
          continue;
        }
        const WBlock wb = load_wblock(m.ring + (size_t)s * stage_bytes + (size_t)cw * kTileBytes, lane);
        mbar_arrive_warp(&m.empty[s], wblock_dep(wb));
        block_terms<T, false>(wb, act, nb, b, terms, lane, row, D.n_rows, nullptr, nullptr);
      }
      mbar_arrive_warp(&m.grp[buf]);
      if (cw == (jj % W)) {
        if (!mbar_wait_bounded(&m.grp[buf], (unsigned)((jj >> 1) & 1), kTimeoutNs)) {
          fail(P);
          return;
        }
        finish_group_prog<T>(terms, D, g, lane);
        mbar_arrive_warp(&m.tfree[buf]);
        if (g == g1 - 1) {
          // The CTA's last row group of the phase: its grp wait followed every
          // earlier finisher's stores (each finisher arrives on the next
          // group's barrier after its own stores), so one fence and one
          // release add publish all of this CTA's rows of the phase.
          __syncwarp();
          __threadfence();
          if (lane == 0) red_release_gpu_add(P.ctr + ph, (unsigned)(g1 - g0));
        }
      }
    }
  }

  // ---- exit: the last CTA out resets the counters for the next launch
  mbar_arrive_warp(m.done);
  if (cw == 0) {
    const bool ok = mbar_wait_bounded(m.done, 0, kTimeoutNs);
    if (lane == 0) {
      if (!ok) {
        fail(P);
      } else if (!*reinterpret_cast<volatile unsigned*>(m.abort)) {
        unsigned* exit_ctr = P.ctr + P.n_phases;
        __threadfence();
        if (atomicAdd(exit_ctr, 1u) == (unsigned)(C - 1)) {
          for (int k = 0; k < P.n_phases; ++k) atomicExch(P.ctr + k, 0u);
          atomicExch(exit_ctr, 0u);
        }
      }
    }
  }
}

template <int T>
struct Kern {
  static void* ptr() { return reinterpret_cast<void*>(q2k_program_kernel<T>); }
};

void* kernel_for(int T) {
  switch (T) {
    case 1: return Kern<1>::ptr();
    case 2: return Kern<2>::ptr();
    case 4: return Kern<4>::ptr();
    case 8: return Kern<8>::ptr();
    default: return nullptr;
  }
}

}  // namespace

struct Q2KProgram {
  uint32_t magic = kProgramMagic;
  int n_phases = 0;
  int T = 0;
  int nb_max = 0;
  int consumers = 0;
  int stages = 0;
  int grid = 0;
  size_t smem = 0;
  float eps = 0.f;
  int device = 0;
  PhaseDev* d_phases = nullptr;
  unsigned* d_ctr = nullptr;
  int64_t counter_words = 0;
};

int q2k_program_create(const ProgPhase* phases, int n_phases, int n_cols, float eps, Q2KProgram** out) {
  if (!phases || !out || n_phases <= 0 || n_phases > (1 << 20)) {
    set_last_error("q2k_program: bad arguments");
    return kBadArgument;
  }
  *out = nullptr;
  if (!kernel_for(n_cols)) {
    set_last_error("q2k_program: n_cols must be 1, 2, 4 or 8 (got %d)", n_cols);
    return kBadArgument;
  }
  int dev = 0;
  SMEAI_CUDA_TRY(cudaGetDevice(&dev));
  std::vector<PhaseDev> hp((size_t)n_phases);
  int nb_max = 0;
  for (int p = 0; p < n_phases; ++p) {
    const ProgPhase& s = phases[p];
    if (!s.w || !s.w->tiles || !s.x || !s.y || s.w->device != dev) {
      set_last_error("q2k_program: phase %d: missing weight, input or output (or weight on another device)", p);
      return kBadArgument;
    }
    const Q2KWeight& w = *s.w;
    if (s.in_mode != kInQ8K && s.in_mode != kInF32 && s.in_mode != kInF32Rms) {
      set_last_error("q2k_program: phase %d: unknown input mode %d", p, s.in_mode);
      return kBadArgument;
    }
    if (s.in_mode == kInQ8K ? (reinterpret_cast<uintptr_t>(s.x) & 3) != 0
                            : ((reinterpret_cast<uintptr_t>(s.x) & 3) != 0 || s.ld_x < w.k)) {
      set_last_error("q2k_program: phase %d: input must be 4-byte aligned (fp32 rows with ld_x >= k)", p);
      return kBadArgument;
    }
    if (s.epi != kEpiStore && s.epi != kEpiResidual && s.epi != kEpiSiluMul) {
      set_last_error("q2k_program: phase %d: unknown epilogue %d", p, s.epi);
      return kBadArgument;
    }
    if (s.epi == kEpiResidual && !s.resid) {
      set_last_error("q2k_program: phase %d: residual epilogue needs a residual pointer", p);
      return kBadArgument;
    }
    if (s.epi == kEpiSiluMul && (w.n_rows & 1)) {
      set_last_error("q2k_program: phase %d: silu*mul needs interleaved (gate, up) row pairs", p);
      return kBadArgument;
    }
    const int64_t out_rows = s.epi == kEpiSiluMul ? w.n_rows / 2 : w.n_rows;
    if (s.ldy < out_rows || (s.epi == kEpiResidual && s.ld_resid < out_rows)) {
      set_last_error("q2k_program: phase %d: leading dimension smaller than the output rows", p);
      return kBadArgument;
    }
    PhaseDev& d = hp[(size_t)p];
    d.tiles = w.tiles;
    d.x = s.x;
    d.y = s.y;
    d.resid = s.resid;
    d.n_rows = w.n_rows;
    d.n_groups = w.n_groups;
    d.ld_x = s.ld_x;
    d.ldy = s.ldy;
    d.ld_resid = s.ld_resid;
    d.nb = w.nb;
    d.in_mode = s.in_mode;
    d.epi = s.epi;
    d.pad = 0;
    nb_max = nb_max > w.nb ? nb_max : w.nb;
  }
  // launch shape: 16 consumer warps (8 when the activation planes of 8 tokens
  // leave too little room) and the deepest power-of-two ring that fits
  int sms = 0;
  SMEAI_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  int optin = 0;
  SMEAI_CUDA_TRY(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  int consumers = 0, stages = 0;
  for (int W : {16, 8}) {
    for (int S = 8; S >= 2; S >>= 1)
      if (prog_smem_bytes(n_cols, nb_max, S, W) <= (size_t)optin) {
        stages = S;
        break;
      }
    if (stages) {
      consumers = W;
      break;
    }
  }
  if (!stages) {
    set_last_error("q2k_program: k=%d super-blocks x %d tokens does not fit in shared memory", nb_max, n_cols);
    return kBadArgument;
  }
  const size_t smem = prog_smem_bytes(n_cols, nb_max, stages, consumers);
  void* kern = kernel_for(n_cols);
  SMEAI_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 0;
  SMEAI_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, (consumers + 1) * 32, smem));
  if (per_sm < 1) {
    set_last_error("q2k_program: the kernel cannot be resident (smem %zu)", smem);
    return kUnsupported;
  }
  Q2KProgram* pr = new Q2KProgram();
  pr->n_phases = n_phases;
  pr->T = n_cols;
  pr->nb_max = nb_max;
  pr->consumers = consumers;
  pr->stages = stages;
  pr->grid = sms;  // one CTA per SM: every SM streams
  pr->smem = smem;
  pr->eps = eps;
  pr->device = dev;
  pr->counter_words = (int64_t)n_phases + 2;
  if (cudaMalloc(&pr->d_phases, sizeof(PhaseDev) * (size_t)n_phases) != cudaSuccess ||
      cudaMalloc(&pr->d_ctr, sizeof(unsigned) * (size_t)pr->counter_words) != cudaSuccess) {
    cudaGetLastError();
    q2k_program_free(pr);
    set_last_error("q2k_program: cudaMalloc failed");
    return kAllocFailed;
  }
  if (cudaMemcpy(pr->d_phases, hp.data(), sizeof(PhaseDev) * (size_t)n_phases, cudaMemcpyHostToDevice) !=
          cudaSuccess ||
      cudaMemset(pr->d_ctr, 0, sizeof(unsigned) * (size_t)pr->counter_words) != cudaSuccess) {
    const cudaError_t e = cudaGetLastError();
    q2k_program_free(pr);
    set_last_error("q2k_program: %s", cudaGetErrorString(e));
    return kCudaError;
  }
  *out = pr;
  return kOk;
}

int q2k_program_run(Q2KProgram* pr, cudaStream_t stream) {
  if (!pr || pr->magic != kProgramMagic) {
    set_last_error("q2k_program_run: not a program handle");
    return kBadArgument;
  }
  ProgParams P;
  P.phases = pr->d_phases;
  P.n_phases = pr->n_phases;
  P.nb_max = pr->nb_max;
  P.eps = pr->eps;
  P.stages = pr->stages;
  P.log2_stages = 31 - __builtin_clz((unsigned)pr->stages);
  P.ctr = pr->d_ctr;
  P.err = device_error_ptr();
  if (!P.err) {
    set_last_error("q2k_program_run: device error word unavailable");
    return kCudaError;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)pr->grid);
  cfg.blockDim = dim3((unsigned)((pr->consumers + 1) * 32));
  cfg.dynamicSmemBytes = pr->smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  switch (pr->T) {
    case 1: e = cudaLaunchKernelEx(&cfg, q2k_program_kernel<1>, P); break;
    case 2: e = cudaLaunchKernelEx(&cfg, q2k_program_kernel<2>, P); break;
    case 4: e = cudaLaunchKernelEx(&cfg, q2k_program_kernel<4>, P); break;
    case 8: e = cudaLaunchKernelEx(&cfg, q2k_program_kernel<8>, P); break;
    default: e = cudaErrorInvalidValue;
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_last_error("q2k_program_run: launch failed: %s", cudaGetErrorString(e));
    return kCudaError;
  }
  return kOk;
}

int q2k_program_reset(Q2KProgram* pr, cudaStream_t stream) {
  if (!pr || pr->magic != kProgramMagic) {
    set_last_error("q2k_program_reset: not a program handle");
    return kBadArgument;
  }
  SMEAI_CUDA_TRY(cudaMemsetAsync(pr->d_ctr, 0, sizeof(unsigned) * (size_t)pr->counter_words, stream));
  return kOk;
}

void q2k_program_free(Q2KProgram* pr) {
  if (!pr || pr->magic != kProgramMagic) return;
  if (pr->d_phases) cudaFree(pr->d_phases);
  if (pr->d_ctr) cudaFree(pr->d_ctr);
  pr->magic = 0;
  delete pr;
}

void q2k_program_shape(const Q2KProgram* pr, int* grid, int* consumers, int* stages, size_t* smem) {
  if (grid) *grid = pr->grid;
  if (consumers) *consumers = pr->consumers;
  if (stages) *stages = pr->stages;
  if (smem) *smem = pr->smem;
}

}  // namespace smeai
