// q2k_program.cu -- a decode step (a chain of dependent Q2_K GEMVs) as ONE
// persistent cooperative kernel.
//
// Batch-1 decode of a Llama-shape stack is ~129 GEMVs (qkv, o, gate/up, down
// per layer, then lm_head), each reading the complete output of an earlier
// one (after an RMSNorm, a silu*mul, or a plain re-quantization to Q8_K).  As
// separate launches every link costs a grid drain, a launch and a refill of
// the weight stream.  Here one CTA per SM runs the whole chain:
//   * warp 0, lane 0 (producer) streams this CTA's weight tiles of EVERY
//     phase, in program order, into a shared-memory ring with cp.async.bulk.
//     Weights do not depend on activations, so the stream runs ahead across
//     phase boundaries as far as the ring reaches;
//   * the consumer warps process the CTA's row groups of each phase exactly
//     as q2k_gemv_kernel does (q2k_core.cuh: same integer core, same ordered
//     float sum, same epilogues), so every output is bit-identical to the
//     separate launches;
//   * the finisher warp of each row group writes the outputs and, when a
//     later phase reads them through an RMSNorm, the group's sum of squares
//     (its 32 rows folded in the fixed order of the CPU restatement); the
//     CTA's last finisher of a phase publishes its rows with one release add
//     on the phase's completion counter;
//   * before phase p, one lane of the CTA waits (acquire loads, bounded by
//     wall time and by the launch's abort word) until phase p-1's counter
//     reaches its group count, while the other warps sleep on an mbarrier;
//     meanwhile its warp copies phase p's descriptor into shared memory, so
//     no field is read through the (then stale) L1 on the critical path;
//     then every warp issues one round of loads -- its own activation blocks,
//     the producer's group sums (an RMSNorm input: each warp folds them to
//     the same 1/rms, no cross-warp barrier), the residual of the groups it
//     will finish -- and quantizes its blocks to Q8_K in shared memory with
//     the standalone quantizer's helpers (same bits);
//   * activation slots in shared memory belong to one warp in every phase, so
//     a warp that runs ahead into the next phase cannot touch a slower warp's
//     operands;
//   * the last CTA to leave puts the counters back to zero for the next launch.
// All CTAs must be resident at once for the cross-CTA waits: the launch is
// cooperative (the runtime refuses a grid that cannot be co-resident).  Every
// wait is bounded; on expiry the kernel records kDevErrTimeout, sets the
// launch's abort word so the other CTAs stop waiting, and returns.
#include <stdio.h>
#include <stdlib.h>

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
  const void* x;            // Q8_K rows, or fp32 rows
  const float* x_part;      // group sums of squares of the input rows (RMS input from a phase), or null
  float* y;
  float* y_part;            // group sums of squares of the output (a later phase's RMS input), or null
  const float* resid;
  int64_t n_rows;
  int64_t n_groups;
  int64_t ld_x;             // token stride of x (floats)
  int64_t ld_xpart;         // token stride of x_part
  int64_t ldy;
  int64_t n_part;           // token stride of y_part (32-row groups of the output)
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
  int l2_ahead;     // ring stages prefetched into L2 ahead of the ring loads
  unsigned* ctr;    // [0, n_phases): row groups finished; [n_phases]: CTAs done; [n_phases + 1]: abort
  unsigned* err;
};

struct PSmem {
  uint8_t* ring;
  int4* qs;
  int* bs;
  float* d;
  float* terms;
  PhaseDev* pd;       // [2] descriptors of the CTA's current and previous phase
  uint64_t* full;
  uint64_t* empty;
  uint64_t* grp;      // [2] all consumer warps wrote a row group's terms
  uint64_t* tfree;    // [2] the finisher has consumed them
  uint64_t* done;
  uint64_t* inready;  // the CTA's poller saw the previous phase complete
  uint64_t* invready; // the poller has put 1/rms of every token in inv[]
  unsigned* gate_fail;
  float* inv;         // [8]
};

__host__ __device__ __forceinline__ size_t al16(size_t v) { return (v + 15) & ~(size_t)15; }

// Q8_K activation slot of warp cw's i-th super-block (b = cw + i * W) and
// token t.  Slots belong to one warp in every phase: a warp that has moved
// on to the next phase's prologue cannot overwrite an activation a slower
// warp of its CTA still reads (the slot would otherwise move with k).
__device__ __forceinline__ int act_slot(int cw, int W, int T, int i, int t) { return cw + W * (t + T * i); }
// slots to allocate: W warps x T tokens x the most blocks one warp gets
__host__ __device__ __forceinline__ size_t act_slots(int T, int nb_max, int W) {
  return (size_t)W * T * ((nb_max + W - 1) / W);
}

__host__ __device__ __forceinline__ size_t prog_fixed_bytes(int T, int nb_max, int W) {
  const size_t slots = act_slots(T, nb_max, W);
  return al16(slots * 256) + al16(slots * 32) + al16(slots * 4) + al16((size_t)2 * T * nb_max * 128) +
         al16(2 * sizeof(PhaseDev)) + 8 * 7 + 16 + 32;
}
__host__ __device__ __forceinline__ size_t prog_smem_bytes(int T, int nb_max, int stages, int consumers) {
  return (size_t)stages * consumers * kTileBytes + prog_fixed_bytes(T, nb_max, consumers) + (size_t)stages * 16;
}

__device__ __forceinline__ PSmem pcarve(uint8_t* base, int T, int nb_max, int stages, int consumers) {
  PSmem m;
  size_t o = 0;
  const size_t slots = act_slots(T, nb_max, consumers);
  m.ring = base;
  o += (size_t)stages * consumers * kTileBytes;
  m.qs = reinterpret_cast<int4*>(base + o);
  o += al16(slots * 256);
  m.bs = reinterpret_cast<int*>(base + o);
  o += al16(slots * 32);
  m.d = reinterpret_cast<float*>(base + o);
  o += al16(slots * 4);
  m.terms = reinterpret_cast<float*>(base + o);
  o += al16((size_t)2 * T * nb_max * 128);
  m.pd = reinterpret_cast<PhaseDev*>(base + o);
  o += al16(2 * sizeof(PhaseDev));
  m.full = reinterpret_cast<uint64_t*>(base + o);
  m.empty = m.full + stages;
  m.grp = m.empty + stages;
  m.tfree = m.grp + 2;
  m.done = m.tfree + 2;
  m.inready = m.done + 1;
  m.invready = m.inready + 1;
  m.gate_fail = reinterpret_cast<unsigned*>(m.invready + 1);
  m.inv = reinterpret_cast<float*>(m.gate_fail + 4);
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

// RMSNorm total of one token's input row of nb super-blocks computed from the
// row itself (an input not produced inside the program), in the fixed order:
// each lane folds its own 32-value groups, then the lanes are folded.
__device__ __forceinline__ float rms_total_plain(const float* row, int nb) {
  const int lane = threadIdx.x & 31;
  float acc = 0.f;
  for (int g = lane; g < nb * 8; g += 32) {
    const float* gp = row + (int64_t)g * 32;
    float a[32];
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const float4 q = __ldcg(reinterpret_cast<const float4*>(gp + i));
      a[i] = __fmul_rn(q.x, q.x);
      a[i + 1] = __fmul_rn(q.y, q.y);
      a[i + 2] = __fmul_rn(q.z, q.z);
      a[i + 3] = __fmul_rn(q.w, q.w);
    }
#pragma unroll
    for (int width = 16; width >= 1; width >>= 1)
#pragma unroll
      for (int l = 0; l < width; ++l) a[l] = __fadd_rn(a[l], a[l + width]);
    acc = __fadd_rn(acc, a[0]);
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
  return acc;
}

// fp32 activation prologue: warp cw quantizes its super-blocks b = cw (mod W)
// of every token to Q8_K in shared memory (after an RMSNorm of each row for
// kInF32Rms), with the arithmetic of rms_q8k_quantize_kernel /
// q8k_quantize_kernel.  The block loads (and, by the caller, the residual
// loads) go out first; for an RMSNorm input warp 0 alone then reads the
// producer's group sums -- one read per CTA, not one per warp, of lines every
// CTA wants -- folds 1/rms of every token into inv[] and releases the other
// warps.  When the warp's blocks fit (T x blocks <= kRegItems) they are all
// in flight at once.  (17 warps leave 96 registers a thread: 3 blocks of 8
// values for one token, 2 for two, otherwise one block at a time.)
template <int T>
__device__ __forceinline__ bool prologue_f32(const ProgParams& P, const PSmem& m, const ActSmem& act,
                                             const PhaseDev& D, int cw, int W, int lane, int& nrms) {
  const int nb = D.nb;
  constexpr int kRegItems = T == 1 ? 3 : (T == 2 ? 2 : 1);
  const bool rms = D.in_mode == kInF32Rms;
  const float* x = static_cast<const float*>(D.x);
  const int nbw = cw < nb ? (nb - cw + W - 1) / W : 0;  // blocks of this warp
  const int items = nbw * T;                            // item = i * T + t, block cw + i * W
  const bool inreg = items <= kRegItems;
  float v[kRegItems][8];
  if (inreg) {
#pragma unroll
    for (int it = 0; it < kRegItems; ++it)
      if (it < items) load8_cg(x + (it % T) * D.ld_x + (cw + (it / T) * W) * QK_K + lane * 8, v[it]);
  }
  float inv[T];
  if (rms) {
    if (cw == 0) {
#pragma unroll 1
      for (int t = 0; t < T; ++t) {
        const float total = D.x_part ? rms_fold_groups_cg(D.x_part + t * D.ld_xpart, nb * 8)
                                     : rms_total_plain(x + t * D.ld_x, nb);
        if (lane == 0) m.inv[t] = rms_inv_from_sum(total, nb * QK_K, P.eps);
      }
      mbar_arrive_warp(m.invready);
    }
    if (!mbar_wait_bounded(m.invready, (unsigned)(nrms & 1), kTimeoutNs)) {
      fail(P);
      return false;
    }
    ++nrms;
#pragma unroll
    for (int t = 0; t < T; ++t) inv[t] = m.inv[t];
  }
  auto quant = [&](int it, float (&u)[8]) {
    const int t = it % T;
    if (rms) {
#pragma unroll
      for (int k = 0; k < 8; ++k) u[k] = __fmul_rn(u[k], inv[t]);
    }
    store_q8k_smem(q8k_quantize_lane(u), act, act_slot(cw, W, T, it / T, t));
  };
  if (inreg) {
#pragma unroll
    for (int it = 0; it < kRegItems; ++it)
      if (it < items) quant(it, v[it]);
  } else {
    for (int it = 0; it < items; ++it) {
      float u[8];
      load8_cg(x + (it % T) * D.ld_x + (cw + (it / T) * W) * QK_K + lane * 8, u);
      quant(it, u);
    }
  }
  return true;
}

// Residual of one row group, T tokens, this lane's row.
template <int T>
__device__ __forceinline__ void load_resid(const PhaseDev& D, int64_t group, int lane, float (&r)[T]) {
  const int64_t orow = group * 32 + lane;
#pragma unroll
  for (int t = 0; t < T; ++t) r[t] = orow < D.n_rows ? __ldcg(D.resid + t * D.ld_resid + orow) : 0.f;
}

// Ordered sum of one row group's super-block terms and the phase's epilogue
// (the arithmetic of finish_group in q2k_gemv.cu); then the group sums of
// squares when a later phase reads this output through an RMSNorm.
template <int T>
__device__ __forceinline__ void finish_group_prog(const float* terms, const PhaseDev& D, int64_t group, int lane,
                                                  const float (&r)[T]) {
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
#pragma unroll
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
      const bool live = orow < D.n_rows;
      if (live) {
        if (D.epi == kEpiResidual) s = __fadd_rn(r[t], s);
        D.y[t * D.ldy + orow] = s;
      }
      if (D.y_part) {
        const float ss = group_sumsq_lane(live ? s : 0.f);
        if (lane == 0) D.y_part[t * D.n_part + group] = ss;
      }
    }
  }
}

// Walks this CTA's ring stages in program order: phase, row group, chunk of
// up to W consecutive super-blocks (incrementally: the producer thread does
// no division per stage).
struct StageCursor {
  int ph = 0, n_phases = 0;
  int64_t g = 0, ng = 0;  // row group within the CTA's range, groups in the range
  int c = 0, nchunks = 0, nb = 0, W = 0;
  const uint8_t* base = nullptr;
  int64_t index = 0;      // stages walked so far (the ring's running index)

  __device__ void load_phase(const ProgParams& P, int64_t cta, int64_t C) {
    for (; ph < n_phases; ++ph) {
      const PhaseDev& D = P.phases[ph];
      const int64_t g0 = cta * D.n_groups / C, g1 = (cta + 1) * D.n_groups / C;
      nb = D.nb;
      nchunks = (nb + W - 1) / W;
      ng = g1 - g0;
      base = D.tiles + g0 * nb * (int64_t)kTileBytes;
      g = 0;
      c = 0;
      if (ng > 0) return;
    }
  }
  __device__ void start(const ProgParams& P, int64_t cta, int64_t C, int w) {
    W = w;
    n_phases = P.n_phases;
    ph = 0;
    index = 0;
    load_phase(P, cta, C);
  }
  __device__ bool valid() const { return ph < n_phases; }
  __device__ const uint8_t* src() const { return base + ((size_t)g * nb + (size_t)c * W) * kTileBytes; }
  __device__ unsigned bytes() const { return (unsigned)(min(W, nb - c * W) * kTileBytes); }
  __device__ void advance(const ProgParams& P, int64_t cta, int64_t C) {
    ++index;
    if (++c < nchunks) return;
    c = 0;
    if (++g < ng) return;
    ++ph;
    load_phase(P, cta, C);
  }
};

template <int T>
__global__ void __launch_bounds__(kMaxWarps * 32, 1) q2k_program_kernel(const ProgParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int W = (blockDim.x >> 5) - 1;
  const int S = P.stages, lgS = P.log2_stages, smask = S - 1;
  const int64_t C = gridDim.x, cta = blockIdx.x;
  const int stage_bytes = W * kTileBytes;
  const PSmem m = pcarve(smem, T, P.nb_max, S, W);
  const unsigned* abort_word = P.ctr + P.n_phases + 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&m.full[s], 1);
      mbar_init(&m.empty[s], W);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&m.grp[b], W);
      mbar_init(&m.tfree[b], 1);
    }
    mbar_init(m.done, W);
    mbar_init(m.inready, 1);
    mbar_init(m.invready, 1);
    *m.gate_fail = 0u;
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == 0) {
    // ---- producer: every phase's tiles of this CTA, in program order, into
    // the ring; and, l2_ahead stages further on, prefetches of the same tiles
    // into L2, so HBM keeps streaming while the consumers sit at a phase
    // boundary with the ring full (the ring loads then hit L2)
    if (lane == 0) {
      StageCursor issue, pref;
      issue.start(P, cta, C, W);
      pref.start(P, cta, C, W);
      bool ok = true;
      int64_t i = 0;
      for (; issue.valid(); issue.advance(P, cta, C), ++i) {
        while (P.l2_ahead > 0 && pref.valid() && pref.index < i + P.l2_ahead) {
          bulk_prefetch_l2(pref.src(), pref.bytes());
          pref.advance(P, cta, C);
        }
        const int s = (int)(i & smask);
        if (i >= S && !mbar_wait_bounded(&m.empty[s], (unsigned)(((i >> lgS) - 1) & 1), kTimeoutNs)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&m.full[s], issue.bytes());
        bulk_copy_g2s(m.ring + (size_t)s * stage_bytes, issue.src(), issue.bytes(), &m.full[s]);
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
  int jj = 0;     // row groups processed by this CTA (terms double buffer, finisher rota)
  int nwait = 0;  // phases this CTA took part in (inready parity, descriptor slot)
  int nrms = 0;   // RMSNorm inputs read (invready parity)
  for (int ph = 0; ph < P.n_phases; ++ph) {
    const int nb = P.phases[ph].nb;
    const int64_t ngr = P.phases[ph].n_groups;
    const int64_t g0 = cta * ngr / C, g1 = (cta + 1) * ngr / C;
    if (g0 == g1) continue;
    const int nchunks = (nb + W - 1) / W;

    // phase ph reads phase ph-1's complete output (and, through it, every
    // earlier phase's): one lane waits, the other warps sleep on inready.
    // Meanwhile warp 0 brings the phase's descriptor into shared memory (the
    // gate's acquire leaves this SM's L1 stale, so reading it in place would
    // cost an L2 round trip before the first activation load and again in
    // every finisher).  The slot alternates per phase this CTA takes part
    // in: the slot written here was last read in the CTA's phase before the
    // previous one, which ended before the previous gate opened.
    PhaseDev& Ds = m.pd[nwait & 1];
    if (cw == 0) {
      constexpr int kWords = (int)(sizeof(PhaseDev) / 4);
      static_assert(sizeof(PhaseDev) % 4 == 0 && kWords <= 32, "phase descriptor copy");
      if (lane < kWords)
        reinterpret_cast<uint32_t*>(&Ds)[lane] = __ldcg(reinterpret_cast<const uint32_t*>(P.phases + ph) + lane);
      if (ph > 0 && lane == 0 && !wait_count(P.ctr + ph - 1, (unsigned)P.phases[ph - 1].n_groups, abort_word)) {
        fail(P);
        *m.gate_fail = 1u;
      }
      mbar_arrive_warp(m.inready);
    }
    if (!mbar_wait_bounded(m.inready, (unsigned)(nwait & 1), kTimeoutNs)) {
      fail(P);
      return;
    }
    ++nwait;
    if (*reinterpret_cast<volatile unsigned*>(m.gate_fail)) return;
    const PhaseDev& D = Ds;

    // one round of loads: the residual of the first row group this warp will
    // finish, and the activation prologue (this warp's super-blocks)
    const int64_t jfirst = ((cw - jj) % W + W) % W;  // local index of that group
    float res[T];
#pragma unroll
    for (int t = 0; t < T; ++t) res[t] = 0.f;
    if (D.epi == kEpiResidual && jfirst < g1 - g0) load_resid<T>(D, g0 + jfirst, lane, res);
    if (D.in_mode == kInQ8K) {
      const uint32_t* src = static_cast<const uint32_t*>(D.x);
      for (int b = cw; b < nb; b += W) {
#pragma unroll 1
        for (int t = 0; t < T; ++t)
          copy_q8k_smem(src + ((int64_t)t * nb + b) * Q8K_BLOCK_WORDS, act, act_slot(cw, W, T, b / W, t), lane);
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
        block_terms<T, false>(wb, act, act_slot(cw, W, T, c, 0), W, nb, b, terms, lane, row, D.n_rows, nullptr,
                              nullptr);
      }
      mbar_arrive_warp(&m.grp[buf]);
      if (cw == (jj % W)) {
        if (!mbar_wait_bounded(&m.grp[buf], (unsigned)((jj >> 1) & 1), kTimeoutNs)) {
          fail(P);
          return;
        }
        if (D.epi == kEpiResidual && g != g0 + jfirst) load_resid<T>(D, g, lane, res);
        finish_group_prog<T>(terms, D, g, lane, res);
        mbar_arrive_warp(&m.tfree[buf]);
        if (g == g1 - 1) {
          // The CTA's last row group of the phase: its grp wait followed every
          // earlier finisher's stores (each finisher arrives on the next
          // group's barrier after its own), and __syncwarp orders this warp's
          // lanes, so one release add publishes all of the CTA's rows.
          __syncwarp();
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
      } else if (!ld_relaxed_gpu(abort_word)) {
        unsigned* exit_ctr = P.ctr + P.n_phases;
        if (atomicAdd(exit_ctr, 1u) == (unsigned)(C - 1)) {
          for (int k = 0; k < P.n_phases; ++k) atomicExch(P.ctr + k, 0u);
          atomicExch(exit_ctr, 0u);
        }
      }
    }
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
  float* d_parts = nullptr;  // every group-sum array
  size_t parts_bytes = 0;
  int l2_ahead = 0;
};

namespace {

struct Range {
  uintptr_t lo = 0, hi = 0;  // bytes [lo, hi)
  bool overlaps(const Range& o) const { return lo < o.hi && o.lo < hi; }
};

Range rows_range(const void* base, int64_t ld, int64_t cols, int64_t len, size_t elem) {
  Range r;
  r.lo = reinterpret_cast<uintptr_t>(base);
  r.hi = r.lo + (size_t)((cols - 1) * ld + len) * elem;
  return r;
}

}  // namespace

int q2k_program_create(const ProgPhase* phases, int n_phases, int n_cols, float eps, Q2KProgram** out) {
  if (!phases || !out || n_phases <= 0 || n_phases > (1 << 20)) {
    set_last_error("q2k_program: bad arguments");
    return kBadArgument;
  }
  *out = nullptr;
  const int T = n_cols;
  if (T != 1 && T != 2 && T != 4 && T != 8) {
    set_last_error("q2k_program: n_cols must be 1, 2, 4 or 8 (got %d)", n_cols);
    return kBadArgument;
  }
  int dev = 0;
  SMEAI_CUDA_TRY(cudaGetDevice(&dev));
  const int n = n_phases;
  std::vector<int64_t> out_rows((size_t)n);
  std::vector<Range> yr((size_t)n);
  std::vector<int> x_src((size_t)n, -1);
  std::vector<int64_t> x_r0((size_t)n, 0);
  std::vector<char> need_part((size_t)n, 0);
  int nb_max = 0;
  for (int p = 0; p < n; ++p) {
    const ProgPhase& s = phases[p];
    if (!s.w || !s.w->tiles || !s.x || !s.y || s.w->device != dev || s.w->fmt != kFmtQ2K) {
      set_last_error("q2k_program: phase %d: missing weight, input or output (or a weight on another device, or not Q2_K)", p);
      return kBadArgument;
    }
    const Q2KWeight& w = *s.w;
    if (s.in_mode != kInQ8K && s.in_mode != kInF32 && s.in_mode != kInF32Rms) {
      set_last_error("q2k_program: phase %d: unknown input mode %d", p, s.in_mode);
      return kBadArgument;
    }
    if (s.in_mode == kInQ8K ? (reinterpret_cast<uintptr_t>(s.x) & 3) != 0
                            : ((reinterpret_cast<uintptr_t>(s.x) & 15) != 0 || s.ld_x < w.k || (s.ld_x & 3))) {
      set_last_error("q2k_program: phase %d: Q8_K input must be 4-byte aligned; fp32 input 16-byte aligned with "
                     "ld_x >= k and a multiple of 4", p);
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
    out_rows[(size_t)p] = s.epi == kEpiSiluMul ? w.n_rows / 2 : w.n_rows;
    if (s.ldy < out_rows[(size_t)p] || (s.epi == kEpiResidual && s.ld_resid < out_rows[(size_t)p])) {
      set_last_error("q2k_program: phase %d: leading dimension smaller than the output rows", p);
      return kBadArgument;
    }
    // An RMSNorm input that an earlier phase wrote (the latest one whose
    // output overlaps it) takes its sum of squares from that phase's group
    // sums: the rows must be a 32-row aligned slice of a store or residual
    // output with the same token stride.
    if (s.in_mode == kInF32Rms) {
      const Range want = rows_range(s.x, s.ld_x, T, w.k, 4);
      for (int q = p - 1; q >= 0; --q) {
        if (!yr[(size_t)q].overlaps(want)) continue;
        const ProgPhase& src = phases[q];
        const intptr_t off = reinterpret_cast<intptr_t>(s.x) - reinterpret_cast<intptr_t>(src.y);
        if (s.ld_x != src.ldy || off < 0 || off % 128 || off / 4 + w.k > out_rows[(size_t)q] ||
            src.epi == kEpiSiluMul) {
          set_last_error("q2k_program: phase %d: an RMSNorm input written by phase %d must be a 32-row aligned "
                         "slice of its store or residual output with the same row stride", p, q);
          return kBadArgument;
        }
        x_src[(size_t)p] = q;
        x_r0[(size_t)p] = off / 4;
        need_part[(size_t)q] = 1;
        break;
      }
    }
    yr[(size_t)p] = rows_range(s.y, s.ldy, T, out_rows[(size_t)p], 4);
    nb_max = nb_max > w.nb ? nb_max : w.nb;
  }
  std::vector<size_t> part_off((size_t)n, 0);
  std::vector<int64_t> n_part((size_t)n, 0);
  size_t parts = 0;
  for (int p = 0; p < n; ++p) {
    n_part[(size_t)p] = (out_rows[(size_t)p] + 31) / 32;
    if (need_part[(size_t)p]) {
      part_off[(size_t)p] = parts;
      parts += al16((size_t)T * n_part[(size_t)p] * 4);
    }
  }
  // launch shape: 16 consumer warps (8 when the activation planes of 8 tokens
  // leave too little room) and the deepest power-of-two ring that fits
  int sms = 0, optin = 0;
  SMEAI_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  SMEAI_CUDA_TRY(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  int consumers = 0, stages = 0;
  for (int W : {16, 8}) {
    for (int S = 8; S >= 2; S >>= 1)
      if (prog_smem_bytes(T, nb_max, S, W) <= (size_t)optin) {
        stages = S;
        break;
      }
    if (stages) {
      consumers = W;
      break;
    }
  }
  if (!stages) {
    set_last_error("q2k_program: k=%d super-blocks x %d tokens does not fit in shared memory", nb_max, T);
    return kBadArgument;
  }
  const size_t smem = prog_smem_bytes(T, nb_max, stages, consumers);
  void* kern = nullptr;
  switch (T) {
    case 1: kern = reinterpret_cast<void*>(q2k_program_kernel<1>); break;
    case 2: kern = reinterpret_cast<void*>(q2k_program_kernel<2>); break;
    case 4: kern = reinterpret_cast<void*>(q2k_program_kernel<4>); break;
    default: kern = reinterpret_cast<void*>(q2k_program_kernel<8>); break;
  }
  SMEAI_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 0;
  SMEAI_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, (consumers + 1) * 32, smem));
  if (per_sm < 1) {
    set_last_error("q2k_program: the kernel cannot be resident (smem %zu)", smem);
    return kUnsupported;
  }
  Q2KProgram* pr = new Q2KProgram();
  pr->n_phases = n;
  pr->T = T;
  pr->nb_max = nb_max;
  pr->consumers = consumers;
  pr->stages = stages;
  pr->grid = sms;  // one CTA per SM: every SM streams
  pr->smem = smem;
  pr->eps = eps;
  pr->device = dev;
  pr->counter_words = (int64_t)n + 2;
  pr->parts_bytes = parts;
  // L2 prefetch of ring stages ahead of the ring loads: off by default
  // (measured on B200, 7B-shape decode: 0.965 ms per token without, 0.985 ms
  // with 8 stages ahead -- the ring alone keeps the stream fed, and the extra
  // requests cost more than they hide).  SMEAI_PROGRAM_L2_AHEAD=n sets it.
  pr->l2_ahead = 0;
  if (const char* e = getenv("SMEAI_PROGRAM_L2_AHEAD")) pr->l2_ahead = atoi(e) < 0 ? 0 : atoi(e);
  if (cudaMalloc(&pr->d_phases, sizeof(PhaseDev) * (size_t)n) != cudaSuccess ||
      cudaMalloc(&pr->d_ctr, sizeof(unsigned) * (size_t)pr->counter_words) != cudaSuccess ||
      (parts && cudaMalloc(&pr->d_parts, parts) != cudaSuccess)) {
    cudaGetLastError();
    q2k_program_free(pr);
    set_last_error("q2k_program: cudaMalloc failed");
    return kAllocFailed;
  }
  uint8_t* pb = reinterpret_cast<uint8_t*>(pr->d_parts);
  std::vector<PhaseDev> hp((size_t)n);
  for (int p = 0; p < n; ++p) {
    const ProgPhase& s = phases[p];
    const Q2KWeight& w = *s.w;
    PhaseDev& d = hp[(size_t)p];
    d = PhaseDev{};
    d.tiles = w.tiles;
    d.x = s.x;
    d.y = s.y;
    d.resid = s.resid;
    d.n_rows = w.n_rows;
    d.n_groups = w.n_groups;
    d.ld_x = s.ld_x;
    d.ldy = s.ldy;
    d.n_part = n_part[(size_t)p];
    d.ld_resid = s.ld_resid;
    d.nb = w.nb;
    d.in_mode = s.in_mode;
    d.epi = s.epi;
    if (need_part[(size_t)p]) d.y_part = reinterpret_cast<float*>(pb + part_off[(size_t)p]);
    const int q = x_src[(size_t)p];
    if (q >= 0) {
      d.x_part = reinterpret_cast<const float*>(pb + part_off[(size_t)q]) + x_r0[(size_t)p] / 32;
      d.ld_xpart = n_part[(size_t)q];
    }
  }
  if (cudaMemcpy(pr->d_phases, hp.data(), sizeof(PhaseDev) * (size_t)n, cudaMemcpyHostToDevice) != cudaSuccess ||
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
  P.l2_ahead = pr->l2_ahead;
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
  if (pr->d_parts) cudaFree(pr->d_parts);
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
