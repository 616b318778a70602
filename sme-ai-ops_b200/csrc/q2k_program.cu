// q2k_program.cu -- a decode step (a chain of dependent Q2_K GEMVs) as ONE
// persistent cooperative kernel whose phases hand their activations to one
// another through tagged words instead of grid-wide barriers.
//
// Batch-1 decode of a Llama-shape stack is ~129 GEMVs (qkv, o, gate/up, down
// per layer, then lm_head), each reading the complete output of an earlier
// one (after an RMSNorm, a silu*mul, or a plain re-quantization to Q8_K).
// One CTA per SM runs the whole chain:
//   * warp 0, lane 0 (producer) streams this CTA's weight tiles of EVERY
//     phase, in program order, into a shared-memory ring with cp.async.bulk.
//     Weights do not depend on activations, so the stream runs ahead across
//     phase boundaries as far as the ring reaches;
//   * row groups are dealt to CTAs round-robin (CTA c takes every C-th group),
//     so a phase's outputs complete in rounds from its first rows to its last
//     and the next phase's early input blocks are ready before the phase
//     ends; the dealing continues from phase to phase, so the CTAs that take
//     one phase's extra groups are not the ones that take the next one's;
//   * the consumer warps process the CTA's row groups of each phase exactly
//     as q2k_gemv_kernel does (q2k_core.cuh: same integer core, same ordered
//     float sum, same epilogues), so every output is bit-identical to the
//     separate launches;
//   * HANDOFF.  Besides the caller-visible fp32 output, every finished value
//     is stored as one 8-byte word {value, launch tag} into a program-owned
//     buffer of its phase (written once per launch, so no phase ever
//     overwrites data a slower CTA still reads).  An 8-byte aligned store is
//     single-copy atomic, so a reader that sees the current tag in a word sees
//     that word's value: no fence, no counter.  A consumer warp polls exactly
//     the input words it needs -- its own 256-value blocks, and for an
//     RMSNorm input the 32-row group sums of squares the producer's finishers
//     publish the same way -- and the load that sees the tag IS the load of
//     the data.  A warp starts a phase as soon as its blocks exist, while
//     other warps and CTAs may still be finishing the previous phase;
//   * inputs written before the launch (the first phase's activations, a
//     residual of outside data) are copied into tagged buffers by all CTAs
//     at the start, followed by the kernel's one grid-wide barrier, so no
//     phase can overwrite caller memory another CTA has yet to read;
//   * the tag is the launch count + 1 (a device word advanced by CTA 0 after
//     the barrier, when every CTA has read it), and the phases' tagged
//     buffers are double-buffered by the tag's parity (with several GPUs a
//     rank may run one launch ahead of another; their layout is the same on
//     every rank, so a peer's copy is this rank's address plus one offset).
// All CTAs must be resident at once: the launch is cooperative (the runtime
// refuses a grid that cannot be co-resident).  Every wait is bounded; on
// expiry the kernel records kDevErrTimeout, stores the launch's tag into the
// abort word so every other waiter of the launch gives up at once, and
// returns (the program must then be reset before its next run).
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "q2k_core.cuh"
#include "q8k_device.cuh"
#include "runtime.h"

namespace smeai {

namespace {

constexpr int kMaxWarps = 19;                    // producer + up to 16 consumers + 2 finishers
// (19 warps keep the 96-register cap of 17: the four schedulers' 16K-register
// files hold at most 5 warps each either way)
constexpr uint32_t kProgramMagic = 0x51325048u;  // "Q2PH"
constexpr uint64_t kAbortCheckNs = 20000;        // waits shorter than this never read the abort word
// Replicas of every group-sum array: the finisher's lanes 0..kSumReps-1 each
// store one, and a warp reads replica (cta + warp) % kSumReps, so the few
// cache lines every warp of the grid needs for an RMSNorm are spread over
// kSumReps places instead of one.
constexpr int kSumReps = 16;
// Row-group terms buffers between the consumer warps and the two finisher
// warps (group jj uses buffer jj mod tbufs).  Measured on B200: four buffers
// (consumers up to three groups ahead of the finishing) took 0.894 ms per
// 7B-shape token against 0.842 ms with two.
constexpr int kMaxTbufs = 2;
constexpr int kDefaultL2Ahead = 0;  // measured on B200: 0.860 ms/token at 0, 0.863 at 4, 0.869 at 8, 0.94 at 12+

// Descriptor of one phase.  The *_ll pointers address the tagged buffers of
// set 0; the kernel adds the set offset of its launch.  Token t, row r of a
// tagged buffer is word [t * ld + r].
struct PhaseDev {
  const uint8_t* tiles;
  const uint8_t* xq;         // kInQ8K: Q8_K blocks (caller memory), contiguous token rows
  const uint64_t* x_ll;      // fp32 input as tagged words
  const uint64_t* xs_ll;     // kInF32Rms: 32-value group sums of squares of the input, tagged,
                             // [token][replica][ld_xsll]
  const float* norm_w;       // kInF32Rms: RMSNorm weight, or null
  float* y;                  // caller-visible output
  uint64_t* y_ll;            // tagged output
  uint64_t* ys_ll;           // tagged group sums of squares of the output (a later RMS input), or null,
                             // [token][replica][ld_ysll]
  const uint64_t* r_ll;      // tagged residual, or null
  int64_t ld_xll, ld_xsll, ldy, ld_yll, ld_ysll, ld_rll;
  int64_t n_rows;
  int64_t n_groups;
  // local output rows [ex_lo, ex_hi) are rows ex_row0.. of the phase's tagged
  // (global) output; with several GPUs every rank stores them into every
  // rank's copy.  One GPU: the identity.
  int64_t ex_lo, ex_hi, ex_row0;
  int x_ext, r_ext;          // input / residual is a copy of outside data: one buffer, no set offset
  int64_t rot;               // row group g of this phase runs on CTA (g + rot) % grid: the dealing
                             // continues from the previous phase, so no CTA takes every phase's extra group
  int nb;
  int in_mode;
  int epi;
  int pad;
};

// Inputs written before the launch, copied into tagged buffers at its start.
// These copies are this GPU's own (never written by peers) and single: the
// previous launch on this GPU, their only other reader, has completed.
struct CopyDev {
  const float* src;
  int64_t ld_src;
  uint64_t* dst;             // tagged, set 0
  int64_t ld_dst;
  uint64_t* sums;            // tagged group sums of squares (set 0), [token][replica][ld_sums], or null
  int64_t ld_sums;
  int64_t len;               // values per token
  int64_t units;             // T * ceil(len / 32): one 32-value group of one token each
};

struct ProgParams {
  const PhaseDev* phases;
  const CopyDev* copies;
  int n_phases;
  int n_copies;
  int nb_max;
  float eps;
  int stages;
  int log2_stages;
  unsigned* ctl;        // [0] launches completed (the tag is ctl[0] + 1), [1] barrier arrivals, [2] abort tag
  unsigned* err;
  uint64_t timeout_ns;  // every bounded wait
  int64_t set_bytes;    // distance between the two sets of tagged buffers
  int tbufs;            // row-group terms buffers: 2, or 1 when two do not fit
  int log2_tbufs;
  int l2_ahead;         // ring stages the L2 prefetch stream runs ahead of the ring loads
  int sys;              // tagged words at system scope (peers store into this GPU's buffers)
  int n_peers;          // other ranks whose copies of the tagged buffers this rank stores into
  int64_t peer_delta[kMaxPeers];  // byte offset from this rank's buffers to peer q's mapping of its own
  int act_chunks;       // Q8_K activation slot chunks per warp and token (the 8-token kernel may reuse them)
};

struct PSmem {
  uint8_t* ring;
  int4* qs;
  int* bs;
  float* d;
  float* terms;       // [tbufs][T * nb_max][32]
  uint64_t* full;
  uint64_t* empty;
  uint64_t* grp;      // [kMaxTbufs] all consumer warps wrote a row group's terms
  uint64_t* tfree;    // [kMaxTbufs] the finisher has consumed them
  // RMSNorm inputs: the first consumer warp to reach the CTA's n-th RMSNorm
  // phase polls the group sums and publishes 1/rms of every token in slot
  // n % 4 (a warp can run at most two phases ahead of the slowest one)
  unsigned* rms_claim;  // highest n + 1 claimed
  unsigned* rms_ready;  // [4] n + 1 once slot n % 4 holds phase n's values
  float* rms_inv;       // [4][8]
};

__host__ __device__ __forceinline__ size_t al16(size_t v) { return (v + 15) & ~(size_t)15; }

// Q8_K activation slot of warp cw's i-th super-block (b = cw + i * W) and
// token t.  Slots belong to one warp in every phase: a warp that has moved
// on to the next phase's prologue cannot overwrite an activation a slower
// warp of its CTA still reads.
__device__ __forceinline__ int act_slot(int cw, int W, int T, int i, int t) { return cw + W * (t + T * i); }
// Slots hold act_chunks chunks of W blocks per token.  A phase whose input
// is a plain fp32 vector and which gives no CTA more than one row group uses
// each block once per CTA: its chunk c is quantized just before use into
// chunk slot c mod act_chunks, so its width does not size the slots (the
// k = 11008 down projection of 8 tokens would take 100 KB).
__host__ __device__ __forceinline__ size_t act_slots(int T, int act_chunks, int W) {
  return (size_t)W * T * act_chunks;
}

__host__ __device__ __forceinline__ size_t prog_fixed_bytes(int T, int nb_max, int act_chunks, int W, int tbufs) {
  const size_t slots = act_slots(T, act_chunks, W);
  return al16(slots * 256) + al16(slots * 32) + al16(slots * 4) + al16((size_t)tbufs * T * nb_max * 128) +
         8 * 2 * kMaxTbufs + 16 + 16 + 32 + 128;
}
__host__ __device__ __forceinline__ size_t prog_smem_bytes(int T, int nb_max, int act_chunks, int stages,
                                                          int consumers, int tbufs) {
  return (size_t)stages * consumers * kTileBytes + prog_fixed_bytes(T, nb_max, act_chunks, consumers, tbufs) +
         (size_t)stages * 16;
}

__device__ __forceinline__ PSmem pcarve(uint8_t* base, int T, int nb_max, int act_chunks, int stages, int consumers,
                                        int tbufs) {
  PSmem m;
  size_t o = 0;
  const size_t slots = act_slots(T, act_chunks, consumers);
  m.ring = base;
  o += (size_t)stages * consumers * kTileBytes;
  m.qs = reinterpret_cast<int4*>(base + o);
  o += al16(slots * 256);
  m.bs = reinterpret_cast<int*>(base + o);
  o += al16(slots * 32);
  m.d = reinterpret_cast<float*>(base + o);
  o += al16(slots * 4);
  m.terms = reinterpret_cast<float*>(base + o);
  o += al16((size_t)tbufs * T * nb_max * 128);
  m.full = reinterpret_cast<uint64_t*>(base + o);
  m.empty = m.full + stages;
  m.grp = m.empty + stages;
  m.tfree = m.grp + kMaxTbufs;
  m.rms_claim = reinterpret_cast<unsigned*>(m.tfree + kMaxTbufs);
  m.rms_ready = m.rms_claim + 4;
  m.rms_inv = reinterpret_cast<float*>(m.rms_ready + 8);
  return m;
}

// ---- tagged words ------------------------------------------------------------
__device__ __forceinline__ uint64_t ll_pack(float v, unsigned tag) {
  return ((uint64_t)tag << 32) | (uint64_t)__float_as_uint(v);
}
__device__ __forceinline__ bool ll_has(uint64_t w, unsigned tag) { return (unsigned)(w >> 32) == tag; }
__device__ __forceinline__ float ll_val(uint64_t w) { return __uint_as_float((unsigned)w); }
// Tagged words are read and written at GPU scope on one GPU, at system scope
// when other GPUs store into this GPU's buffers (the flag is uniform).
__device__ __forceinline__ void ll_st_scoped(uint64_t* p, uint64_t w, int sys) {
  if (sys) asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
  else asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t ll_ld_scoped(const uint64_t* p, int sys) {
  uint64_t w;
  if (sys) asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  else asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
__device__ __forceinline__ void ll_ld2_scoped(const uint64_t* p, uint64_t& a, uint64_t& b, int sys) {
  if (sys) asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
  else asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
template <typename Ptr>
__device__ __forceinline__ Ptr set_ptr(Ptr p, int64_t off) {
  return reinterpret_cast<Ptr>(reinterpret_cast<uintptr_t>(p) + off);
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
__device__ __forceinline__ void st_relaxed_gpu(unsigned* p, unsigned v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// A finished tagged word into this rank's buffer and every peer's copy.
__device__ __forceinline__ void ll_put(const ProgParams& P, uint64_t* p, uint64_t w) {
  ll_st_scoped(p, w, P.sys);
  for (int q = 0; q < P.n_peers; ++q) ll_st_scoped(set_ptr(p, P.peer_delta[q]), w, 1);
}

// Record a timeout and make every other waiter of this launch give up.
__device__ __forceinline__ void fail(const ProgParams& P, unsigned tag) {
  raise_device_error(P.err, kDevErrTimeout);
  st_relaxed_gpu(P.ctl + 2, tag);
}

// mbarrier wait bounded by the time limit that also gives up at once when
// the launch has been aborted.
__device__ __forceinline__ bool pwait(uint64_t* bar, unsigned parity, const ProgParams& P, unsigned tag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    const uint64_t el = global_timer_ns() - t0;
    if (el > kAbortCheckNs && ld_relaxed_gpu(P.ctl + 2) == tag) return false;
    if (el > P.timeout_ns) {
      fail(P, tag);
      return false;
    }
  }
}

// Bounded wait state of one warp's poll loop.  The abort word and the clock
// are read only every 8th retry, and the abort word only after the wait has
// lasted kAbortCheckNs: every waiting warp of the grid reads the same abort
// word, and in a healthy launch no wait lasts that long.
struct Poll {
  uint64_t t0 = 0;
  int iter = 0;
  // Called after a poll found something missing: false when the launch was
  // aborted or the time limit ran out.
  __device__ __forceinline__ bool again(const ProgParams& P, unsigned tag) {
    if (iter++ == 0) t0 = global_timer_ns();
    if ((iter & 7) == 0) {
      const uint64_t el = global_timer_ns() - t0;
      if (el > kAbortCheckNs && ld_relaxed_gpu(P.ctl + 2) == tag) return false;
      if (el > P.timeout_ns) {
        fail(P, tag);
        return false;
      }
    }
    __nanosleep(256);
    return true;
  }
};

// Eight consecutive tagged values of this lane (a 2 KB block per warp).
struct LL8 {
  uint64_t w[8];
};
__device__ __forceinline__ void ll_load8(const uint64_t* p, LL8& r, int sys) {
#pragma unroll
  for (int k = 0; k < 8; k += 2) ll_ld2_scoped(p + k, r.w[k], r.w[k + 1], sys);
}
__device__ __forceinline__ bool ll_ready8(const LL8& r, unsigned tag) {
  bool ok = true;
#pragma unroll
  for (int k = 0; k < 8; ++k) ok &= ll_has(r.w[k], tag);
  return ok;
}
// Wait until every word of the warp's block carries `tag` (r holds a first
// load): every retry re-reads the whole block, so the retry that finds the
// last word also brings the values.
__device__ __forceinline__ bool ll_wait8(const uint64_t* p, LL8& r, unsigned tag, const ProgParams& P) {
  if (__all_sync(0xffffffffu, ll_ready8(r, tag))) return true;
  Poll pl;
  for (;;) {
    if (!pl.again(P, tag)) return false;
    ll_load8(p, r, P.sys);
    if (__all_sync(0xffffffffu, ll_ready8(r, tag))) return true;
  }
}

// RMSNorm total of one token from the producer's G tagged group sums, in the
// fixed order (lane l adds groups l, l + 32, ... ascending, then the lanes
// fold at distances 16, 8, 4, 2, 1).  false on timeout / abort.
__device__ bool ll_rms_total(const uint64_t* sums, int G, unsigned tag, const ProgParams& P, float& total) {
  const int lane = threadIdx.x & 31;
  float acc = 0.f;
  for (int g0 = 0; g0 < G; g0 += 32 * 8) {
    uint64_t w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int g = g0 + lane + 32 * j;
      w[j] = g < G ? ll_ld_scoped(sums + g, P.sys) : ((uint64_t)tag << 32);
    }
    Poll pl;
    for (;;) {
      bool ok = true;
#pragma unroll
      for (int j = 0; j < 8; ++j) ok &= ll_has(w[j], tag);
      if (__all_sync(0xffffffffu, ok)) break;
      if (!pl.again(P, tag)) return false;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int g = g0 + lane + 32 * j;
        if (g < G && !ll_has(w[j], tag)) w[j] = ll_ld_scoped(sums + g, P.sys);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (g0 + lane + 32 * j < G) acc = __fadd_rn(acc, ll_val(w[j]));
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
  total = acc;
  return true;
}

// Q8_K of one tagged input block of warp cw (block b, token t) into the
// warp's activation slot, after an RMSNorm (1/rms inv, times the norm weight)
// when rms is set -- the standalone quantizer's arithmetic.  w holds a first
// load of the block; the wait for its tags is bounded.
template <int T>
__device__ __forceinline__ bool quant_block(const ProgParams& P, const ActSmem& act, const PhaseDev& D,
                                            const uint64_t* src, LL8& w, bool rms, float inv, int b, int slot,
                                            int lane, unsigned tag) {
  if (!ll_wait8(src, w, tag, P)) return false;
  float u[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) u[k] = ll_val(w.w[k]);
  if (rms) {
#pragma unroll
    for (int k = 0; k < 8; ++k) u[k] = __fmul_rn(u[k], inv);
    if (D.norm_w) {
      const float4 g0 = __ldg(reinterpret_cast<const float4*>(D.norm_w + b * QK_K + lane * 8));
      const float4 g1 = __ldg(reinterpret_cast<const float4*>(D.norm_w + b * QK_K + lane * 8 + 4));
      u[0] = __fmul_rn(u[0], g0.x);
      u[1] = __fmul_rn(u[1], g0.y);
      u[2] = __fmul_rn(u[2], g0.z);
      u[3] = __fmul_rn(u[3], g0.w);
      u[4] = __fmul_rn(u[4], g1.x);
      u[5] = __fmul_rn(u[5], g1.y);
      u[6] = __fmul_rn(u[6], g1.z);
      u[7] = __fmul_rn(u[7], g1.w);
    }
  }
  store_q8k_smem(q8k_quantize_lane(u), act, slot);
  return true;
}

// Activation prologue of warp cw for one phase.  Its super-blocks are
// b = cw (mod W); item it = i * T + t is block cw + i * W of token t.
//  * Q8_K input (caller memory): staged into the warp's slots.
//  * RMSNorm input: the producer's group sums and the warp's block are
//    polled in ONE loop (one token, one block per warp, k <= 8192),
//    so the retry that finds the last word also holds every value; then the
//    blocks are normalized and quantized.  Returns *ready = all items.
//  * plain input: nothing here -- ensure_item() polls and quantizes each
//    block when the warp first needs it, so the phase starts on its early
//    blocks while later ones are still being produced.
template <int T>
__device__ __forceinline__ bool prologue(const ProgParams& P, const ActSmem& act, const PhaseDev& D, int cw,
                                         int W, int lane, unsigned tag, int64_t so, unsigned& ready,
                                         unsigned* m_rms_claim, unsigned* m_rms_ready, float* m_rms_inv,
                                         unsigned& nrms) {
  const int nb = D.nb;
  ready = 0u;
  if (D.in_mode == kInQ8K) {  // caller memory, complete before the launch
    const uint32_t* src = reinterpret_cast<const uint32_t*>(D.xq);
    for (int b = cw; b < nb; b += W) {
#pragma unroll 1
      for (int t = 0; t < T; ++t)
        copy_q8k_smem(src + ((int64_t)t * nb + b) * Q8K_BLOCK_WORDS, act, act_slot(cw, W, T, b / W, t), lane);
    }
    ready = ~0u;
    return true;
  }
  if (D.in_mode != kInF32Rms) return true;
  const uint64_t* x = set_ptr(D.x_ll, D.x_ext ? 0 : so);
  const int nbw = cw < nb ? (nb - cw + W - 1) / W : 0;  // blocks of this warp
  const int items = nbw * T;
  auto src = [&](int it) { return x + (it % T) * D.ld_xll + (cw + (it / T) * W) * QK_K + lane * 8; };
  const int G = nb * 8;  // group sums per token
  const int n = (int)(nrms & 3);
  // the warp's blocks and norm weights go out first; they are checked (and,
  // if still incomplete, re-read) once 1/rms is known
  LL8 r0;
  const bool one = items == 1;
  if (one) ll_load8(src(0), r0, P.sys);
  float4 g0 = make_float4(0.f, 0.f, 0.f, 0.f), g1 = g0;
  if (one && D.norm_w) {
    g0 = __ldg(reinterpret_cast<const float4*>(D.norm_w + cw * QK_K + lane * 8));
    g1 = __ldg(reinterpret_cast<const float4*>(D.norm_w + cw * QK_K + lane * 8 + 4));
  }
  unsigned prev = 0;
  if (lane == 0) prev = atomicMax(m_rms_claim, nrms + 1);
  prev = __shfl_sync(0xffffffffu, prev, 0);
  if (prev < nrms + 1) {
    // this warp polls the group sums (one replica per CTA) for the CTA
    const uint64_t* sums = set_ptr(D.xs_ll, D.x_ext ? 0 : so) + (int)(blockIdx.x % kSumReps) * D.ld_xsll;
#pragma unroll 1
    for (int t = 0; t < T; ++t) {
      float total;
      if (!ll_rms_total(sums + t * kSumReps * D.ld_xsll, G, tag, P, total)) return false;
      if (lane == 0) m_rms_inv[n * 8 + t] = rms_inv_from_sum(total, nb * QK_K, P.eps);
    }
    __syncwarp();
    __threadfence_block();
    if (lane == 0) *reinterpret_cast<volatile unsigned*>(m_rms_ready + n) = nrms + 1;
  } else {
    // another warp polls: wait (bounded) for its shared-memory flag; meanwhile
    // watch the warp's own block (one word per 32-value group: 64 bytes per
    // retry) and fetch it whole once every group has landed, so the block is
    // in registers when 1/rms arrives
    bool have = !one || __all_sync(0xffffffffu, ll_ready8(r0, tag));
    const uint64_t t0 = global_timer_ns();
    for (int k = 0; *reinterpret_cast<volatile unsigned*>(m_rms_ready + n) != nrms + 1; ++k) {
      if (!have && (k & 7) == 7) {
        const bool probe_ok = (lane & 3) != 3 || ll_has(ll_ld_scoped(src(0) + 7, P.sys), tag);
        if (__all_sync(0xffffffffu, probe_ok)) {
          ll_load8(src(0), r0, P.sys);
          have = __all_sync(0xffffffffu, ll_ready8(r0, tag));
        }
      }
      __nanosleep(32);
      if ((k & 255) == 255) {
        const uint64_t el = global_timer_ns() - t0;
        if (el > kAbortCheckNs && ld_relaxed_gpu(P.ctl + 2) == tag) return false;
        if (el > P.timeout_ns) {
          fail(P, tag);
          return false;
        }
      }
    }
    __threadfence_block();
  }
  ++nrms;
  float inv[T];
#pragma unroll
  for (int t = 0; t < T; ++t) inv[t] = *reinterpret_cast<volatile float*>(m_rms_inv + n * 8 + t);
  if (one) {
    if (!ll_wait8(src(0), r0, tag, P)) return false;
    float u[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) u[k] = __fmul_rn(ll_val(r0.w[k]), inv[0]);
    if (D.norm_w) {
      u[0] = __fmul_rn(u[0], g0.x);
      u[1] = __fmul_rn(u[1], g0.y);
      u[2] = __fmul_rn(u[2], g0.z);
      u[3] = __fmul_rn(u[3], g0.w);
      u[4] = __fmul_rn(u[4], g1.x);
      u[5] = __fmul_rn(u[5], g1.y);
      u[6] = __fmul_rn(u[6], g1.z);
      u[7] = __fmul_rn(u[7], g1.w);
    }
    store_q8k_smem(q8k_quantize_lane(u), act, act_slot(cw, W, T, 0, 0));
  } else {
    for (int it = 0; it < items; ++it) {
      LL8 w;
      ll_load8(src(it), w, P.sys);
      if (!quant_block<T>(P, act, D, src(it), w, true, inv[it % T], cw + (it / T) * W,
                          act_slot(cw, W, T, it / T, it % T), lane, tag))
        return false;
    }
  }
  ready = ~0u;
  return true;
}

// Plain fp32 input: block i of warp cw (all tokens), polled and quantized
// the first time the warp needs it, into chunk slot ic (i, or i mod
// act_chunks when the phase's blocks are used once per CTA).
template <int T>
__device__ __forceinline__ bool ensure_block(const ProgParams& P, const ActSmem& act, const PhaseDev& D, int cw,
                                          int W, int lane, unsigned tag, int64_t so, int i, int ic,
                                          unsigned& ready) {
  const uint64_t* x = set_ptr(D.x_ll, D.x_ext ? 0 : so);
  const int b = cw + i * W;
  constexpr int kBatch = T <= 2 ? T : 1;  // tokens whose loads go out together
#pragma unroll 1
  for (int t0 = 0; t0 < T; t0 += kBatch) {
    LL8 w[kBatch];
#pragma unroll
    for (int t = 0; t < kBatch; ++t) ll_load8(x + (t0 + t) * D.ld_xll + b * QK_K + lane * 8, w[t], P.sys);
#pragma unroll
    for (int t = 0; t < kBatch; ++t)
      if (!quant_block<T>(P, act, D, x + (t0 + t) * D.ld_xll + b * QK_K + lane * 8, w[t], false, 1.f, b,
                          act_slot(cw, W, T, ic, t0 + t), lane, tag))
        return false;
  }
  ready |= 1u << i;
  return true;
}

// Ordered sum of one row group's super-block terms and the phase's epilogue
// (the arithmetic of finish_group in q2k_gemv.cu); the caller-visible store,
// the tagged store, and the group sums of squares when a later phase reads
// this output through an RMSNorm.
// Issue the residual loads of a row group (one tagged word per lane and
// token) ahead of the wait for the group's terms.
template <int T>
__device__ __forceinline__ void resid_issue(const PhaseDev& D, int64_t group, int lane, unsigned tag, int64_t so,
                                            uint64_t (&w)[T], int sys) {
  const int64_t orow = group * 32 + lane;
#pragma unroll
  for (int t = 0; t < T; ++t)
    w[t] = (D.epi == kEpiResidual && orow < D.n_rows) ? ll_ld_scoped(set_ptr(D.r_ll, D.r_ext ? 0 : so) + t * D.ld_rll + orow, sys)
                                                      : ((uint64_t)tag << 32);
}

template <int T>
__device__ __forceinline__ bool finish_group_prog(const ProgParams& P, const float* terms, const PhaseDev& D,
                                                  int64_t group, int lane, unsigned tag, int64_t so,
                                                  uint64_t (&w)[T]) {
  const int nb = D.nb;
  uint64_t* yl = set_ptr(D.y_ll, so);
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
          const float h = __fmul_rn(sg, u);
          D.y[t * D.ldy + orow] = h;
          if (orow >= D.ex_lo && orow < D.ex_hi) ll_put(P, yl + t * D.ld_yll + D.ex_row0 + (orow - D.ex_lo), ll_pack(h, tag));
        }
      }
    }
    return true;
  }
  const int64_t orow = group * 32 + lane;
  const bool live = orow < D.n_rows;
  float r[T];
  if (D.epi == kEpiResidual) {  // the residual loads went out before the terms wait
    const uint64_t* rl = set_ptr(D.r_ll, D.r_ext ? 0 : so);
    Poll pl;
    for (;;) {
      bool ok = true;
#pragma unroll
      for (int t = 0; t < T; ++t) ok &= ll_has(w[t], tag);
      if (__all_sync(0xffffffffu, ok)) break;
      if (!pl.again(P, tag)) return false;
#pragma unroll
      for (int t = 0; t < T; ++t)
        if (live && !ll_has(w[t], tag)) w[t] = ll_ld_scoped(rl + t * D.ld_rll + orow, P.sys);
    }
#pragma unroll
    for (int t = 0; t < T; ++t) r[t] = ll_val(w[t]);
  }
  uint64_t* ysl = D.ys_ll ? set_ptr(D.ys_ll, so) : nullptr;
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
    if (live) {
      if (D.epi == kEpiResidual) s = __fadd_rn(r[t], s);
      D.y[t * D.ldy + orow] = s;
      if (orow >= D.ex_lo && orow < D.ex_hi) ll_put(P, yl + t * D.ld_yll + D.ex_row0 + (orow - D.ex_lo), ll_pack(s, tag));
    }
    if (ysl) {  // the group's sum of squares (its rows all exchanged: ex_lo, ex_row0 32-row aligned)
      const float ss = group_sumsq_lane(live ? s : 0.f);
      const int64_t gg = (D.ex_row0 + group * 32 - D.ex_lo) >> 5;
      if (lane < kSumReps && group * 32 >= D.ex_lo && group * 32 < D.ex_hi)
        ll_put(P, ysl + (t * kSumReps + lane) * D.ld_ysll + gg, ll_pack(ss, tag));
    }
  }
  return true;
}

// Walks this CTA's row groups in program order (phase, then c, c + C, ...);
// jj counts them (the terms buffer of group jj is jj mod tbufs).
struct GroupCursor {
  int ph = 0, n_phases = 0, jj = 0;
  int64_t g = 0, ng = 0;

  __device__ void seek(const ProgParams& P, int64_t cta, int64_t C) {
    for (; ph < n_phases; ++ph) {
      const PhaseDev& D = P.phases[ph];
      const int64_t first = (cta + C - D.rot) % C;
      if (first < D.n_groups) {
        g = first;
        ng = D.n_groups;
        return;
      }
    }
  }
  __device__ void start(const ProgParams& P, int64_t cta, int64_t C) {
    n_phases = P.n_phases;
    ph = 0;
    jj = 0;
    seek(P, cta, C);
  }
  __device__ bool valid() const { return ph < n_phases; }
  __device__ void next(const ProgParams& P, int64_t cta, int64_t C) {
    if (!valid()) return;
    ++jj;
    g += C;
    if (g < ng) return;
    ++ph;
    seek(P, cta, C);
  }
};

// Walks this CTA's ring stages in program order: phase, row group (c, c + C,
// ...), chunk of up to W consecutive super-blocks (incrementally: the
// producer thread does no division per stage).
struct StageCursor {
  int ph = 0, n_phases = 0;
  int64_t g = 0, ng = 0, C = 1;
  int c = 0, nchunks = 0, nb = 0, W = 0;
  const uint8_t* tiles = nullptr;

  __device__ void load_phase(const ProgParams& P, int64_t cta) {
    for (; ph < n_phases; ++ph) {
      const PhaseDev& D = P.phases[ph];
      const int64_t first = (cta + C - D.rot) % C;
      if (first < D.n_groups) {
        nb = D.nb;
        nchunks = (nb + W - 1) / W;
        ng = D.n_groups;
        tiles = D.tiles;
        g = first;
        c = 0;
        return;
      }
    }
  }
  __device__ void start(const ProgParams& P, int64_t cta, int64_t nctas, int w) {
    W = w;
    C = nctas;
    n_phases = P.n_phases;
    ph = 0;
    load_phase(P, cta);
  }
  __device__ bool valid() const { return ph < n_phases; }
  __device__ const uint8_t* src() const { return tiles + ((size_t)g * nb + (size_t)c * W) * kTileBytes; }
  __device__ unsigned bytes() const { return (unsigned)(min(W, nb - c * W) * kTileBytes); }
  __device__ void advance(const ProgParams& P, int64_t cta) {
    if (++c < nchunks) return;
    c = 0;
    g += C;
    if (g < ng) return;
    ++ph;
    load_phase(P, cta);
  }
};

// Copy the launch's outside inputs into their tagged buffers: one warp per
// 32-value group of one token, with the group's sum of squares when an
// RMSNorm reads it (the finishers' fold: one value per lane).
__device__ void copy_inputs(const ProgParams& P, unsigned tag, int64_t so, int64_t gw, int64_t nw, int lane) {
  int j = 0;
  int64_t base = 0;
  for (int64_t u = gw;; u += nw) {
    while (j < P.n_copies && u >= base + P.copies[j].units) {
      base += P.copies[j].units;
      ++j;
    }
    if (j >= P.n_copies) return;
    const CopyDev& cp = P.copies[j];
    const int64_t per_tok = (cp.len + 31) / 32;
    const int64_t t = (u - base) / per_tok, grp = (u - base) - t * per_tok;
    const int64_t i = grp * 32 + lane;
    const float v = i < cp.len ? cp.src[t * cp.ld_src + i] : 0.f;
    if (i < cp.len) ll_st_scoped(set_ptr(cp.dst, so) + t * cp.ld_dst + i, ll_pack(v, tag), P.sys);
    if (cp.sums) {
      const float ss = group_sumsq_lane(v);
      if (lane < kSumReps)
        ll_st_scoped(set_ptr(cp.sums, so) + (t * kSumReps + lane) * cp.ld_sums + grp, ll_pack(ss, tag), P.sys);
    }
  }
}

template <int T>
__global__ void __launch_bounds__(kMaxWarps * 32, 1) q2k_program_kernel(const ProgParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int W = (blockDim.x >> 5) - 3;   // warp 0 producer, 1..W consumers, W+1 and W+2 finishers
  const int S = P.stages, lgS = P.log2_stages, smask = S - 1;
  const int64_t C = gridDim.x, cta = blockIdx.x;
  const int stage_bytes = W * kTileBytes;
  // the 1/2/4-token kernels size the slots from nb_max (act_chunks is then
  // ceil(nb_max / W)); only the 8-token kernel reads the reuse-aware count
  const PSmem m = pcarve(smem, T, P.nb_max, T == 8 ? P.act_chunks : (P.nb_max + W - 1) / W, S, W, P.tbufs);
  // every thread reads the launch count before the CTA's first sync, i.e.
  // before its CTA can arrive at the grid barrier after which CTA 0 advances it
  const unsigned tag = ld_relaxed_gpu(P.ctl) + 1u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&m.full[s], 1);
      mbar_init(&m.empty[s], W);
    }
    for (int b = 0; b < kMaxTbufs; ++b) {
      mbar_init(&m.grp[b], W);
      mbar_init(&m.tfree[b], 1);
    }
    *m.rms_claim = 0u;
    for (int k = 0; k < 4; ++k) m.rms_ready[k] = 0u;
    mbar_fence_init();
  }
  __syncthreads();
  const int64_t so = (int64_t)(tag & 1u) * P.set_bytes;

  if (warp == 0) {
    // ---- producer: every phase's tiles of this CTA, in program order
    if (lane == 0) {
      // A second cursor runs l2_ahead stages ahead and asks the TMA engine to
      // bring those tiles into L2: while the consumers wait at a phase
      // boundary with the ring full, HBM keeps streaming into L2, and the ring
      // then refills from L2 instead of at the HBM rate.
      StageCursor issue, pref;
      issue.start(P, cta, C, W);
      pref.start(P, cta, C, W);
      int64_t npref = 0;
      bool ok = true;
      int64_t i = 0;
      for (; issue.valid(); issue.advance(P, cta), ++i) {
        for (; P.l2_ahead > 0 && pref.valid() && npref < i + P.l2_ahead; pref.advance(P, cta), ++npref)
          bulk_prefetch_l2(pref.src(), pref.bytes());
        const int s = (int)(i & smask);
        if (i >= S && !pwait(&m.empty[s], (unsigned)(((i >> lgS) - 1) & 1), P, tag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&m.full[s], issue.bytes());
        bulk_copy_g2s(m.ring + (size_t)s * stage_bytes, issue.src(), issue.bytes(), &m.full[s]);
      }
      if (!ok) {
        fail(P, tag);
        for (int64_t j = (i > S ? i - S : 0); j < i; ++j)
          mbar_wait_bounded(&m.full[j & smask], (unsigned)((j >> lgS) & 1), P.timeout_ns);
      }
    }
    return;
  }

  if (warp > W) {
    // ---- finishers: finisher f finishes the CTA's row groups jj = f
    // (mod 2) in order, group jj from terms buffer jj mod tbufs -- the
    // ordered sum, the epilogue and the stores run beside the consumers'
    // next tiles instead of in one consumer's path; a group's residual loads
    // go out before the wait for the finisher's previous group
    const int nfin = P.tbufs < 2 ? P.tbufs : 2;
    const int f = warp - W - 1;
    if (f >= nfin) return;
    GroupCursor cur;
    cur.start(P, cta, C);
    for (int k = 0; k < f; ++k) cur.next(P, cta, C);
    uint64_t rw[T];
    if (cur.valid()) resid_issue<T>(P.phases[cur.ph], cur.g, lane, tag, so, rw, P.sys);
    while (cur.valid()) {
      // the descriptor by value: the group's stores cannot make the compiler
      // reload its fields from global memory
      const PhaseDev D = P.phases[cur.ph];
      const int64_t g = cur.g;
      const int buf = cur.jj & (P.tbufs - 1), use = cur.jj >> P.log2_tbufs;
      GroupCursor nx = cur;
      for (int k = 0; k < nfin; ++k) nx.next(P, cta, C);
      // the next group's residual loads go out before this group's wait
      uint64_t rn[T];
      if (nx.valid()) resid_issue<T>(P.phases[nx.ph], nx.g, lane, tag, so, rn, P.sys);
      const float* terms = m.terms + (size_t)buf * T * P.nb_max * 32;
      if (!pwait(&m.grp[buf], (unsigned)(use & 1), P, tag)) return;
      const bool ok = finish_group_prog<T>(P, terms, D, g, lane, tag, so, rw);
      mbar_arrive_warp(&m.tfree[buf]);
      if (!ok) return;
#pragma unroll
      for (int t = 0; t < T; ++t) rw[t] = rn[t];
      cur = nx;
    }
    return;
  }

  // ---- consumers
  const int cw = warp - 1;
  const ActSmem act = {m.qs, m.bs, m.d};

  // outside inputs -> tagged buffers, then the one grid-wide barrier: after
  // it no CTA reads caller memory a phase may overwrite
  copy_inputs(P, tag, 0, cta * W + cw, C * W, lane);
  asm volatile("bar.sync 1, %0;" ::"r"(W * 32) : "memory");
  if (cw == 0) {
    int ok = 1;
    if (lane == 0) {
      red_release_gpu_add(P.ctl + 1, 1u);
      const unsigned target = tag * (unsigned)C;
      if ((int)(ld_acquire_gpu(P.ctl + 1) - target) < 0) {
        const uint64_t t0 = global_timer_ns();
        for (int k = 0; (int)(ld_acquire_gpu(P.ctl + 1) - target) < 0; ++k) {
          if ((k & 15) == 15 && (ld_relaxed_gpu(P.ctl + 2) == tag || global_timer_ns() - t0 > P.timeout_ns)) {
            fail(P, tag);
            ok = 0;
            break;
          }
        }
      }
      if (ok && cta == 0) st_relaxed_gpu(P.ctl, tag);  // every CTA has read the count: advance it
    }
    __syncwarp();
  }
  asm volatile("bar.sync 1, %0;" ::"r"(W * 32) : "memory");
  if (ld_relaxed_gpu(P.ctl + 2) == tag) return;

  int64_t i = 0;  // ring stage, in step with the producer
  int jj = 0;     // row groups processed by this CTA (terms buffers)
  unsigned nrms = 0;  // RMSNorm phases this warp has entered
  for (int ph = 0; ph < P.n_phases; ++ph) {
    const PhaseDev& D = P.phases[ph];
    const int64_t ngr = D.n_groups;
    const int64_t first = (cta + C - D.rot) % C;
    if (first >= ngr) continue;
    const int nb = D.nb;
    const int nchunks = (nb + W - 1) / W;
    unsigned ready;
    if (!prologue<T>(P, act, D, cw, W, lane, tag, so, ready, m.rms_claim, m.rms_ready, m.rms_inv, nrms)) return;
    __syncwarp();

    // 8 tokens: the activation fragments of a one-chunk phase are read once
    // per phase (the warp's block is the same for all its row groups)
    Act8Frag fr;
    bool fr_loaded = false;
    // this CTA's row groups of the phase: first, first + C, ...
    for (int64_t g = first; g < ngr; g += C, ++jj) {
      // terms buffer of this group and how many times it was used before
      const int buf = jj & (P.tbufs - 1);
      const int use = jj >> P.log2_tbufs;
      float* terms = m.terms + (size_t)buf * T * P.nb_max * 32;
      if (use >= 1 && !pwait(&m.tfree[buf], (unsigned)((use - 1) & 1), P, tag)) return;
      const int64_t row = g * 32 + lane;
      // chunk slot of chunk c: c, wrapping at act_chunks in the 8-token kernel
      // (only a phase whose blocks are used once wraps; the other kernels
      // never reuse slots: their code and shared-memory carve are those of
      // the kernel before slot reuse, which measured 1.8% faster at 1 token
      // on B200 than one carving from act_chunks)
      constexpr bool kReuse = T == 8;
      int icw = 0;
      for (int c = 0; c < nchunks; ++c, ++i, icw = icw + 1 == P.act_chunks ? 0 : icw + 1) {
        const int ic = kReuse ? icw : c;
        const int s = (int)(i & smask);
        const int b = c * W + cw;
        if (b < nb && !(ready & (1u << c)) && !ensure_block<T>(P, act, D, cw, W, lane, tag, so, c, ic, ready))
          return;
        if (!pwait(&m.full[s], (unsigned)((i >> lgS) & 1), P, tag)) return;
        if (b >= nb) {  // the group's last chunk is short
          mbar_arrive_warp(&m.empty[s]);
          continue;
        }
        // the slot is released after the integer core has used every loaded
        // register (the arrive follows their last use in program order)
        const uint8_t* tile = m.ring + (size_t)s * stage_bytes + (size_t)cw * kTileBytes;
        if constexpr (T == 8) {
          // 8 tokens: mma.sync m16n8k32 with N = the tokens, 2.3x fewer cycles
          // per tile than the dp4a core on B200, the same terms bit for bit
          if (nchunks > 1 || !fr_loaded) {
            load_act8_frag(act, act_slot(cw, W, T, ic, 0), W, lane, fr);
            fr_loaded = true;
          }
          block_terms_mma8(tile, fr, act, act_slot(cw, W, T, ic, 0), W, nb, b, terms, lane);
        } else {
          const WBlock wb = load_wblock(tile, lane);
          block_terms<T, false>(wb, act, act_slot(cw, W, T, ic, 0), W, nb, b, terms, lane, row, D.n_rows, nullptr,
                                nullptr);
        }
        mbar_arrive_warp(&m.empty[s]);
      }
      mbar_arrive_warp(&m.grp[buf]);
    }
  }
}

// Final output of a phase on every rank: its tagged (global) words of the
// launch that just completed, as plain floats (bounded wait for the words
// other ranks store).
__global__ void q2k_program_gather_kernel(const uint64_t* src, int64_t ld_src, int64_t rows, int T, float* dst,
                                          int64_t ldd, const unsigned* ctl, int64_t set_bytes, int sys,
                                          uint64_t timeout_ns, unsigned* err) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * T) return;
  const unsigned tag = ld_relaxed_gpu(ctl);
  const int64_t t = i / rows, r = i - t * rows;
  const uint64_t* p = set_ptr(src, (int64_t)(tag & 1u) * set_bytes) + t * ld_src + r;
  uint64_t w = ll_ld_scoped(p, sys);
  if (!ll_has(w, tag)) {
    const uint64_t t0 = global_timer_ns();
    while (!ll_has(w, tag)) {
      if (global_timer_ns() - t0 > timeout_ns) {
        raise_device_error(err, kDevErrTimeout);
        return;
      }
      __nanosleep(128);
      w = ll_ld_scoped(p, sys);
    }
  }
  dst[t * ldd + r] = ll_val(w);
}

}  // namespace

struct Q2KProgram {
  uint32_t magic = kProgramMagic;
  int n_phases = 0;
  int n_copies = 0;
  int T = 0;
  int nb_max = 0;
  int consumers = 0;
  int stages = 0;
  int tbufs = 2;
  int act_chunks = 1;
  int l2_ahead = 0;
  int grid = 0;
  size_t smem = 0;
  float eps = 0.f;
  int device = 0;
  int rank = 0, world = 1;
  PhaseDev* d_phases = nullptr;
  CopyDev* d_copies = nullptr;
  unsigned* d_ctl = nullptr;
  uint64_t* d_ll = nullptr;  // both sets of the phases' tagged outputs (same layout on every rank)
  size_t set_bytes = 0;
  uint64_t* d_ext = nullptr; // tagged copies of outside inputs (this GPU's own)
  size_t ext_bytes = 0;
  std::vector<PhaseDev> host_phases;
  std::vector<int64_t> out_rows_global;
  int n_peers = 0;
  int64_t peer_delta[kMaxPeers] = {};
  void* peer_base[kMaxPeers] = {};
  bool connected = true;
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

int64_t round_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

// Where a phase's fp32 input or residual comes from: rows r0.. of phase
// src's tagged (global) output, or an outside input (ext >= 0).
struct Source {
  int src = -1;
  int64_t r0 = 0;
  int ext = -1;
};

struct Ext {
  const float* ptr;
  int64_t ld, len;
  bool sums;
  int64_t off_ll = 0, off_sums = 0, ld_ll = 0, ld_sums = 0;  // word offsets in a set
};

// One phase with its wiring resolved.
struct Spec {
  const Q2KWeight* w;
  int in_mode, epi;
  const uint8_t* xq;     // kInQ8K input (caller memory)
  Source x, r;
  const float* norm_w;
  float* y;
  int64_t ldy;
  int64_t out_local;     // local output rows
  int64_t out_global;    // rows of the tagged output
  int64_t ex_lo, ex_hi, ex_row0;
};

int add_ext(std::vector<Ext>& ext, const float* ptr, int64_t ld, int64_t len, bool sums) {
  for (size_t e = 0; e < ext.size(); ++e)
    if (ext[e].ptr == ptr && ext[e].ld == ld && ext[e].len == len) {
      ext[e].sums = ext[e].sums || sums;
      return (int)e;
    }
  ext.push_back(Ext{ptr, ld, len, sums});
  return (int)ext.size() - 1;
}

// Checks common to both front ends, then device state, descriptors and the
// launch shape.
int build_program(std::vector<Spec>& sp, std::vector<Ext>& ext, int T, float eps, int dev, int rank, int world,
                  Q2KProgram** out) {
  const int n = (int)sp.size();
  int nb_max = 0;
  std::vector<char> need_sums((size_t)n, 0);
  for (int p = 0; p < n; ++p) {
    const Spec& s = sp[(size_t)p];
    nb_max = nb_max > s.w->nb ? nb_max : s.w->nb;
    if (s.in_mode == kInF32Rms && s.x.src >= 0) {
      const Spec& q = sp[(size_t)s.x.src];
      if (q.epi == kEpiSiluMul || s.x.r0 % 32 || q.ex_lo % 32 || q.ex_row0 % 32) {
        set_last_error("q2k_program: phase %d: an RMSNorm input must be a 32-row aligned slice of a store or "
                       "residual output", p);
        return kBadArgument;
      }
      need_sums[(size_t)s.x.src] = 1;
    }
    for (const Source* src : {&s.x, &s.r}) {
      if (src->src < 0) continue;
      if (src->src >= p) {
        set_last_error("q2k_program: phase %d reads phase %d, which does not run before it", p, src->src);
        return kBadArgument;
      }
    }
    if (s.x.src >= 0 && (s.x.r0 < 0 || s.x.r0 % 32 || s.x.r0 + s.w->k > sp[(size_t)s.x.src].out_global)) {
      set_last_error("q2k_program: phase %d: input rows [%lld, +%lld) are not a 32-row aligned slice of phase "
                     "%d's output", p, (long long)s.x.r0, (long long)s.w->k, s.x.src);
      return kBadArgument;
    }
    if (s.epi == kEpiResidual && s.r.src >= 0 &&
        (s.r.r0 < 0 || s.r.r0 + s.out_local > sp[(size_t)s.r.src].out_global)) {
      set_last_error("q2k_program: phase %d: the residual lies outside phase %d's output", p, s.r.src);
      return kBadArgument;
    }
  }

  // tagged buffers of one set (word offsets): phase outputs, their group
  // sums, the outside inputs (and their group sums)
  std::vector<int64_t> off_y((size_t)n), ld_yll((size_t)n), off_ys((size_t)n, -1), ld_ys((size_t)n, 0);
  int64_t words = 0;
  for (int p = 0; p < n; ++p) {
    ld_yll[(size_t)p] = round_up(sp[(size_t)p].out_global, 32);
    off_y[(size_t)p] = words;
    words += T * ld_yll[(size_t)p];
    if (need_sums[(size_t)p]) {
      ld_ys[(size_t)p] = round_up((sp[(size_t)p].out_global + 31) / 32, 2);
      off_ys[(size_t)p] = words;
      words += (int64_t)T * kSumReps * ld_ys[(size_t)p];
    }
  }
  const size_t set_bytes = (size_t)round_up(words * 8, 256);
  int64_t ewords = 0;
  for (Ext& e : ext) {
    e.ld_ll = round_up(e.len, 32);
    e.off_ll = ewords;
    ewords += T * e.ld_ll;
    if (e.sums) {
      e.ld_sums = round_up((e.len + 31) / 32, 2);
      e.off_sums = ewords;
      ewords += (int64_t)T * kSumReps * e.ld_sums;
    }
  }
  const size_t ext_bytes = (size_t)round_up((ewords > 0 ? ewords : 1) * 8, 256);

  // launch shape: 16 consumer warps (8 when the activation planes of 8 tokens
  // leave too little room); then, in this order of preference, two terms
  // buffers and a ring of at least 4 stages, two buffers and 2 stages, a
  // single buffer (8 tokens of a k = 11008 input); the deepest power-of-two
  // ring that fits
  int sms = 0, optin = 0;
  SMEAI_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  SMEAI_CUDA_TRY(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  int consumers = 0, stages = 0, tbufs = 0, act_chunks = 0;
  // chunk slots per warp: the widest phase's chunks (full), or -- for 8
  // tokens, when that does not fit the shape -- the same except plain fp32
  // inputs of phases with at most one row group per CTA (their blocks are
  // used once; the 8-token kernel reuses their slots)
  auto chunks_for = [&](int W, bool reuse) {
    int c = 1;
    for (const Spec& s : sp) {
      const int nch = (s.w->nb + W - 1) / W;
      const int need = (reuse && s.in_mode == kInF32 && s.w->n_groups <= sms) ? 1 : nch;
      c = c > need ? c : need;
    }
    return c;
  };
  static const int kShapes[3][2] = {{kMaxTbufs, 4}, {kMaxTbufs, 2}, {1, 2}};  // {tbufs, min stages}
  for (int W : {16, 8}) {
    for (const auto& sh : kShapes) {
      for (bool reuse : {false, true}) {
        if (reuse && T != 8) continue;
        const int ac = chunks_for(W, reuse);
        for (int S = 8; S >= sh[1]; S >>= 1)
          if (prog_smem_bytes(T, nb_max, ac, S, W, sh[0]) <= (size_t)optin) {
            stages = S;
            break;
          }
        if (stages) {
          act_chunks = ac;
          break;
        }
      }
      if (stages) {
        tbufs = sh[0];
        break;
      }
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
  const size_t smem = prog_smem_bytes(T, nb_max, act_chunks, stages, consumers, tbufs);
  void* kern = nullptr;
  switch (T) {
    case 1: kern = reinterpret_cast<void*>(q2k_program_kernel<1>); break;
    case 2: kern = reinterpret_cast<void*>(q2k_program_kernel<2>); break;
    case 4: kern = reinterpret_cast<void*>(q2k_program_kernel<4>); break;
    default: kern = reinterpret_cast<void*>(q2k_program_kernel<8>); break;
  }
  SMEAI_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 0;
  SMEAI_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, (consumers + 3) * 32, smem));
  if (per_sm < 1) {
    set_last_error("q2k_program: the kernel cannot be resident (smem %zu)", smem);
    return kUnsupported;
  }
  Q2KProgram* pr = new Q2KProgram();
  pr->n_phases = n;
  pr->n_copies = (int)ext.size();
  pr->T = T;
  pr->nb_max = nb_max;
  pr->consumers = consumers;
  pr->stages = stages;
  pr->tbufs = tbufs;
  pr->act_chunks = act_chunks;
  // L2 prefetch distance in ring stages: SMEAI_PROGRAM_L2_AHEAD=n overrides
  // the default (for tuning sweeps)
  pr->l2_ahead = kDefaultL2Ahead;
  if (const char* e = getenv("SMEAI_PROGRAM_L2_AHEAD")) pr->l2_ahead = atoi(e) < 0 ? 0 : atoi(e);
  pr->grid = sms;  // one CTA per SM: every SM streams
  pr->smem = smem;
  pr->eps = eps;
  pr->device = dev;
  pr->rank = rank;
  pr->world = world;
  pr->connected = world == 1;
  pr->set_bytes = set_bytes;
  pr->ext_bytes = ext_bytes;
  if (device_malloc((void**)&pr->d_phases, sizeof(PhaseDev) * (size_t)n) != cudaSuccess ||
      device_malloc((void**)&pr->d_copies, sizeof(CopyDev) * (ext.empty() ? 1 : ext.size())) != cudaSuccess ||
      device_malloc((void**)&pr->d_ctl, sizeof(unsigned) * 4) != cudaSuccess ||
      device_malloc((void**)&pr->d_ll, 2 * set_bytes) != cudaSuccess ||
      device_malloc((void**)&pr->d_ext, ext_bytes) != cudaSuccess) {
    cudaGetLastError();
    q2k_program_free(pr);
    set_last_error("q2k_program: cudaMalloc failed");
    return kAllocFailed;
  }
  uint64_t* ll = pr->d_ll;
  uint64_t* el = pr->d_ext;
  std::vector<PhaseDev> hp((size_t)n);
  int64_t rot = 0;
  for (int p = 0; p < n; ++p) {
    const Spec& s = sp[(size_t)p];
    const Q2KWeight& w = *s.w;
    PhaseDev& d = hp[(size_t)p];
    d = PhaseDev{};
    d.tiles = w.tiles;
    d.in_mode = s.in_mode;
    d.norm_w = s.norm_w;
    d.y = s.y;
    d.ldy = s.ldy;
    d.y_ll = ll + off_y[(size_t)p];
    d.ld_yll = ld_yll[(size_t)p];
    if (off_ys[(size_t)p] >= 0) {
      d.ys_ll = ll + off_ys[(size_t)p];
      d.ld_ysll = ld_ys[(size_t)p];
    }
    d.n_rows = w.n_rows;
    d.n_groups = w.n_groups;
    d.ex_lo = s.ex_lo;
    d.ex_hi = s.ex_hi;
    d.ex_row0 = s.ex_row0;
    d.rot = rot % sms;
    rot += w.n_groups;
    d.nb = w.nb;
    d.epi = s.epi;
    if (s.in_mode == kInQ8K) {
      d.xq = s.xq;
    } else if (s.x.src >= 0) {
      d.x_ll = ll + off_y[(size_t)s.x.src] + s.x.r0;
      d.ld_xll = ld_yll[(size_t)s.x.src];
      if (s.in_mode == kInF32Rms) {
        d.xs_ll = ll + off_ys[(size_t)s.x.src] + s.x.r0 / 32;
        d.ld_xsll = ld_ys[(size_t)s.x.src];
      }
    } else {
      const Ext& e = ext[(size_t)s.x.ext];
      d.x_ext = 1;
      d.x_ll = el + e.off_ll;
      d.ld_xll = e.ld_ll;
      if (s.in_mode == kInF32Rms) {
        d.xs_ll = el + e.off_sums;
        d.ld_xsll = e.ld_sums;
      }
    }
    if (s.epi == kEpiResidual) {
      if (s.r.src >= 0) {
        d.r_ll = ll + off_y[(size_t)s.r.src] + s.r.r0;
        d.ld_rll = ld_yll[(size_t)s.r.src];
      } else {
        d.r_ext = 1;
        d.r_ll = el + ext[(size_t)s.r.ext].off_ll + s.r.r0;
        d.ld_rll = ext[(size_t)s.r.ext].ld_ll;
      }
    }
  }
  std::vector<CopyDev> hc(ext.size());
  for (size_t e = 0; e < ext.size(); ++e) {
    CopyDev& c = hc[e];
    c.src = ext[e].ptr;
    c.ld_src = ext[e].ld;
    c.dst = el + ext[e].off_ll;
    c.ld_dst = ext[e].ld_ll;
    c.sums = ext[e].sums ? el + ext[e].off_sums : nullptr;
    c.ld_sums = ext[e].ld_sums;
    c.len = ext[e].len;
    c.units = (int64_t)T * ((ext[e].len + 31) / 32);
  }
  if (cudaMemcpy(pr->d_phases, hp.data(), sizeof(PhaseDev) * (size_t)n, cudaMemcpyHostToDevice) != cudaSuccess ||
      (!hc.empty() &&
       cudaMemcpy(pr->d_copies, hc.data(), sizeof(CopyDev) * hc.size(), cudaMemcpyHostToDevice) != cudaSuccess) ||
      cudaMemset(pr->d_ctl, 0, sizeof(unsigned) * 4) != cudaSuccess ||
      cudaMemset(pr->d_ll, 0, 2 * set_bytes) != cudaSuccess || cudaMemset(pr->d_ext, 0, ext_bytes) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess) {
    const cudaError_t e = cudaGetLastError();
    q2k_program_free(pr);
    set_last_error("q2k_program: %s", cudaGetErrorString(e));
    return kCudaError;
  }
  pr->host_phases = hp;
  for (const Spec& s : sp) pr->out_rows_global.push_back(s.out_global);
  *out = pr;
  return kOk;
}

int check_phase_common(int p, const Q2KWeight* w, int dev, int in_mode, int epi, const float* norm_w) {
  if (!w || !w->tiles || w->device != dev || w->fmt != kFmtQ2K) {
    set_last_error("q2k_program: phase %d: missing weight (or a weight on another device, or not Q2_K)", p);
    return kBadArgument;
  }
  if (in_mode != kInQ8K && in_mode != kInF32 && in_mode != kInF32Rms) {
    set_last_error("q2k_program: phase %d: unknown input mode %d", p, in_mode);
    return kBadArgument;
  }
  if (norm_w && (in_mode != kInF32Rms || (reinterpret_cast<uintptr_t>(norm_w) & 15))) {
    set_last_error("q2k_program: phase %d: an RMSNorm weight needs the RMS input mode and 16-byte alignment", p);
    return kBadArgument;
  }
  if (epi != kEpiStore && epi != kEpiResidual && epi != kEpiSiluMul) {
    set_last_error("q2k_program: phase %d: unknown epilogue %d", p, epi);
    return kBadArgument;
  }
  if (epi == kEpiSiluMul && (w->n_rows & 1)) {
    set_last_error("q2k_program: phase %d: silu*mul needs interleaved (gate, up) row pairs", p);
    return kBadArgument;
  }
  return kOk;
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
  for (int p = 0; p < n; ++p) {
    const ProgPhase& s = phases[p];
    int st = check_phase_common(p, s.w, dev, s.in_mode, s.epi, s.norm_w);
    if (st) return st;
    if (!s.x || !s.y) {
      set_last_error("q2k_program: phase %d: missing input or output", p);
      return kBadArgument;
    }
    const Q2KWeight& w = *s.w;
    if (s.in_mode == kInQ8K ? (reinterpret_cast<uintptr_t>(s.x) & 3) != 0 : (s.ld_x < w.k)) {
      set_last_error("q2k_program: phase %d: Q8_K input must be 4-byte aligned; fp32 input needs ld_x >= k", p);
      return kBadArgument;
    }
    if (s.epi == kEpiResidual && !s.resid) {
      set_last_error("q2k_program: phase %d: residual epilogue needs a residual pointer", p);
      return kBadArgument;
    }
    out_rows[(size_t)p] = s.epi == kEpiSiluMul ? w.n_rows / 2 : w.n_rows;
    if (s.ldy < out_rows[(size_t)p] || (s.epi == kEpiResidual && s.ld_resid < out_rows[(size_t)p])) {
      set_last_error("q2k_program: phase %d: leading dimension smaller than the output rows", p);
      return kBadArgument;
    }
    yr[(size_t)p] = rows_range(s.y, s.ldy, T, out_rows[(size_t)p], 4);
  }

  // Where each fp32 input and residual comes from: the latest earlier phase
  // whose output overlaps it (it must then be a slice of that output with the
  // same token stride), or the caller's memory before the launch.
  std::vector<Ext> ext;
  auto find_src = [&](int p, const void* ptr, int64_t ld, int64_t len, bool rms, const char* what,
                      Source& src) -> int {
    const Range want = rows_range(ptr, ld, T, len, 4);
    for (int q = p - 1; q >= 0; --q) {
      if (!yr[(size_t)q].overlaps(want)) continue;
      const ProgPhase& sq = phases[q];
      const intptr_t off = reinterpret_cast<intptr_t>(ptr) - reinterpret_cast<intptr_t>(sq.y);
      if (ld != sq.ldy || off < 0 || off % 128 || off / 4 + len > out_rows[(size_t)q] ||
          (rms && sq.epi == kEpiSiluMul)) {
        set_last_error("q2k_program: phase %d: a %s written by phase %d must be a 32-row aligned slice of its "
                       "output with the same row stride (and, for an RMSNorm input, not a silu*mul output)",
                       p, what, q);
        return kBadArgument;
      }
      src.src = q;
      src.r0 = off / 4;
      return kOk;
    }
    src.ext = add_ext(ext, static_cast<const float*>(ptr), ld, len, rms);
    return kOk;
  };
  std::vector<Spec> sp((size_t)n);
  for (int p = 0; p < n; ++p) {
    const ProgPhase& s = phases[p];
    const Q2KWeight& w = *s.w;
    Spec& d = sp[(size_t)p];
    d = Spec{};
    d.w = s.w;
    d.in_mode = s.in_mode;
    d.epi = s.epi;
    d.norm_w = s.norm_w;
    d.y = s.y;
    d.ldy = s.ldy;
    d.out_local = d.out_global = out_rows[(size_t)p];
    d.ex_lo = 0;
    d.ex_hi = out_rows[(size_t)p];
    d.ex_row0 = 0;
    if (s.in_mode != kInQ8K) {
      int st = find_src(p, s.x, s.ld_x, w.k, s.in_mode == kInF32Rms, "input", d.x);
      if (st) return st;
    } else {
      d.xq = static_cast<const uint8_t*>(s.x);
      const Range q8 = rows_range(s.x, w.nb * (int64_t)Q8K_BLOCK_BYTES, T, w.nb * (int64_t)Q8K_BLOCK_BYTES, 1);
      for (int q = 0; q < n; ++q)
        if (yr[(size_t)q].overlaps(q8)) {
          set_last_error("q2k_program: phase %d's Q8_K input overlaps phase %d's output", p, q);
          return kBadArgument;
        }
    }
    if (s.epi == kEpiResidual) {
      int st = find_src(p, s.resid, s.ld_resid, out_rows[(size_t)p], false, "residual", d.r);
      if (st) return st;
    }
    if (s.norm_w) {
      const Range nw = rows_range(s.norm_w, 0, 1, w.k, 4);
      for (int q = 0; q < n; ++q)
        if (yr[(size_t)q].overlaps(nw)) {
          set_last_error("q2k_program: phase %d's RMSNorm weight overlaps phase %d's output", p, q);
          return kBadArgument;
        }
    }
  }
  return build_program(sp, ext, T, eps, dev, 0, 1, out);
}

int q2k_mg_program_create(const MGPhase* phases, int n_phases, int n_cols, float eps, int rank, int world,
                          Q2KProgram** out) {
  if (!phases || !out || n_phases <= 0 || n_phases > (1 << 20) || world < 1 || world > kMaxPeers ||
      rank < 0 || rank >= world) {
    set_last_error("q2k_mg_program: bad arguments (1 <= world <= %d)", kMaxPeers);
    return kBadArgument;
  }
  *out = nullptr;
  const int T = n_cols;
  if (T != 1 && T != 2 && T != 4 && T != 8) {
    set_last_error("q2k_mg_program: n_cols must be 1, 2, 4 or 8 (got %d)", n_cols);
    return kBadArgument;
  }
  int dev = 0;
  SMEAI_CUDA_TRY(cudaGetDevice(&dev));
  std::vector<Ext> ext;
  std::vector<Spec> sp((size_t)n_phases);
  for (int p = 0; p < n_phases; ++p) {
    const MGPhase& s = phases[p];
    int st = check_phase_common(p, s.w, dev, s.in_mode, s.epi, s.norm_w);
    if (st) return st;
    if (s.in_mode == kInQ8K) {
      set_last_error("q2k_mg_program: phase %d: the multi-GPU program takes fp32 inputs", p);
      return kBadArgument;
    }
    const Q2KWeight& w = *s.w;
    Spec& d = sp[(size_t)p];
    d = Spec{};
    d.w = s.w;
    d.in_mode = s.in_mode;
    d.epi = s.epi;
    d.norm_w = s.norm_w;
    d.y = s.y;
    d.ldy = s.ldy;
    d.out_local = s.epi == kEpiSiluMul ? w.n_rows / 2 : w.n_rows;
    d.out_global = s.out_rows;
    d.ex_lo = s.ex_lo;
    d.ex_hi = s.ex_hi;
    d.ex_row0 = s.ex_row0;
    if (!s.y || s.ldy < d.out_local || s.ex_lo < 0 || s.ex_hi > d.out_local || s.ex_lo > s.ex_hi ||
        s.ex_row0 < 0 || s.ex_row0 + (s.ex_hi - s.ex_lo) > s.out_rows || s.ex_lo % 16 || s.ex_row0 % 16) {
      set_last_error("q2k_mg_program: phase %d: bad output (local rows [ex_lo, ex_hi) must map inside the "
                     "%lld global rows, 16-row aligned)", p, (long long)s.out_rows);
      return kBadArgument;
    }
    if (s.x_src >= 0) {
      d.x.src = s.x_src;
      d.x.r0 = s.x_row0;
    } else {
      if (!s.x || s.ld_x < w.k) {
        set_last_error("q2k_mg_program: phase %d: an outside input needs x with ld_x >= k", p);
        return kBadArgument;
      }
      d.x.ext = add_ext(ext, s.x, s.ld_x, w.k, s.in_mode == kInF32Rms);
    }
    if (s.epi == kEpiResidual) {
      if (s.r_src >= 0) {
        d.r.src = s.r_src;
        d.r.r0 = s.r_row0;
      } else {
        if (!s.resid || s.ld_resid < s.r_row0 + d.out_local) {
          set_last_error("q2k_mg_program: phase %d: an outside residual needs resid rows covering the output", p);
          return kBadArgument;
        }
        // the whole residual row is copied; the phase reads from r_row0 on
        d.r.ext = add_ext(ext, s.resid, s.ld_resid, s.r_row0 + d.out_local, false);
        d.r.r0 = s.r_row0;
      }
    }
  }
  return build_program(sp, ext, T, eps, dev, rank, world, out);
}

int q2k_program_ipc_handle(Q2KProgram* pr, void* handle64) {
  if (!pr || pr->magic != kProgramMagic || !handle64) {
    set_last_error("q2k_program_ipc_handle: bad arguments");
    return kBadArgument;
  }
  cudaIpcMemHandle_t h;
  SMEAI_CUDA_TRY(cudaIpcGetMemHandle(&h, pr->d_ll));
  memcpy(handle64, &h, sizeof(h) < 64 ? sizeof(h) : 64);
  return kOk;
}

int q2k_program_connect(Q2KProgram* pr, const void* handles, int world) {
  if (!pr || pr->magic != kProgramMagic || !handles || world != pr->world) {
    set_last_error("q2k_program_connect: bad arguments (world must match the program's)");
    return kBadArgument;
  }
  const uint8_t* hb = static_cast<const uint8_t*>(handles);
  int k = 0;
  for (int q = 0; q < world; ++q) {
    if (q == pr->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, hb + (size_t)q * 64, sizeof(h));
    void* ptr = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      cudaGetLastError();
      for (int j = 0; j < k; ++j) cudaIpcCloseMemHandle(pr->peer_base[j]);
      pr->n_peers = 0;
      set_last_error("q2k_program_connect: mapping rank %d's buffers failed: %s", q, cudaGetErrorString(e));
      return kCudaError;
    }
    pr->peer_base[k] = ptr;
    pr->peer_delta[k] = reinterpret_cast<intptr_t>(ptr) - reinterpret_cast<intptr_t>(pr->d_ll);
    ++k;
  }
  pr->n_peers = k;
  pr->connected = true;
  return kOk;
}

int q2k_program_run(Q2KProgram* pr, cudaStream_t stream) {
  if (!pr || pr->magic != kProgramMagic) {
    set_last_error("q2k_program_run: not a program handle");
    return kBadArgument;
  }
  if (!pr->connected) {
    set_last_error("q2k_program_run: a multi-GPU program must be connected to its peers first");
    return kBadArgument;
  }
  ProgParams P;
  P.phases = pr->d_phases;
  P.copies = pr->d_copies;
  P.n_phases = pr->n_phases;
  P.n_copies = pr->n_copies;
  P.nb_max = pr->nb_max;
  P.eps = pr->eps;
  P.stages = pr->stages;
  P.log2_stages = 31 - __builtin_clz((unsigned)pr->stages);
  P.ctl = pr->d_ctl;
  P.err = device_error_ptr();
  if (!P.err) {
    set_last_error("q2k_program_run: device error word unavailable");
    return kCudaError;
  }
  P.timeout_ns = pr->world > 1 ? peer_wait_timeout_ns() : wait_timeout_ns();
  P.set_bytes = (int64_t)pr->set_bytes;
  P.tbufs = pr->tbufs;
  P.log2_tbufs = pr->tbufs == 4 ? 2 : (pr->tbufs == 2 ? 1 : 0);
  P.act_chunks = pr->act_chunks;
  P.l2_ahead = pr->l2_ahead;
  P.sys = pr->world > 1 ? 1 : 0;
  P.n_peers = pr->n_peers;
  for (int q = 0; q < kMaxPeers; ++q) P.peer_delta[q] = pr->peer_delta[q];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)pr->grid);
  cfg.blockDim = dim3((unsigned)((pr->consumers + 3) * 32));
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

int q2k_program_gather(Q2KProgram* pr, int phase, float* y, int64_t ldy, cudaStream_t stream) {
  if (!pr || pr->magic != kProgramMagic || phase < 0 || phase >= pr->n_phases || !y ||
      ldy < pr->out_rows_global[(size_t)phase]) {
    set_last_error("q2k_program_gather: bad arguments");
    return kBadArgument;
  }
  unsigned* err = device_error_ptr();
  if (!err) {
    set_last_error("q2k_program_gather: device error word unavailable");
    return kCudaError;
  }
  const PhaseDev& d = pr->host_phases[(size_t)phase];
  const int64_t rows = pr->out_rows_global[(size_t)phase];
  const int64_t n = rows * pr->T;
  q2k_program_gather_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(
      d.y_ll, d.ld_yll, rows, pr->T, y, ldy, pr->d_ctl, (int64_t)pr->set_bytes, pr->world > 1 ? 1 : 0,
      pr->world > 1 ? peer_wait_timeout_ns() : wait_timeout_ns(), err);
  SMEAI_CUDA_TRY(cudaGetLastError());
  return kOk;
}

int q2k_program_reset(Q2KProgram* pr, cudaStream_t stream) {
  if (!pr || pr->magic != kProgramMagic) {
    set_last_error("q2k_program_reset: not a program handle");
    return kBadArgument;
  }
  SMEAI_CUDA_TRY(cudaMemsetAsync(pr->d_ctl, 0, sizeof(unsigned) * 4, stream));
  SMEAI_CUDA_TRY(cudaMemsetAsync(pr->d_ll, 0, 2 * pr->set_bytes, stream));
  SMEAI_CUDA_TRY(cudaMemsetAsync(pr->d_ext, 0, pr->ext_bytes, stream));
  return kOk;
}

void q2k_program_free(Q2KProgram* pr) {
  if (!pr || pr->magic != kProgramMagic) return;
  for (int q = 0; q < pr->n_peers; ++q)
    if (pr->peer_base[q]) cudaIpcCloseMemHandle(pr->peer_base[q]);
  if (pr->d_phases) cudaFree(pr->d_phases);
  if (pr->d_copies) cudaFree(pr->d_copies);
  if (pr->d_ctl) cudaFree(pr->d_ctl);
  if (pr->d_ll) cudaFree(pr->d_ll);
  if (pr->d_ext) cudaFree(pr->d_ext);
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
