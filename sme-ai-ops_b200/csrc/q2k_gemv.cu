// q2k_gemv.cu -- Q2_K x Q8_K decode GEMV (1..8 activation rows), the
// HBM-bound core of the reference's Q2_K mul_mat (ggml_vec_dot_q2_K_q8_K /
// ggml_gemv_q2_K_8x8_q8_K, llama.cpp/doc/SME_Q2K_OPTIMIZATION.md:105-136).
//
// Persistent, TMA-fed design (one CTA per SM at most):
//   * weights live in the tile layout built by q2k_repack_kernel: one 2688-byte
//     tile per (32-row group, super-block), the tiles of a group contiguous;
//     a CTA owns a contiguous range of row groups, i.e. one contiguous span of
//     tiles;
//   * warp 0 is the producer: one lane streams the CTA's tiles into a ring of
//     up to 32 shared-memory stages with cp.async.bulk (the TMA engine),
//     completing on per-stage mbarriers.  It starts at kernel entry, before
//     griddepcontrol.wait, so the first ~86 KB per SM of this matrix stream in
//     while the previous kernel in the stream is still running;
//   * consumer warp w handles super-blocks b = w (mod 8) of every row group;
//     lane = row.  After griddepcontrol.wait it quantizes its own activation
//     blocks to Q8_K (fp32 input, optionally RMS-normalized; or stages ggml
//     Q8_K blocks) into 16-byte aligned shared-memory planes -- the same code
//     as the standalone quantizer, so the blocks are identical;
//   * integer core per (row, super-block): 2-bit quants masked in place into
//     dp4a.u32.s32, one accumulator per shift plane weighted by the 4-bit
//     scales, planes shifted back at the end -- exact, equal to ggml's isum;
//     the min term is dp2a on the Q8_K bsums;
//   * the float term fmaf(d_x*d, isum, -(d_x*dmin*summs)) of each super-block
//     goes to shared memory; when all warps have finished a row group one warp
//     sums the terms in ascending super-block order (the rounding sequence of
//     the CPU restatement of ggml's generic dot, so outputs are bit-identical)
//     and applies the epilogue: store, residual add, or silu(gate)*up over
//     interleaved (gate, up) row pairs;
//   * every wait is an mbarrier wait bounded by wall time: on expiry the
//     kernel records kDevErrTimeout in the device error word and returns (the
//     producer first waits, bounded, for its copies in flight).
#include "common.cuh"
#include "kernels.h"
#include "runtime.h"
#include "q8k_device.cuh"
#include "q2k_core.cuh"
#include "q3k_core.cuh"
#include "q6k_core.cuh"

#include <stdio.h>
#include <stdlib.h>

namespace smeai {

namespace {


constexpr int kMaxConsumers = 16;
constexpr int kMaxThreads = (kMaxConsumers + 1) * 32;

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait until *sig reaches (*epoch + 1) * count (wrap-safe); false on
// timeout, and false at once when this device's error word is already set: a
// step in which one wait gave up cannot complete, so every later wait of the
// step returns immediately instead of running out its own limit.
__device__ bool peer_wait(const unsigned* sig, const unsigned* epoch, unsigned count, const unsigned* err,
                          uint64_t timeout_ns) {
  const unsigned target = (ld_acquire_sys(epoch) + 1u) * count;
  const uint64_t t0 = now_ns();
  while ((int)(ld_acquire_sys(sig) - target) < 0) {
    if (*reinterpret_cast<const volatile unsigned*>(err)) return false;
    if (now_ns() - t0 > timeout_ns) return false;
    __nanosleep(64);
  }
  return true;
}
// Publish a CTA's finished row groups to every rank, once: the consumer warps'
// stores (to this GPU and the peers) are ordered by the mbarrier before the
// one system-scope fence and the signal increments (ng each).
__device__ __forceinline__ void peer_signal(const PeerExchange& ex, unsigned ng) {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  for (int q = 0; q < ex.n_sig; ++q)
    asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(ex.sig[q]), "r"(ng) : "memory");
}

struct GemvParams {
  const uint8_t* tiles;
  int nb;
  int64_t n_rows;
  int64_t n_groups;
  const void* x;     // Q8_K blocks (kInQ8K) or fp32 rows
  int64_t ld_x;      // fp32 row stride in floats
  float eps;         // RMSNorm epsilon (kInF32Rms)
  const float* norm_w;  // RMSNorm weight (kInF32Rms), or null
  float* y;
  int64_t ldy;
  const float* resid;
  int64_t ld_resid;
  int32_t* isum_out;
  int32_t* summs_out;
  unsigned* err;
  uint64_t timeout_ns;       // bounded waits on this GPU's own work
  uint64_t peer_timeout_ns;  // bounded wait on other GPUs' rows
  int stages;        // ring depth (a power of two)
  int log2_stages;
  PeerExchange ex;   // cross-GPU output exchange (n_dst = n_sig = 0 and no wait_sig: off)
};

// Shared-memory carve-up for T tokens (16-byte aligned pieces).
struct Smem {
  uint8_t* ring;   // [stages][consumers][tile bytes of the weight format]
  int4* qs;        // [T*nb][16]  256 int8 per block
  int* bs;         // [T*nb][8]   16 int16 bsums per block
  float* d;        // [T*nb]
  float* rsum;     // [T][8 nb + 1] RMS group sums (8 per super-block), then 1/rms
  float* terms;    // [2][T*nb][32]
  uint64_t* full;  // [stages]
  uint64_t* empty; // [stages]
  uint64_t* grp;   // [2] all consumer lanes finished a row group
  uint64_t* tfree; // [2] the finisher has consumed the terms buffer
  uint64_t* rms;   // [2] group sums written / 1/rms ready
  uint64_t* done;  // [1] every consumer warp has finished its row groups (peer signal)
};

__host__ __device__ __forceinline__ size_t align16(size_t v) { return (v + 15) & ~(size_t)15; }

__host__ __device__ __forceinline__ size_t smem_fixed_bytes(int T, int nb) {
  return align16((size_t)T * nb * 256) + align16((size_t)T * nb * 32) + align16((size_t)T * nb * 4) +
         align16((size_t)T * (8 * nb + 1) * 4) + align16((size_t)2 * T * nb * 128) + 8 * 7;
}
__host__ __device__ __forceinline__ size_t smem_total_bytes(int T, int nb, int stages, int consumers, int tile) {
  return (size_t)stages * consumers * tile + smem_fixed_bytes(T, nb) + (size_t)stages * 16;
}

__device__ __forceinline__ Smem carve(uint8_t* base, int T, int nb, int stages, int consumers, int tile) {
  Smem m;
  size_t o = 0;
  m.ring = base;
  o += (size_t)stages * consumers * tile;
  m.qs = reinterpret_cast<int4*>(base + o);
  o += align16((size_t)T * nb * 256);
  m.bs = reinterpret_cast<int*>(base + o);
  o += align16((size_t)T * nb * 32);
  m.d = reinterpret_cast<float*>(base + o);
  o += align16((size_t)T * nb * 4);
  m.rsum = reinterpret_cast<float*>(base + o);
  o += align16((size_t)T * (8 * nb + 1) * 4);
  m.terms = reinterpret_cast<float*>(base + o);
  o += align16((size_t)2 * T * nb * 128);
  m.full = reinterpret_cast<uint64_t*>(base + o);
  m.empty = m.full + stages;
  m.grp = m.empty + stages;
  m.tfree = m.grp + 2;
  m.rms = m.tfree + 2;
  m.done = m.rms + 2;
  return m;
}

// Ordered sum over super-blocks of one row group, then the epilogue.
template <int T, int EPI, bool PEER>
__device__ __forceinline__ void finish_group(const float* terms, int nb, int64_t group, int lane,
                                             const GemvParams& p) {
  if constexpr (EPI == kEpiSiluMul) {
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
        if (2 * orow < p.n_rows) {
          const float sg = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
          const float h = __fmul_rn(sg, u);
          p.y[t * p.ldy + orow] = h;
          if constexpr (PEER) {
            if (orow >= p.ex.row0)
              for (int q = 0; q < p.ex.n_dst; ++q) p.ex.dst[q][t * p.ex.ld_dst + (orow - p.ex.row0)] = h;
          }
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
      if (orow < p.n_rows) {
        if constexpr (EPI == kEpiResidual) s = __fadd_rn(p.resid[t * p.ld_resid + orow], s);
        p.y[t * p.ldy + orow] = s;
        if constexpr (PEER) {
          if (orow >= p.ex.row0)
            for (int q = 0; q < p.ex.n_dst; ++q) p.ex.dst[q][t * p.ex.ld_dst + (orow - p.ex.row0)] = s;
        }
      }
    }
  }
}

// F: the weight format (FmtQ2K, FmtQ3K in q3k_core.cuh) -- tile size, the
// lane's block load and the integer core; everything else is shared.  PEER:
// the cross-GPU exchange of p.ex is compiled in (a separate instance, so the
// single-GPU kernels carry none of its code).
template <class F, int T, int EPI, int IN, bool SUMS, bool PEER>
__global__ void __launch_bounds__(kMaxThreads) q2k_gemv_kernel(const GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kConsumers = (blockDim.x >> 5) - 1;
  const int nb = p.nb, S = p.stages, lgS = p.log2_stages, smask = S - 1;
  const int64_t C = gridDim.x;
  const int64_t g0 = (int64_t)blockIdx.x * p.n_groups / C, g1 = ((int64_t)blockIdx.x + 1) * p.n_groups / C;
  const int ng = (int)(g1 - g0);
  // a stage is one bulk copy of kConsumers consecutive super-blocks of one row
  // group (fewer in the group's last chunk); consumer warp w takes block w of it
  const int nchunks = (nb + kConsumers - 1) / kConsumers;
  const int n_stages = ng * nchunks;
  constexpr int kTile = F::kTile;
  const int stage_bytes = kConsumers * kTile;
  const Smem m = carve(smem, T, nb, S, kConsumers, kTile);
  const ActSmem act = {m.qs, m.bs, m.d};

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&m.full[s], 1);
      mbar_init(&m.empty[s], kConsumers);
    }
    mbar_init(&m.grp[0], kConsumers);
    mbar_init(&m.grp[1], kConsumers);
    mbar_init(&m.tfree[0], 1);
    mbar_init(&m.tfree[1], 1);
    mbar_init(&m.rms[0], kConsumers);
    mbar_init(&m.rms[1], 1);
    mbar_init(&m.done[0], kConsumers);
    mbar_fence_init();
  }
  __syncthreads();
  pdl_trigger();

  if (warp == 0) {
    // ---- producer: stream this CTA's tiles (independent of earlier kernels)
    if (lane == 0) {
      const uint8_t* src = p.tiles + g0 * nb * (int64_t)kTile;
      int i = 0;
      bool ok = true;
      for (; i < n_stages; ++i) {
        const int s = i & smask;
        if (i >= S && !mbar_wait_or_error(&m.empty[s], (unsigned)(((i >> lgS) - 1) & 1), p.timeout_ns, p.err)) {
          ok = false;
          break;
        }
        const int j = i / nchunks, c = i - j * nchunks;
        const int nblk = min(kConsumers, nb - c * kConsumers);
        mbar_arrive_expect_tx(&m.full[s], (unsigned)(nblk * kTile));
        bulk_copy_g2s(m.ring + (size_t)s * stage_bytes, src + ((size_t)j * nb + (size_t)c * kConsumers) * kTile,
                      (unsigned)(nblk * kTile), &m.full[s]);
      }
      if (!ok) {
        raise_device_error(p.err, kDevErrTimeout);
        for (int j = (i > S ? i - S : 0); j < i; ++j)
          mbar_wait_bounded(&m.full[j & smask], (unsigned)((j >> lgS) & 1), p.timeout_ns);
      }
    }
    return;
  }

  // ---- consumers
  const int cw = warp - 1;
  pdl_wait();
  const bool peer_in = PEER && p.ex.wait_sig != nullptr;
  if (peer_in) {  // the input holds rows other GPUs store: wait for all of them
    int ok = 1;
    if (cw == 0 && lane == 0) {
      ok = peer_wait(p.ex.wait_sig, p.ex.epoch, p.ex.wait_count, p.err, p.peer_timeout_ns) ? 1 : 0;
      if (!ok) raise_device_error(p.err, kDevErrTimeout);
    }
    int all;  // the consumer warps meet (named barrier 1) and learn the waiter's result
    asm volatile(
        "{\n .reg .pred pi, po;\n setp.ne.s32 pi, %1, 0;\n bar.red.and.pred po, 1, %2, pi;\n"
        " selp.s32 %0, 1, 0, po;\n}"
        : "=r"(all)
        : "r"(ok), "r"(kConsumers * 32)
        : "memory");
    if (!all) return;
  }

  // activation prologue: this warp's own super-blocks b = cw (mod kConsumers)
  if constexpr (IN == kInQ8K) {
    const uint32_t* src = static_cast<const uint32_t*>(p.x);
    for (int b = cw; b < nb; b += kConsumers) {
#pragma unroll 1
      for (int t = 0; t < T; ++t)
        copy_q8k_smem(src + ((int64_t)t * nb + b) * Q8K_BLOCK_WORDS, act, t * nb + b, lane);
    }
  } else {
    const float* x = static_cast<const float*>(p.x);
    if constexpr (IN == kInF32Rms) {
      const int gs = 8 * nb + 1;  // group sums per token, then 1/rms
      for (int i = cw; i < T * nb; i += kConsumers) {
        const int t = i / nb, b = i - t * nb;
        float v[8];
        if (peer_in) load8_cg(x + t * p.ld_x + b * QK_K + lane * 8, v);
        else load8(x + t * p.ld_x + b * QK_K + lane * 8, v);
        const float s = group_sumsq_load8(v);
        if ((lane & 3) == 0) m.rsum[t * gs + b * 8 + (lane >> 2)] = s;
      }
      mbar_arrive_warp(&m.rms[0]);
      if (cw == 0) {
        if (!mbar_wait_bounded(&m.rms[0], 0, p.timeout_ns)) {
          raise_device_error(p.err, kDevErrTimeout);
          return;
        }
#pragma unroll 1
        for (int t = 0; t < T; ++t) {
          const float total = rms_fold_groups(m.rsum + t * gs, 8 * nb);
          if (lane == 0) m.rsum[t * gs + 8 * nb] = rms_inv_from_sum(total, nb * QK_K, p.eps);
        }
        mbar_arrive_warp(&m.rms[1]);
      }
      if (!mbar_wait_bounded(&m.rms[1], 0, p.timeout_ns)) {
        raise_device_error(p.err, kDevErrTimeout);
        return;
      }
    }
    for (int b = cw; b < nb; b += kConsumers) {
#pragma unroll 1
      for (int t = 0; t < T; ++t) {
        float v[8];
        if (peer_in) load8_cg(x + t * p.ld_x + b * QK_K + lane * 8, v);
        else load8(x + t * p.ld_x + b * QK_K + lane * 8, v);
        if constexpr (IN == kInF32Rms) {
          const float inv = m.rsum[t * (8 * nb + 1) + 8 * nb];
#pragma unroll
          for (int k = 0; k < 8; ++k) v[k] = __fmul_rn(v[k], inv);
          if (p.norm_w) {
            float g[8];
            load8(p.norm_w + b * QK_K + lane * 8, g);
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = __fmul_rn(v[k], g[k]);
          }
        }
        store_q8k_smem(q8k_quantize_lane(v), act, t * nb + b);
      }
    }
  }
  __syncwarp();

  // main loop over this CTA's row groups
  for (int j = 0; j < ng; ++j) {
    const int buf = j & 1;
    float* terms = m.terms + (size_t)buf * T * nb * 32;
    if (!SUMS && j >= 2 && !mbar_wait_bounded(&m.tfree[buf], (unsigned)(((j >> 1) - 1) & 1), p.timeout_ns)) {
      raise_device_error(p.err, kDevErrTimeout);
      return;
    }
    const int64_t group = g0 + j;
    const int64_t row = group * 32 + lane;
    for (int c = 0; c < nchunks; ++c) {
      const int i = j * nchunks + c;
      const int s = i & smask;
      const int b = c * kConsumers + cw;
      if (!mbar_wait_bounded(&m.full[s], (unsigned)((i >> lgS) & 1), p.timeout_ns)) {
        raise_device_error(p.err, kDevErrTimeout);
        return;
      }
      if (b >= nb) {  // the group's last chunk is short: nothing for this warp
        mbar_arrive_warp(&m.empty[s]);
        continue;
      }
      const uint8_t* tile = m.ring + (size_t)s * stage_bytes + (size_t)cw * kTile;
      if constexpr (std::is_same<F, FmtQ2K>::value && T == 8 && !SUMS) {
        // 8 tokens: the tile on mma.sync m16n8k32 (the same terms bit for bit,
        // 2.3x fewer cycles on B200); it reads the tile from shared memory,
        // so the slot is released after the core
        Act8Frag fr;
        load_act8_frag(act, b, nb, lane, fr);
        block_terms_mma8(tile, fr, act, b, nb, nb, b, terms, lane);
        mbar_arrive_warp(&m.empty[s]);
      } else {
        const typename F::Block wb = F::load(tile, lane);
        mbar_arrive_warp(&m.empty[s], F::dep(wb));
        F::template terms<T, SUMS>(wb, act, b, nb, nb, b, terms, lane, row, p.n_rows, p.isum_out, p.summs_out);
      }
    }
    if constexpr (!SUMS) {
      mbar_arrive_warp(&m.grp[buf]);
      if (cw == (j % kConsumers)) {
        if (!mbar_wait_bounded(&m.grp[buf], (unsigned)((j >> 1) & 1), p.timeout_ns)) {
          raise_device_error(p.err, kDevErrTimeout);
          return;
        }
        finish_group<T, EPI, PEER>(terms, nb, group, lane, p);
        mbar_arrive_warp(&m.tfree[buf]);
      }
    }
  }
  if constexpr (PEER) {
    // every group counts (its CTA no longer reads the input): one signal per CTA
    if (p.ex.n_sig) {
      mbar_arrive_warp(m.done);
      if (cw == 0 && lane == 0) {
        if (mbar_wait_bounded(m.done, 0u, p.timeout_ns)) peer_signal(p.ex, (unsigned)ng);
        else raise_device_error(p.err, kDevErrTimeout);
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

constexpr int kSmemLimit = 227 * 1024;

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 148;
    }
    cached[dev] = n;
  }
  return cached[dev];
}

struct Plan {
  int ctas_per_sm;
  int consumers;
  int stages;
};

// Launch shape of the GEMV for T tokens, nb super-blocks per row and
// n_groups 32-row groups (measured on B200, graph-timed, batch 1): below ~6
// groups per SM one CTA per SM with 16 consumer warps (a stage is then one
// 43 KB bulk copy -- large copies keep the TMA engine ahead); above it four
// CTAs per SM with 8 consumer warps.  The ring takes the deepest power of
// two that fits in the CTA's share of shared memory (half the SM for one CTA,
// so the next kernel's CTA can be resident during the tail).  The override
// SMEAI_GEMV_PLAN="ctas_per_sm,consumers,stages" exists for tuning sweeps.
Plan plan_for(int T, int nb, int64_t n_groups, int tile = kTileBytes) {
  const int sms = num_sms();
  Plan pl;
  if (n_groups < 6 * sms) pl = {1, 16, 0};
  else pl = {4, 8, 0};
  static int ov[3] = {-1, -1, -1};
  static bool read = false;
  if (!read) {
    read = true;
    const char* e = getenv("SMEAI_GEMV_PLAN");
    if (e) sscanf(e, "%d,%d,%d", &ov[0], &ov[1], &ov[2]);
  }
  if (ov[0] > 0) pl.ctas_per_sm = ov[0];
  if (ov[1] > 0 && ov[1] <= kMaxConsumers) pl.consumers = ov[1];
  const size_t fixed = smem_fixed_bytes(T, nb);
  const size_t budget = (size_t)kSmemLimit / (size_t)(pl.ctas_per_sm < 2 ? 2 : pl.ctas_per_sm);
  const size_t stage = (size_t)pl.consumers * tile + 16;
  const int cap = pl.ctas_per_sm == 1 ? 16 : 8;
  for (int s = cap; s >= 2; s >>= 1)
    if ((ov[2] <= 0 || s <= ov[2]) && fixed + (size_t)s * stage <= budget) {
      pl.stages = s;
      break;
    }
  // fallback: one CTA per SM with the whole shared memory, fewer consumer
  // warps when a stage of large tiles (Q6_K: 6784 bytes) leaves no room
  for (int c = pl.consumers; !pl.stages && c >= 4; c >>= 1)
    for (int s = 8; s >= 2; s >>= 1)
      if (fixed + (size_t)s * ((size_t)c * tile + 16) <= (size_t)kSmemLimit) {
        pl.stages = s;
        pl.consumers = c;
        pl.ctas_per_sm = 1;
        break;
      }
  return pl;
}

int plan_stages(int T, int nb, int tile) { return plan_for(T, nb, 1, tile).stages; }

template <class F, int T, int EPI, int IN, bool SUMS, bool PEER = false>
int launch_gemv(const Q2KWeight& w, GemvParams p, cudaStream_t stream) {
  auto kern = q2k_gemv_kernel<F, T, EPI, IN, SUMS, PEER>;
  const Plan pl = plan_for(T, w.nb, w.n_groups, F::kTile);
  if (pl.stages <= 0) {
    set_last_error("q2k_gemv: k=%lld too large for %d tokens per launch", (long long)w.k, T);
    return kBadArgument;
  }
  p.stages = pl.stages;
  p.log2_stages = 31 - __builtin_clz((unsigned)pl.stages);
  p.n_groups = w.n_groups;
  p.err = device_error_ptr();
  if (!p.err) {
    set_last_error("q2k_gemv: device error word unavailable");
    return kCudaError;
  }
  p.timeout_ns = wait_timeout_ns();
  p.peer_timeout_ns = peer_wait_timeout_ns();
  const size_t smem = smem_total_bytes(T, w.nb, pl.stages, pl.consumers, F::kTile);
  static unsigned configured = 0;  // per template instance, one bit per device
  int dev = 0;
  SMEAI_CUDA_TRY(cudaGetDevice(&dev));
  if (!(configured & (1u << (dev & 31)))) {
    SMEAI_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit));
    configured |= 1u << (dev & 31);
  }
  const int64_t max_ctas = (int64_t)num_sms() * pl.ctas_per_sm;
  const int64_t ctas = w.n_groups < max_ctas ? w.n_groups : max_ctas;
  SMEAI_CUDA_TRY(launch(kern, dim3((unsigned)ctas), dim3((pl.consumers + 1) * 32), smem, stream, p));
  return kOk;
}

template <class F, int EPI, int IN, bool PEER = false>
int dispatch_t(int T, const Q2KWeight& w, const GemvParams& p, cudaStream_t s) {
  switch (T) {
    case 1: return launch_gemv<F, 1, EPI, IN, false, PEER>(w, p, s);
    case 2: return launch_gemv<F, 2, EPI, IN, false, PEER>(w, p, s);
    case 4: return launch_gemv<F, 4, EPI, IN, false, PEER>(w, p, s);
    case 8: return launch_gemv<F, 8, EPI, IN, false, PEER>(w, p, s);
    default: return kBadArgument;
  }
}

template <int IN>
int dispatch_epi(int epi, int T, const Q2KWeight& w, const GemvParams& p, cudaStream_t s, bool peer = false) {
  if (w.fmt == kFmtQ3K || w.fmt == kFmtQ6K) {  // Q3_K / Q6_K weights: the store epilogue
    if (epi != kEpiStore) {
      set_last_error("gemv: only the store epilogue is built for Q3_K and Q6_K weights");
      return kBadArgument;
    }
    return w.fmt == kFmtQ3K ? dispatch_t<FmtQ3K, kEpiStore, IN>(T, w, p, s)
                            : dispatch_t<FmtQ6K, kEpiStore, IN>(T, w, p, s);
  }
  if constexpr (IN != kInQ8K) {
    if (peer) {
      switch (epi) {
        case kEpiStore: return dispatch_t<FmtQ2K, kEpiStore, IN, true>(T, w, p, s);
        case kEpiResidual: return dispatch_t<FmtQ2K, kEpiResidual, IN, true>(T, w, p, s);
        case kEpiSiluMul: return dispatch_t<FmtQ2K, kEpiSiluMul, IN, true>(T, w, p, s);
        default: break;
      }
    }
  }
  switch (epi) {
    case kEpiStore: return dispatch_t<FmtQ2K, kEpiStore, IN>(T, w, p, s);
    case kEpiResidual: return dispatch_t<FmtQ2K, kEpiResidual, IN>(T, w, p, s);
    case kEpiSiluMul: return dispatch_t<FmtQ2K, kEpiSiluMul, IN>(T, w, p, s);
    default:
      set_last_error("q2k_gemv: unknown epilogue %d", epi);
      return kBadArgument;
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
  if (device_malloc((void**)&tiles, bytes) != cudaSuccess) {
    cudaGetLastError();
    set_last_error("q2k_repack: cudaMalloc of %zu bytes failed", bytes);
    return kAllocFailed;
  }
  const int st = q2k_repack_into(w_blocks_dev, n_rows, k, tiles, out, stream);
  if (st != kOk) cudaFree(tiles);
  return st;
}

int q2k_gemv_any(const Q2KWeight& w, int in_mode, const void* x, int64_t ld_x, float eps, int64_t n_cols,
                 float* y, int64_t ldy, int epilogue, const float* resid, int64_t ld_resid, cudaStream_t stream,
                 const PeerExchange* ex, const float* norm_w) {
  if (!w.tiles || !x || !y || n_cols <= 0) {
    set_last_error("q2k_gemv: bad arguments");
    return kBadArgument;
  }
  if (ex) {
    const bool single = n_cols == 1 || n_cols == 2 || n_cols == 4 || n_cols == 8;
    if (!single || ex->n_dst < 0 || ex->n_dst > kMaxPeers || ex->n_sig < 0 || ex->n_sig > kMaxPeers ||
        (ex->wait_sig && (!ex->epoch || !ex->wait_count)) || in_mode == kInQ8K ||
        ex->row0 < 0 || ex->row0 % 16 || (ex->n_dst && ex->ld_dst <= 0)) {
      set_last_error("q2k_gemv: bad peer exchange (1/2/4/8 tokens, <= %d peers, fp32 input, "
                     "row0 a multiple of 16)", kMaxPeers);
      return kBadArgument;
    }
    for (int q = 0; q < ex->n_dst; ++q)
      if (!ex->dst[q]) {
        set_last_error("q2k_gemv: NULL peer destination %d", q);
        return kBadArgument;
      }
    for (int q = 0; q < ex->n_sig; ++q)
      if (!ex->sig[q]) {
        set_last_error("q2k_gemv: NULL peer signal %d", q);
        return kBadArgument;
      }
    if (w.fmt != kFmtQ2K) {
      set_last_error("q2k_gemv: the peer exchange is built for Q2_K weights");
      return kBadArgument;
    }
  }
  if (in_mode == kInQ8K && (reinterpret_cast<uintptr_t>(x) & 3)) {
    set_last_error("q2k_gemv: Q8_K activations must be 4-byte aligned");
    return kBadArgument;
  }
  if (in_mode != kInQ8K && ((reinterpret_cast<uintptr_t>(x) & 3) || ld_x < w.k)) {
    set_last_error("q2k_gemv: fp32 activations must be 4-byte aligned with ld_x >= k");
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
  for (int64_t c0 = 0; c0 < n_cols;) {
    const int64_t rem = n_cols - c0;
    int T = rem >= 8 ? 8 : (rem >= 4 ? 4 : (rem >= 2 ? 2 : 1));
    while (T > 1 && plan_stages(T, w.nb, fmt_tile_bytes(w.fmt)) <= 0) T >>= 1;
    GemvParams p = {};
    p.tiles = w.tiles;
    p.nb = w.nb;
    p.n_rows = w.n_rows;
    p.x = in_mode == kInQ8K ? static_cast<const void*>(static_cast<const uint8_t*>(x) +
                                                       c0 * (int64_t)w.nb * Q8K_BLOCK_BYTES)
                            : static_cast<const void*>(static_cast<const float*>(x) + c0 * ld_x);
    p.ld_x = ld_x;
    p.eps = eps;
    p.norm_w = in_mode == kInF32Rms ? norm_w : nullptr;
    p.y = y + c0 * ldy;
    p.ldy = ldy;
    p.resid = resid ? resid + c0 * ld_resid : nullptr;
    p.ld_resid = ld_resid;
    if (ex) p.ex = *ex;
    int st;
    switch (in_mode) {
      case kInQ8K: st = dispatch_epi<kInQ8K>(epilogue, T, w, p, stream); break;
      case kInF32: st = dispatch_epi<kInF32>(epilogue, T, w, p, stream, ex != nullptr); break;
      case kInF32Rms: st = dispatch_epi<kInF32Rms>(epilogue, T, w, p, stream, ex != nullptr); break;
      default:
        set_last_error("q2k_gemv: unknown input mode %d", in_mode);
        return kBadArgument;
    }
    if (st != kOk) return st;
    c0 += T;
  }
  return kOk;
}

namespace {
// The epoch advances only when the step completed: after a timeout the
// error word stays set and the step counter keeps its value, so late signals
// of the failed step can never satisfy a wait of the next one (the host must
// see the error and rebuild the exchange before running another step).
__global__ void peer_step_end_kernel(const unsigned* sig, unsigned count, unsigned* epoch, unsigned* err,
                                     uint64_t timeout_ns) {
  if (!peer_wait(sig, epoch, count, err, timeout_ns)) {
    raise_device_error(err, kDevErrTimeout);
    return;
  }
  *epoch = *epoch + 1u;
}
}  // namespace

int peer_step_end(const unsigned* sig, unsigned count, unsigned* epoch, cudaStream_t stream) {
  if (!sig || !epoch || !count) {
    set_last_error("peer_step_end: bad arguments");
    return kBadArgument;
  }
  unsigned* err = device_error_ptr();
  if (!err) {
    set_last_error("peer_step_end: device error word unavailable");
    return kCudaError;
  }
  peer_step_end_kernel<<<1, 1, 0, stream>>>(sig, count, epoch, err, peer_wait_timeout_ns());
  SMEAI_CUDA_TRY(cudaGetLastError());
  return kOk;
}

int q2k_gemv(const Q2KWeight& w, const void* xq, int64_t n_cols, float* y, int64_t ldy, int epilogue,
             const float* resid, int64_t ld_resid, cudaStream_t stream) {
  return q2k_gemv_any(w, kInQ8K, xq, 0, 0.f, n_cols, y, ldy, epilogue, resid, ld_resid, stream);
}

int q2k_block_sums(const Q2KWeight& w, const void* xq, int32_t* isum, int32_t* summs, cudaStream_t stream) {
  if (!w.tiles || !xq || !isum || !summs) {
    set_last_error("q2k_block_sums: bad arguments");
    return kBadArgument;
  }
  GemvParams p = {};
  p.tiles = w.tiles;
  p.nb = w.nb;
  p.n_rows = w.n_rows;
  p.x = xq;
  p.isum_out = isum;
  p.summs_out = summs;
  if (w.fmt == kFmtQ3K) return launch_gemv<FmtQ3K, 1, kEpiStore, kInQ8K, true, false>(w, p, stream);
  if (w.fmt == kFmtQ6K) return launch_gemv<FmtQ6K, 1, kEpiStore, kInQ8K, true, false>(w, p, stream);
  return launch_gemv<FmtQ2K, 1, kEpiStore, kInQ8K, true, false>(w, p, stream);
}

}  // namespace smeai
