// q2k_gemm_tc.cu -- Q2_K x Q8_K prefill GEMM on the sm_100a tensor cores
// (tcgen05.mma with TMEM accumulators): the M > 8 case of the reference's Q2_K
// mul_mat (ggml_gemm_q2_K_8x8_q8_K, llama.cpp/doc/SME_Q2K_OPTIMIZATION.md:105-113).
//
// Exactness: the operands are small integers.  The 16 sub-block products
// run as tcgen05.mma kind::i8 -- A = scale * q2 as u8 (0..45), B = the Q8_K
// quants as s8 -- into s32 TMEM accumulators, exact by construction; the
// min term runs as one kind::f16 MMA on values held exactly in fp16 (Q8_K
// bsums in [-2032, 2032], 4-bit mins in [0, 15], every partial sum an
// integer below 2^24) into an fp32 accumulator:
//   D1[n][m] = isum  = sum_i (scale_j(i) * q2_i) * q8_i   (8 i8 MMAs, K = 256)
//   D2[n][m] = summs = sum_j min_j * bsums_j             (1 f16 MMA, K = 16)
// -- the integers ggml's generic dot computes.  The epilogue then applies
// ggml's combine per super-block,
//   acc += fmaf(d_x*d, isum, -(d_x*dmin*summs)),   super-blocks ascending,
// so the output equals the CPU restatement (and the GEMV) bit for bit.
//
// CTA tile: 128 weight rows (UMMA M, operand A) x 128 activation rows (UMMA N,
// operand B), looping over super-blocks.  Warp roles:
//   warp 0      producer: one lane issues cp.async.bulk copies -- the four
//               32-row Q2_K tiles of the super-block, the activation atoms and
//               bsums (pre-laid-out in UMMA order by gemm_prepass_kernel);
//   warp 1      allocates 512 TMEM columns; one lane issues the MMAs and the
//               tcgen05.commit arrivals;
//   warps 2-5   dequantize: thread = weight row; each 2-bit plane of 4 quants
//               masked and multiplied by its 4-bit scale in one 32-bit
//               multiply (4 u8 products, none above 45), written straight
//               into the 128-byte-swizzled K-major layout the MMA reads; the
//               16 mins as fp16;
//   warps 6-13  epilogue: drain the double-buffered TMEM accumulators
//               (tcgen05.ld), combine, accumulate in registers, store.
// Stages: A/B operand atoms for two super-blocks (a 128-row x 128-byte atom
// holds one 128-weight half), 2 super-block slots for raw Q2_K tiles and min
// operands, 2 TMEM accumulator buffers (D1 + D2 each).
// Every wait is an mbarrier wait bounded by wall time; on expiry the kernel
// records kDevErrTimeout, the roles stop, in-flight copies and MMAs are
// drained (bounded), TMEM is freed and the kernel returns.  No multicast.
#include "common.cuh"
#include "kernels.h"

namespace smeai {

namespace {

constexpr int kTM = 128;                        // weight rows per tile
constexpr int kTN = 128;                        // activation rows per tile
constexpr int kAtomBytes = 128 * 128;           // 128 rows x 128 B (128 int8 of K: one half super-block)
constexpr int kMinBytes = 128 * 32;             // 128 rows x 16 fp16
constexpr int kRawBytes = 4 * kTileBytes;       // four 32-row Q2_K tiles
#ifndef SMEAI_GEMM_DQ_WARPS
#define SMEAI_GEMM_DQ_WARPS 4
#endif
constexpr int kDqWarps = SMEAI_GEMM_DQ_WARPS;   // dequant warps: 4 row quarters x (1 or 2) K halves each
constexpr int kEpiWarp0 = 2 + kDqWarps;         // first epilogue warp
constexpr int kThreads = (kEpiWarp0 + 8) * 32;
constexpr int kTmemCols = 512;
constexpr uint64_t kTimeoutNs = 2000000000ull;

struct GemmParams {
  const uint8_t* tiles;   // Q2_K tile layout
  int nb;
  int64_t n_rows;
  int64_t n_groups;
  const uint8_t* bq;      // activation atoms [token tile][nb*2][kAtomBytes]
  const uint8_t* bs;      // bsums [token tile][nb][kMinBytes]
  const float* dx;        // [n_cols][nb]
  int64_t n_cols;
  float* y;
  int64_t ldy;
  int epi;                // kEpiStore, kEpiResidual (y = resid + acc), kEpiSiluMul (interleaved gate/up rows)
  const float* resid;
  int64_t ld_resid;
  unsigned* err;
  int raw_log2;           // log2 of the raw Q2_K tile slots (4, or 2 for a long k)
};

// ---- tcgen05 helpers ---------------------------------------------------------
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, int8 inputs, s32 accumulate.
__device__ __forceinline__ void tc_mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      :
      : "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, fp16 inputs, fp32 accumulate.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      :
      : "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// The same, naming the registers of the loads it completes, so that no use
// of them can be scheduled above the wait.
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&a)[16], uint32_t (&b)[16]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]), "+r"(a[8]),
        "+r"(a[9]), "+r"(a[10]), "+r"(a[11]), "+r"(a[12]), "+r"(a[13]), "+r"(a[14]), "+r"(a[15]), "+r"(b[0]),
        "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7]), "+r"(b[8]), "+r"(b[9]),
        "+r"(b[10]), "+r"(b[11]), "+r"(b[12]), "+r"(b[13]), "+r"(b[14]), "+r"(b[15])
      :
      : "memory");
}

// Packed fp32 pairs (two lanes of one 64-bit register, each op IEEE-rounded
// per lane exactly as the scalar op): half the instructions of the combine.
__device__ __forceinline__ uint64_t pack_f32x2(float lo, float hi) {
  return (uint64_t)__float_as_uint(lo) | ((uint64_t)__float_as_uint(hi) << 32);
}
__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// Shared-memory matrix descriptor (sm_100 format, version 1).
__device__ __forceinline__ uint64_t smem_desc(const void* p, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint32_t layout) {
  const uint32_t a = smem_addr(p);
  return (uint64_t)((a >> 4) & 0x3FFF) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}
constexpr uint32_t kLayoutSw128 = 2, kLayoutNone = 0;

// Instruction descriptors (both operands K-major, M = 128, N = 128):
// kind::f16 with fp16 A and B and an fp32 D (D format 1 at bit 4) ...
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kTN >> 3) << 17) | ((uint32_t)(kTM >> 4) << 24);
// ... and kind::i8 with signed A and B (format 1 at bits 7-9 and 10-12; A's
// values, 0..45, read the same either way) and an s32 D (format 2 at bit 4).
constexpr uint32_t kIdescI8 = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTN >> 3) << 17) |
                              ((uint32_t)(kTM >> 4) << 24);

// Byte offset of (row r, byte k) in one 128-row x 128-byte swizzled atom
// (the 16-byte chunks of a row XORed with the row's index mod 8).
__host__ __device__ __forceinline__ uint32_t sw128_off(uint32_t r, uint32_t k) {
  return r * 128u + ((((k >> 4) & 7u) ^ (r & 7u)) << 4) + (k & 15u);
}
// Byte offset of (row r, k < 16) in the no-swizzle K-major 128 x 16 fp16 tile:
// 8-row x 16-byte core matrices, K halves 128 B apart, 8-row groups 256 B apart.
__host__ __device__ __forceinline__ uint32_t min_off(uint32_t r, uint32_t k) {
  return (r & 7u) * 16u + (k >> 3) * 128u + (r >> 3) * 256u + (k & 7u) * 2u;
}

// fp16 pairs from two small non-negative integers in bytes 0,1 (sel 0x4140)
// or 2,3 (sel 0x4342) of v: 1024 + b exactly, minus 1024.
__device__ __forceinline__ uint32_t bytes_to_half2(uint32_t v, uint32_t sel) {
  const uint32_t packed = __byte_perm(v, 0x64646464u, sel);
  __half2 h = *reinterpret_cast<const __half2*>(&packed);
  h = __hsub2(h, __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400)));
  return *reinterpret_cast<uint32_t*>(&h);
}

struct GemmSmem {
  uint8_t* a;        // [4][kAtomBytes]  slot (b & 1) * 2 + half
  uint8_t* b;        // [4][kAtomBytes]
  uint8_t* a2;       // [2][kMinBytes]
  uint8_t* b2;       // [2][kMinBytes]
  uint8_t* raw;      // [raw slots][kRawBytes]
  float* sdx;        // [nb][kTN]
  uint64_t* full;    // [4]  per atom slot: dequant (128) + producer (1, tx)
  uint64_t* empty;   // [4]  per atom slot: commit
  uint64_t* rfull;   // [kMaxRaw]  producer (tx)
  uint64_t* rempty;  // [kMaxRaw]  dequant (128)
  uint64_t* mfull;   // [2]  dequant (128) + producer (1, tx)
  uint64_t* mempty;  // [2]  commit
  uint64_t* afull;   // [2]  commit
  uint64_t* aempty;  // [2]  epilogue (256)
  uint64_t* drain;   // [1]  commit (abort path)
  uint32_t* tmem;    // allocated TMEM base
  int* abort;
};

// Raw Q2_K tiles come from HBM: four super-blocks of them in flight keep the
// dequant warps fed across the load latency; two when four do not fit (k
// above 20224).
constexpr int kMaxRaw = 4;
size_t gemm_smem_bytes(int nb, int raw_slots) {
  return 1024 /* alignment slack */ + 8 * (size_t)kAtomBytes + 4 * (size_t)kMinBytes +
         (size_t)raw_slots * kRawBytes + (size_t)kTN * nb * 4 + 40 * 8 + 16;
}

__device__ __forceinline__ GemmSmem carve_gemm(uint8_t* base, int nb, int raw_slots) {
  GemmSmem m;
  uint8_t* p = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(base) + 1023) & ~(uintptr_t)1023);
  m.a = p;
  p += 4 * kAtomBytes;
  m.b = p;
  p += 4 * kAtomBytes;
  m.a2 = p;
  p += 2 * kMinBytes;
  m.b2 = p;
  p += 2 * kMinBytes;
  m.raw = p;
  p += (size_t)raw_slots * kRawBytes;
  m.sdx = reinterpret_cast<float*>(p);
  p += (size_t)kTN * nb * 4;
  uint64_t* bars = reinterpret_cast<uint64_t*>(p);
  m.full = bars;
  m.empty = bars + 4;
  m.rfull = bars + 8;
  m.rempty = m.rfull + kMaxRaw;
  m.mfull = m.rempty + kMaxRaw;
  m.mempty = m.mfull + 2;
  m.afull = m.mempty + 2;
  m.aempty = m.afull + 2;
  m.drain = m.aempty + 2;
  m.tmem = reinterpret_cast<uint32_t*>(m.drain + 1);
  m.abort = reinterpret_cast<int*>(m.drain + 2);
  return m;
}

// Bounded wait that also gives up once another role has aborted.
__device__ __forceinline__ bool wait_or_abort(const GemmSmem& m, uint64_t* bar, unsigned parity, unsigned* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*reinterpret_cast<volatile int*>(m.abort)) return false;
    if (global_timer_ns() - t0 > kTimeoutNs) {
      *reinterpret_cast<volatile int*>(m.abort) = 1;
      raise_device_error(err, kDevErrTimeout);
      return false;
    }
  }
}

// The same for a whole warp: every lane waits (each acquires the phase for
// its own reads), and the warp leaves together if any lane gave up, so the
// warp-collective operations after it (tcgen05.ld, one-arrival-per-warp
// barriers) always run converged.
__device__ __forceinline__ bool wait_warp(const GemmSmem& m, uint64_t* bar, unsigned parity, unsigned* err) {
  return __all_sync(0xffffffffu, wait_or_abort(m, bar, parity, err));
}

__global__ void __launch_bounds__(kThreads, 1) q2k_gemm_tc_kernel(const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = p.nb;
  const int64_t row_tile = blockIdx.x, tok_tile = blockIdx.y;
  const int64_t n0 = row_tile * kTM, m0 = tok_tile * kTN;
  const int RL = p.raw_log2, RS = 1 << RL;
  const GemmSmem m = carve_gemm(smem_raw, nb, RS);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 4; ++i) {
      mbar_init(&m.full[i], 128 + 1);  // the 4 dequant warps of the atom's half + the producer
      mbar_init(&m.empty[i], 1);
    }
    for (int i = 0; i < kMaxRaw; ++i) {
      mbar_init(&m.rfull[i], 1);
      mbar_init(&m.rempty[i], 32 * kDqWarps);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&m.mfull[i], 32 * kDqWarps + 1);
      mbar_init(&m.mempty[i], 1);
      mbar_init(&m.afull[i], 1);
      mbar_init(&m.aempty[i], 256);
    }
    mbar_init(m.drain, 1);
    *m.abort = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(m.tmem)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  pdl_trigger();
  pdl_wait();   // the activation operands come from the prepass kernel
  // activation scales of this tile: sdx[block][token] (0 past the last token)
  if (warp >= kEpiWarp0) {
    for (int i = threadIdx.x - kEpiWarp0 * 32; i < kTN * nb; i += 8 * 32) {
      const int64_t tok = m0 + i / nb;
      m.sdx[(i % nb) * kTN + i / nb] = tok < p.n_cols ? p.dx[tok * nb + (i % nb)] : 0.f;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *m.tmem;

  if (warp == 0) {
    // ---------------- producer
    if (lane == 0) {
      int issued_raw[kMaxRaw] = {-1, -1, -1, -1}, issued_m[2] = {-1, -1}, issued_b[4] = {-1, -1, -1, -1};
      for (int b = 0; b < nb; ++b) {
        const int r = b & 1, rr = b & (RS - 1);
        if ((b >= RS && !wait_or_abort(m, &m.rempty[rr], ((b >> RL) - 1) & 1, p.err)) ||
            (b >= 2 && !wait_or_abort(m, &m.mempty[r], ((b >> 1) - 1) & 1, p.err)))
          break;
        int groups = 0;
        for (int gi = 0; gi < 4; ++gi)
          if (row_tile * 4 + gi < p.n_groups) ++groups;
        mbar_arrive_expect_tx(&m.rfull[rr], (unsigned)(groups * kTileBytes));
        for (int gi = 0; gi < groups; ++gi) {
          const int64_t g = row_tile * 4 + gi;
          bulk_copy_g2s(m.raw + rr * kRawBytes + gi * kTileBytes, p.tiles + (g * nb + b) * (int64_t)kTileBytes,
                        kTileBytes, &m.rfull[rr]);
        }
        issued_raw[rr] = b;
        mbar_arrive_expect_tx(&m.mfull[r], kMinBytes);
        bulk_copy_g2s(m.b2 + r * kMinBytes, p.bs + (tok_tile * nb + b) * (int64_t)kMinBytes, kMinBytes,
                      &m.mfull[r]);
        issued_m[r] = b;
        bool ok = true;
        for (int h = 0; h < 2; ++h) {
          const int sl = r * 2 + h;
          if (b >= 2 && !wait_or_abort(m, &m.empty[sl], ((b >> 1) - 1) & 1, p.err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&m.full[sl], kAtomBytes);
          bulk_copy_g2s(m.b + sl * kAtomBytes, p.bq + ((tok_tile * nb + b) * 2 + h) * (int64_t)kAtomBytes,
                        kAtomBytes, &m.full[sl]);
          issued_b[sl] = b;
        }
        if (!ok) break;
      }
      if (*reinterpret_cast<volatile int*>(m.abort)) {
        // drain: the last copy issued into each slot lands before we leave
        for (int rr = 0; rr < RS; ++rr)
          if (issued_raw[rr] >= 0) mbar_wait_bounded(&m.rfull[rr], (issued_raw[rr] >> RL) & 1, kTimeoutNs);
        for (int r = 0; r < 2; ++r)
          if (issued_m[r] >= 0) mbar_wait_bounded(&m.mfull[r], (issued_m[r] >> 1) & 1, kTimeoutNs);
        for (int sl = 0; sl < 4; ++sl)
          if (issued_b[sl] >= 0) mbar_wait_bounded(&m.full[sl], (issued_b[sl] >> 1) & 1, kTimeoutNs);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      const uint32_t lbo_sw = 16, sbo_sw = 1024;      // 8-row groups of 128-byte rows
      for (int b = 0; b < nb; ++b) {
        const int r = b & 1;
        if (b >= 2 && !wait_or_abort(m, &m.aempty[r], ((b >> 1) - 1) & 1, p.err)) break;
        tc_fence_after();
        const uint32_t d1 = tmem + (uint32_t)(r * 256), d2 = d1 + 128;
        bool ok = true;
        for (int h = 0; h < 2; ++h) {
          const int sl = r * 2 + h;
          if (!wait_or_abort(m, &m.full[sl], (b >> 1) & 1, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = smem_desc(m.a + sl * kAtomBytes, lbo_sw, sbo_sw, kLayoutSw128);
          const uint64_t db = smem_desc(m.b + sl * kAtomBytes, lbo_sw, sbo_sw, kLayoutSw128);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)   // 32 int8 of K = 32 bytes per MMA
            tc_mma_i8(d1, da + 2 * kk, db + 2 * kk, kIdescI8, (h | kk) != 0);
          tc_commit(&m.empty[sl]);
        }
        if (!ok || !wait_or_abort(m, &m.mfull[r], (b >> 1) & 1, p.err)) break;
        tc_fence_after();
        tc_mma_f16(d2, smem_desc(m.a2 + r * kMinBytes, 128, 256, kLayoutNone),
                   smem_desc(m.b2 + r * kMinBytes, 128, 256, kLayoutNone), kIdesc, 0);
        tc_commit(&m.mempty[r]);
        tc_commit(&m.afull[r]);
      }
      // every MMA issued by this thread has completed before TMEM is freed
      tc_commit(m.drain);
      mbar_wait_bounded(m.drain, 0, kTimeoutNs);
    }
  } else if (warp < kEpiWarp0) {
    // ---------------- dequantize: thread = (weight row, 128-weight half)
    const int dw = warp - 2;
    const int h0 = dw >> 2;                      // first K half (atom) this warp fills
    constexpr int kHStep = kDqWarps / 4;         // 1: both halves; 2: one half
    const int t = (dw & 3) * 32 + lane;          // weight row within the tile
    const int gi = t >> 5, l = t & 31;
    const bool present = row_tile * 4 + gi < p.n_groups;
    for (int b = 0; b < nb; ++b) {
      const int r = b & 1, rr = b & (RS - 1);
      if (!wait_warp(m, &m.rfull[rr], (b >> RL) & 1, p.err)) break;
      uint4 q[4], sc;
      if (present) {
        const uint8_t* tile = m.raw + rr * kRawBytes + gi * kTileBytes;
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if ((c >> 1) % kHStep == h0 % kHStep) q[c] = reinterpret_cast<const uint4*>(tile + c * 512)[l];
        sc = reinterpret_cast<const uint4*>(tile + 2048)[l];
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) q[c] = make_uint4(0, 0, 0, 0);
        sc = make_uint4(0, 0, 0, 0);
      }
      mbar_arrive(&m.rempty[rr]);
      const uint32_t scw[4] = {sc.x, sc.y, sc.z, sc.w};
      // this warp's halves' mins (8 each) into the no-swizzle 128 x 16 operand
      if (b >= 2 && !wait_warp(m, &m.mempty[r], ((b >> 1) - 1) & 1, p.err)) break;
      {
        uint8_t* dst = m.a2 + r * kMinBytes;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          if (hh % kHStep != h0 % kHStep) continue;
          uint32_t h[4];
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const uint32_t mins = (scw[2 * hh + k] >> 4) & 0x0F0F0F0Fu;
            h[2 * k] = bytes_to_half2(mins, 0x4140);
            h[2 * k + 1] = bytes_to_half2(mins, 0x4342);
          }
          *reinterpret_cast<uint4*>(dst + min_off(t, (uint32_t)(8 * hh))) = make_uint4(h[0], h[1], h[2], h[3]);
        }
        fence_async_smem();
        mbar_arrive(&m.mfull[r]);
      }
      // half hh = weights 128hh..128hh+127 (one atom): K byte 32s + l within
      // the atom for qs byte l of the half and shift plane s; each 32-bit
      // product is 4 bytes scale * q (no carry: at most 45)
      bool ok = true;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        if (hh % kHStep != h0 % kHStep) continue;
        const int sl = r * 2 + hh;
        if (b >= 2 && !wait_warp(m, &m.empty[sl], ((b >> 1) - 1) & 1, p.err)) {
          ok = false;
          break;
        }
        uint8_t* dst = m.a + sl * kAtomBytes;
#pragma unroll
        for (int s = 0; s < 4; ++s) {
#pragma unroll
          for (int part = 0; part < 2; ++part) {      // quants l = 16*part .. 16*part+15
            const uint4 qc = q[2 * hh + part];
            const int j = 8 * hh + 2 * s + part;       // sub-block
            const uint32_t scale = (scw[j >> 2] >> (8 * (j & 3))) & 0xFu;
            const uint4 v = make_uint4(((qc.x >> (2 * s)) & 0x03030303u) * scale,
                                       ((qc.y >> (2 * s)) & 0x03030303u) * scale,
                                       ((qc.z >> (2 * s)) & 0x03030303u) * scale,
                                       ((qc.w >> (2 * s)) & 0x03030303u) * scale);
            *reinterpret_cast<uint4*>(dst + sw128_off((uint32_t)t, (uint32_t)(32 * s + 16 * part))) = v;
          }
        }
        fence_async_smem();
        mbar_arrive(&m.full[sl]);
      }
      if (!ok) break;
    }
  } else {
    // ---------------- epilogue: 8 warps; TMEM lane quarter = warp % 4
    const int quarter = warp & 3;
    const int half = (warp - kEpiWarp0) >> 2;    // token columns half*64 .. +63
    const int t = quarter * 32 + lane;           // weight row within the tile
    const int64_t row = n0 + t;
    const int64_t g = row >> 5;
    uint64_t acc[32];                            // token pairs (2c, 2c+1)
#pragma unroll
    for (int c = 0; c < 32; ++c) acc[c] = 0ull;
    bool ok = true;
    // d|dmin of this row, one super-block ahead (the weights are read-only, so
    // the load goes out before the accumulator wait and its latency hides
    // behind the previous super-block's combine)
    const unsigned* dm_src = reinterpret_cast<const unsigned*>(p.tiles + g * nb * (int64_t)kTileBytes + 2560) +
                             (row & 31);
    const bool live_row = g < p.n_groups;
    unsigned dm_next = live_row ? __ldg(dm_src) : 0u;
    const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
    for (int b = 0; b < nb; ++b) {
      const int r = b & 1;
      const unsigned dm = dm_next;
      if (live_row && b + 1 < nb) dm_next = __ldg(dm_src + (int64_t)(b + 1) * (kTileBytes / 4));
      if (!wait_warp(m, &m.afull[r], (b >> 1) & 1, p.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float dw = __half2float(__ushort_as_half((unsigned short)(dm & 0xffffu)));
      const float dmw = __half2float(__ushort_as_half((unsigned short)(dm >> 16)));
      // term = fmaf(dx*d, isum, -(dx*dmin*summs)) per token, two tokens per
      // packed op; -(dx*dmin) is formed as dx*(-dmin) and -(p*summs) as
      // (-p)*summs, both exact negations of the rounded products
      const uint64_t dw2 = pack_f32x2(dw, dw), ndmw2 = pack_f32x2(-dmw, -dmw);
      const float* sdx = m.sdx + b * kTN + half * 64;
      const uint32_t col0 = (uint32_t)(r * 256 + half * 64);
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t vi[16], vm[16];
        tmem_ld16(lane_base + col0 + (uint32_t)(cc * 16), vi);
        tmem_ld16(lane_base + col0 + (uint32_t)(cc * 16) + 128, vm);
        tmem_ld_wait(vi, vm);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int c = cc * 8 + k;                // token pair
          const uint64_t dx2 = *reinterpret_cast<const uint64_t*>(sdx + 2 * c);
          const uint64_t dall2 = mul_f32x2(dx2, dw2), ndmn2 = mul_f32x2(dx2, ndmw2);
          const uint64_t is2 = pack_f32x2(__int2float_rn((int)vi[2 * k]), __int2float_rn((int)vi[2 * k + 1]));
          const uint64_t sm2 = (uint64_t)vm[2 * k] | ((uint64_t)vm[2 * k + 1] << 32);
          const uint64_t term2 = fma_f32x2(dall2, is2, mul_f32x2(ndmn2, sm2));
          acc[c] = add_f32x2(acc[c], term2);
        }
      }
      tc_fence_before();
      mbar_arrive(&m.aempty[r]);
    }
    if (ok && p.epi == kEpiSiluMul) {
      // rows 2i (gate) and 2i+1 (up) sit in adjacent lanes: the even lane
      // writes h_i = silu(gate) * up, the arithmetic of the GEMV's epilogue
      // (fully unrolled: a runtime index into acc would put the accumulators
      // in local memory for the whole main loop)
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const int64_t tok = m0 + half * 64 + c;
        const float gsum = __uint_as_float((uint32_t)(acc[c >> 1] >> (32 * (c & 1))));
        const float usum = __shfl_down_sync(0xffffffffu, gsum, 1);
        if (!(lane & 1) && row + 1 < p.n_rows && tok < p.n_cols) {
          const float sg = __fdiv_rn(gsum, __fadd_rn(1.0f, expf(-gsum)));
          p.y[tok * p.ldy + (row >> 1)] = __fmul_rn(sg, usum);
        }
      }
    } else if (ok && row < p.n_rows) {
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const int64_t tok = m0 + half * 64 + c;
        float v = __uint_as_float((uint32_t)(acc[c >> 1] >> (32 * (c & 1))));
        if (tok < p.n_cols) {
          if (p.epi == kEpiResidual) v = __fadd_rn(p.resid[tok * p.ld_resid + row], v);
          p.y[tok * p.ldy + row] = v;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

// Activation operands in UMMA order: the Q8_K quants as int8 in swizzled
// 128-row x 128-byte atoms per (token tile, super-block, half), bsums as fp16
// in the no-swizzle 128x16 tile per (token tile, super-block), d as fp32
// [n_cols][nb].  One warp per (token, super-block); tokens past n_cols stay
// zero (the buffers are cleared).
__global__ void gemm_prepass_kernel(const uint8_t* __restrict__ xq, int64_t n_cols, int nb, uint8_t* __restrict__ bq,
                                    uint8_t* __restrict__ bs, float* __restrict__ dx) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t wid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (wid >= n_cols * nb) return;
  const int64_t tok = wid / nb;
  const int b = (int)(wid % nb);
  const uint8_t* blk = xq + wid * Q8K_BLOCK_BYTES;
  const int64_t tile = tok / kTN;
  const uint32_t rr = (uint32_t)(tok % kTN);
  // lane l: quants 8l..8l+7 -> half l / 16, bytes 8(l % 16) .. of its atom row
  const uint32_t w0 = *reinterpret_cast<const uint32_t*>(blk + 4 + 8 * lane);
  const uint32_t w1 = *reinterpret_cast<const uint32_t*>(blk + 8 + 8 * lane);
  uint8_t* atom = bq + ((tile * nb + b) * 2 + (lane >> 4)) * (int64_t)kAtomBytes;
  *reinterpret_cast<uint2*>(atom + sw128_off(rr, (uint32_t)(8 * (lane & 15)))) = make_uint2(w0, w1);
  if (lane < 16) {
    const int16_t s = *reinterpret_cast<const int16_t*>(blk + 260 + 2 * lane);
    *reinterpret_cast<__half*>(bs + (tile * nb + b) * (int64_t)kMinBytes + min_off(rr, (uint32_t)lane)) =
        __int2half_rn(s);
  }
  if (lane == 0) dx[tok * nb + b] = *reinterpret_cast<const float*>(blk);
}

}  // namespace

size_t q2k_gemm_scratch_bytes(int64_t n_cols, int nb) {
  const int64_t tiles = (n_cols + kTN - 1) / kTN;
  return (size_t)tiles * nb * 2 * kAtomBytes + (size_t)tiles * nb * kMinBytes + (size_t)n_cols * nb * 4 + 256;
}

int q2k_gemm_tc(const Q2KWeight& w, const void* xq, int64_t n_cols, float* y, int64_t ldy, void* scratch,
                size_t scratch_bytes, cudaStream_t stream, int epi, const float* resid, int64_t ld_resid) {
  const int64_t out_rows = epi == kEpiSiluMul ? w.n_rows / 2 : w.n_rows;
  if (!w.tiles || !xq || !y || n_cols <= 0 || ldy < out_rows || w.fmt != kFmtQ2K) {
    set_last_error("q2k_gemm_tc: bad arguments (a Q2_K weight is required)");
    return kBadArgument;
  }
  if ((epi != kEpiStore && epi != kEpiResidual && epi != kEpiSiluMul) ||
      (epi == kEpiResidual && (!resid || ld_resid < out_rows)) || (epi == kEpiSiluMul && (w.n_rows & 1))) {
    set_last_error("q2k_gemm_tc: bad epilogue (residual needs resid with ld_resid >= rows; silu*mul needs "
                   "interleaved gate/up row pairs)");
    return kBadArgument;
  }
  if (reinterpret_cast<uintptr_t>(xq) & 3) {
    set_last_error("q2k_gemm_tc: Q8_K activations must be 4-byte aligned");
    return kBadArgument;
  }
  const int nb = w.nb;
  const size_t need = q2k_gemm_scratch_bytes(n_cols, nb);
  if (!scratch || scratch_bytes < need || (reinterpret_cast<uintptr_t>(scratch) & 255)) {
    set_last_error("q2k_gemm_tc: scratch of %zu bytes (256-aligned) required", need);
    return kBadArgument;
  }
  const int raw_slots = gemm_smem_bytes(nb, kMaxRaw) <= 227 * 1024 ? kMaxRaw : 2;
  const size_t smem = gemm_smem_bytes(nb, raw_slots);
  if (smem > 227 * 1024) {
    set_last_error("q2k_gemm_tc: k=%lld too large", (long long)w.k);
    return kBadArgument;
  }
  unsigned* err = device_error_ptr();
  if (!err) {
    set_last_error("q2k_gemm_tc: device error word unavailable");
    return kCudaError;
  }
  const int64_t tiles = (n_cols + kTN - 1) / kTN;
  uint8_t* bq = static_cast<uint8_t*>(scratch);
  uint8_t* bs = bq + (size_t)tiles * nb * 2 * kAtomBytes;
  float* dx = reinterpret_cast<float*>(bs + (size_t)tiles * nb * kMinBytes);
  // padding tokens of a partial last tile must read as zero (the prepass
  // writes every byte of the real tokens' rows)
  if (n_cols % kTN) {
    SMEAI_CUDA_TRY(cudaMemsetAsync(bq + (size_t)(tiles - 1) * nb * 2 * kAtomBytes, 0, (size_t)nb * 2 * kAtomBytes,
                                   stream));
    SMEAI_CUDA_TRY(cudaMemsetAsync(bs + (size_t)(tiles - 1) * nb * kMinBytes, 0, (size_t)nb * kMinBytes, stream));
  }
  const int64_t warps = n_cols * nb;
  SMEAI_CUDA_TRY(launch(gemm_prepass_kernel, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0, stream,
                        static_cast<const uint8_t*>(xq), n_cols, nb, bq, bs, dx));
  static unsigned configured = 0;
  int dev = 0;
  SMEAI_CUDA_TRY(cudaGetDevice(&dev));
  if (!(configured & (1u << (dev & 31)))) {
    SMEAI_CUDA_TRY(cudaFuncSetAttribute(q2k_gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    configured |= 1u << (dev & 31);
  }
  GemmParams p;
  p.tiles = w.tiles;
  p.nb = nb;
  p.n_rows = w.n_rows;
  p.n_groups = w.n_groups;
  p.bq = bq;
  p.bs = bs;
  p.dx = dx;
  p.n_cols = n_cols;
  p.y = y;
  p.ldy = ldy;
  p.epi = epi;
  p.resid = resid;
  p.ld_resid = ld_resid;
  p.err = err;
  p.raw_log2 = raw_slots == 4 ? 2 : 1;
  const dim3 grid((unsigned)((w.n_rows + kTM - 1) / kTM), (unsigned)tiles);
  SMEAI_CUDA_TRY(launch(q2k_gemm_tc_kernel, grid, dim3(kThreads), smem, stream, p));
  return kOk;
}

}  // namespace smeai
