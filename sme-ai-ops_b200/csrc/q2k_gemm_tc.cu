// q2k_gemm_tc.cu -- Q2_K x Q8_K prefill GEMM on the sm_100a tensor cores
// (tcgen05.mma with TMEM accumulators): the M > 8 case of the reference's Q2_K
// mul_mat (ggml_gemm_q2_K_8x8_q8_K, llama.cpp/doc/SME_Q2K_OPTIMIZATION.md:105-113).
//
// Exactness: the MMA operands are small integers held exactly in fp16 --
// Q8_K quants q8 in [-127, 127], scaled 2-bit weights scale*q in [0, 45],
// Q8_K bsums in [-2032, 2032], 4-bit mins in [0, 15] -- so every product and
// every partial sum of one 256-value super-block is an integer below 2^24 and
// the fp32 TMEM accumulators hold ggml's integer sums exactly:
//   D1[n][m] = isum  = sum_i (scale_j(i) * q2_i) * q8_i       (16 MMAs, K = 256)
//   D2[n][m] = summs = sum_j min_j * bsums_j                 (1 MMA,  K = 16)
// The epilogue then applies ggml's combine per super-block,
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
//   warps 2-5   dequantize: thread = weight row; 2-bit quants times 4-bit scale
//               into fp16, written straight into the 128-byte-swizzled K-major
//               shared-memory layout the MMA reads; the 16 mins likewise;
//   warps 6-13  epilogue: drain the double-buffered TMEM accumulators
//               (tcgen05.ld), combine, accumulate in registers, store.
// Stages: 4 quarter-super-block A/B stages (64 K each), 2 super-block slots for
// raw Q2_K tiles and min operands, 2 TMEM accumulator buffers (D1 + D2 each).
// Every wait is an mbarrier wait bounded by wall time; on expiry the kernel
// records kDevErrTimeout, the roles stop, in-flight copies and MMAs are
// drained (bounded), TMEM is freed and the kernel returns.  No multicast.
#include "common.cuh"
#include "kernels.h"

namespace smeai {

namespace {

constexpr int kTM = 128;                        // weight rows per tile
constexpr int kTN = 128;                        // activation rows per tile
constexpr int kAtomBytes = 128 * 128;           // 128 rows x 128 B (64 fp16 of K)
constexpr int kMinBytes = 128 * 32;             // 128 rows x 16 fp16
constexpr int kRawBytes = 4 * kTileBytes;       // four 32-row Q2_K tiles
constexpr int kThreads = 14 * 32;
constexpr int kTmemCols = 512;
constexpr uint64_t kTimeoutNs = 2000000000ull;

struct GemmParams {
  const uint8_t* tiles;   // Q2_K tile layout
  int nb;
  int64_t n_rows;
  int64_t n_groups;
  const uint8_t* bq;      // activation atoms [token tile][nb*4][kAtomBytes]
  const uint8_t* bs;      // bsums [token tile][nb][kMinBytes]
  const float* dx;        // [n_cols][nb]
  int64_t n_cols;
  float* y;
  int64_t ldy;
  unsigned* err;
};

// ---- tcgen05 helpers ---------------------------------------------------------
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
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

// Shared-memory matrix descriptor (sm_100 format, version 1).
__device__ __forceinline__ uint64_t smem_desc(const void* p, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint32_t layout) {
  const uint32_t a = smem_addr(p);
  return (uint64_t)((a >> 4) & 0x3FFF) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}
constexpr uint32_t kLayoutSw128 = 2, kLayoutNone = 0;

// Instruction descriptor: fp16 A and B, fp32 D, both K-major, M = 128, N = 128.
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kTN >> 3) << 17) | ((uint32_t)(kTM >> 4) << 24);

// Byte offset of (row r, k) in one 128-row x 64-K swizzled fp16 atom.
__host__ __device__ __forceinline__ uint32_t sw128_off(uint32_t r, uint32_t k) {
  return r * 128u + ((((k >> 3) & 7u) ^ (r & 7u)) << 4) + ((k & 7u) << 1);
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
  uint8_t* a;        // [4][kAtomBytes]
  uint8_t* b;        // [4][kAtomBytes]
  uint8_t* a2;       // [2][kMinBytes]
  uint8_t* b2;       // [2][kMinBytes]
  uint8_t* raw;      // [2][kRawBytes]
  float* sdx;        // [kTN][nb]
  uint64_t* full;    // [4]  dequant (128) + producer (1, tx)
  uint64_t* empty;   // [4]  commit
  uint64_t* rfull;   // [2]  producer (tx)
  uint64_t* rempty;  // [2]  dequant (128)
  uint64_t* mfull;   // [2]  dequant (128) + producer (1, tx)
  uint64_t* mempty;  // [2]  commit
  uint64_t* afull;   // [2]  commit
  uint64_t* aempty;  // [2]  epilogue (256)
  uint64_t* drain;   // [1]  commit (abort path)
  uint32_t* tmem;    // allocated TMEM base
  int* abort;
};

size_t gemm_smem_bytes(int nb) {
  return 1024 /* alignment slack */ + 8 * (size_t)kAtomBytes + 4 * (size_t)kMinBytes + 2 * (size_t)kRawBytes +
         (size_t)kTN * nb * 4 + 32 * 8 + 16;
}

__device__ __forceinline__ GemmSmem carve_gemm(uint8_t* base, int nb) {
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
  p += 2 * kRawBytes;
  m.sdx = reinterpret_cast<float*>(p);
  p += (size_t)kTN * nb * 4;
  uint64_t* bars = reinterpret_cast<uint64_t*>(p);
  m.full = bars;
  m.empty = bars + 4;
  m.rfull = bars + 8;
  m.rempty = bars + 10;
  m.mfull = bars + 12;
  m.mempty = bars + 14;
  m.afull = bars + 16;
  m.aempty = bars + 18;
  m.drain = bars + 20;
  m.tmem = reinterpret_cast<uint32_t*>(bars + 21);
  m.abort = reinterpret_cast<int*>(bars + 22);
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

__global__ void __launch_bounds__(kThreads, 1) q2k_gemm_tc_kernel(const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = p.nb;
  const int64_t row_tile = blockIdx.x, tok_tile = blockIdx.y;
  const int64_t n0 = row_tile * kTM, m0 = tok_tile * kTN;
  const GemmSmem m = carve_gemm(smem_raw, nb);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 4; ++i) {
      mbar_init(&m.full[i], 128 + 1);
      mbar_init(&m.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&m.rfull[i], 1);
      mbar_init(&m.rempty[i], 128);
      mbar_init(&m.mfull[i], 128 + 1);
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
  // activation scales of this tile: sdx[token][block] (0 past the last token)
  if (warp >= 6) {
    for (int i = threadIdx.x - 6 * 32; i < kTN * nb; i += 8 * 32) {
      const int64_t tok = m0 + i / nb;
      m.sdx[i] = tok < p.n_cols ? p.dx[tok * nb + (i % nb)] : 0.f;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *m.tmem;

  if (warp == 0) {
    // ---------------- producer
    if (lane == 0) {
      int issued_raw[2] = {-1, -1}, issued_m[2] = {-1, -1}, issued_b[4] = {-1, -1, -1, -1};
      for (int b = 0; b < nb; ++b) {
        const int r = b & 1;
        if (b >= 2 && (!wait_or_abort(m, &m.rempty[r], ((b >> 1) - 1) & 1, p.err) ||
                       !wait_or_abort(m, &m.mempty[r], ((b >> 1) - 1) & 1, p.err)))
          break;
        int groups = 0;
        for (int gi = 0; gi < 4; ++gi)
          if (row_tile * 4 + gi < p.n_groups) ++groups;
        mbar_arrive_expect_tx(&m.rfull[r], (unsigned)(groups * kTileBytes));
        for (int gi = 0; gi < groups; ++gi) {
          const int64_t g = row_tile * 4 + gi;
          bulk_copy_g2s(m.raw + r * kRawBytes + gi * kTileBytes, p.tiles + (g * nb + b) * (int64_t)kTileBytes,
                        kTileBytes, &m.rfull[r]);
        }
        issued_raw[r] = b;
        mbar_arrive_expect_tx(&m.mfull[r], kMinBytes);
        bulk_copy_g2s(m.b2 + r * kMinBytes, p.bs + (tok_tile * nb + b) * (int64_t)kMinBytes, kMinBytes,
                      &m.mfull[r]);
        issued_m[r] = b;
        bool ok = true;
        for (int a = 0; a < 4; ++a) {
          if (b >= 1 && !wait_or_abort(m, &m.empty[a], (b - 1) & 1, p.err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&m.full[a], kAtomBytes);
          bulk_copy_g2s(m.b + a * kAtomBytes, p.bq + ((tok_tile * nb + b) * 4 + a) * (int64_t)kAtomBytes,
                        kAtomBytes, &m.full[a]);
          issued_b[a] = b;
        }
        if (!ok) break;
      }
      if (*reinterpret_cast<volatile int*>(m.abort)) {
        // drain: the last copy issued into each slot lands before we leave
        for (int r = 0; r < 2; ++r) {
          if (issued_raw[r] >= 0) mbar_wait_bounded(&m.rfull[r], (issued_raw[r] >> 1) & 1, kTimeoutNs);
          if (issued_m[r] >= 0) mbar_wait_bounded(&m.mfull[r], (issued_m[r] >> 1) & 1, kTimeoutNs);
        }
        for (int a = 0; a < 4; ++a)
          if (issued_b[a] >= 0) mbar_wait_bounded(&m.full[a], issued_b[a] & 1, kTimeoutNs);
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
        for (int a = 0; a < 4; ++a) {
          if (!wait_or_abort(m, &m.full[a], b & 1, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = smem_desc(m.a + a * kAtomBytes, lbo_sw, sbo_sw, kLayoutSw128);
          const uint64_t db = smem_desc(m.b + a * kAtomBytes, lbo_sw, sbo_sw, kLayoutSw128);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)   // 16 fp16 of K = 32 bytes per MMA
            tc_mma_f16(d1, da + 2 * kk, db + 2 * kk, kIdesc, (a | kk) != 0);
          tc_commit(&m.empty[a]);
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
  } else if (warp < 6) {
    // ---------------- dequantize: thread = weight row of the tile
    const int t = threadIdx.x - 64;              // 0..127
    const int gi = t >> 5, l = t & 31;
    const bool present = row_tile * 4 + gi < p.n_groups;
    for (int b = 0; b < nb; ++b) {
      const int r = b & 1;
      if (!wait_or_abort(m, &m.rfull[r], (b >> 1) & 1, p.err)) break;
      uint4 q[4], sc;
      if (present) {
        const uint8_t* tile = m.raw + r * kRawBytes + gi * kTileBytes;
#pragma unroll
        for (int c = 0; c < 4; ++c) q[c] = reinterpret_cast<const uint4*>(tile + c * 512)[l];
        sc = reinterpret_cast<const uint4*>(tile + 2048)[l];
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) q[c] = make_uint4(0, 0, 0, 0);
        sc = make_uint4(0, 0, 0, 0);
      }
      mbar_arrive(&m.rempty[r]);
      const uint32_t scw[4] = {sc.x, sc.y, sc.z, sc.w};
      // the 16 mins into the no-swizzle 128 x 16 operand
      if (b >= 2 && !wait_or_abort(m, &m.mempty[r], ((b >> 1) - 1) & 1, p.err)) break;
      {
        uint32_t h[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t mins = (scw[k] >> 4) & 0x0F0F0F0Fu;
          h[2 * k] = bytes_to_half2(mins, 0x4140);
          h[2 * k + 1] = bytes_to_half2(mins, 0x4342);
        }
        uint8_t* dst = m.a2 + r * kMinBytes;
        *reinterpret_cast<uint4*>(dst + min_off(t, 0)) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4*>(dst + min_off(t, 8)) = make_uint4(h[4], h[5], h[6], h[7]);
        fence_async_smem();
        mbar_arrive(&m.mfull[r]);
      }
      // four quarters: quarter a = weights 64a..64a+63 = half a>>1, shift
      // planes 2(a&1) and 2(a&1)+1, 32 quants each from qs chunks 2h, 2h+1
      bool ok = true;
#pragma unroll 1
      for (int a = 0; a < 4; ++a) {
        if (b >= 1 && !wait_or_abort(m, &m.empty[a], (b - 1) & 1, p.err)) {
          ok = false;
          break;
        }
        const int h = a >> 1;
        uint8_t* dst = m.a + a * kAtomBytes;
#pragma unroll
        for (int sp = 0; sp < 2; ++sp) {
          const int s = 2 * (a & 1) + sp;
#pragma unroll
          for (int part = 0; part < 2; ++part) {      // quants l = 16*part .. 16*part+15
            const uint4 qc = q[2 * h + part];
            const int j = 8 * h + 2 * s + part;        // sub-block
            const uint32_t scale = (scw[j >> 2] >> (8 * (j & 3))) & 0xFu;
            const uint32_t w[4] = {qc.x, qc.y, qc.z, qc.w};
#pragma unroll
            for (int half8 = 0; half8 < 2; ++half8) {  // 8 quants -> one 16-byte chunk
              const uint32_t v0 = ((w[2 * half8] >> (2 * s)) & 0x03030303u) * scale;
              const uint32_t v1 = ((w[2 * half8 + 1] >> (2 * s)) & 0x03030303u) * scale;
              const uint4 hv = make_uint4(bytes_to_half2(v0, 0x4140), bytes_to_half2(v0, 0x4342),
                                          bytes_to_half2(v1, 0x4140), bytes_to_half2(v1, 0x4342));
              const uint32_t kin = (uint32_t)(sp * 32 + part * 16 + half8 * 8);  // K within the quarter
              *reinterpret_cast<uint4*>(dst + sw128_off((uint32_t)t, kin)) = hv;
            }
          }
        }
        fence_async_smem();
        mbar_arrive(&m.full[a]);
      }
      if (!ok) break;
    }
  } else {
    // ---------------- epilogue: 8 warps; TMEM lane quarter = warp % 4
    const int quarter = warp & 3;
    const int half = (warp - 6) >> 2;            // token columns half*64 .. +63
    const int t = quarter * 32 + lane;           // weight row within the tile
    const int64_t row = n0 + t;
    const int64_t g = row >> 5;
    float acc[64];
#pragma unroll
    for (int c = 0; c < 64; ++c) acc[c] = 0.f;
    bool ok = true;
    for (int b = 0; b < nb; ++b) {
      const int r = b & 1;
      if (!wait_or_abort(m, &m.afull[r], (b >> 1) & 1, p.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float dw = 0.f, dmw = 0.f;
      if (g < p.n_groups) {
        const unsigned dm = *reinterpret_cast<const unsigned*>(p.tiles + (g * nb + b) * (int64_t)kTileBytes + 2560 +
                                                               (row & 31) * 4);
        dw = __half2float(__ushort_as_half((unsigned short)(dm & 0xffffu)));
        dmw = __half2float(__ushort_as_half((unsigned short)(dm >> 16)));
      }
      const uint32_t lane_base = tmem + ((uint32_t)(quarter * 32) << 16);
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t vi[16], vm[16];
        const uint32_t col = (uint32_t)(r * 256 + half * 64 + cc * 16);
        tmem_ld16(lane_base + col, vi);
        tmem_ld16(lane_base + col + 128, vm);
        tmem_ld_wait();
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const int c = cc * 16 + k;
          const float dx = m.sdx[(half * 64 + c) * nb + b];
          const float dall = __fmul_rn(dx, dw), dmn = __fmul_rn(dx, dmw);
          const float term = __fmaf_rn(dall, __uint_as_float(vi[k]), -__fmul_rn(dmn, __uint_as_float(vm[k])));
          acc[c] = __fadd_rn(acc[c], term);
        }
      }
      tc_fence_before();
      mbar_arrive(&m.aempty[r]);
    }
    if (ok && row < p.n_rows) {
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const int64_t tok = m0 + half * 64 + c;
        if (tok < p.n_cols) p.y[tok * p.ldy + row] = acc[c];
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

// Activation operands in UMMA order: q8 as fp16 in swizzled 128x64 atoms per
// (token tile, super-block, quarter), bsums as fp16 in the no-swizzle 128x16
// tile per (token tile, super-block), d as fp32 [n_cols][nb].  One warp per
// (token, super-block); tokens past n_cols stay zero (the buffers are cleared).
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
  // lane l: quants 8l..8l+7 (one 16-byte chunk), quarter (8l)/64
  const uint32_t w0 = *reinterpret_cast<const uint32_t*>(blk + 4 + 8 * lane);
  const uint32_t w1 = *reinterpret_cast<const uint32_t*>(blk + 8 + 8 * lane);
  uint32_t h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t w = i < 2 ? w0 : w1;
    const int8_t lo = (int8_t)((w >> (16 * (i & 1))) & 0xff), hi = (int8_t)((w >> (16 * (i & 1) + 8)) & 0xff);
    __half2 v = __halves2half2(__int2half_rn(lo), __int2half_rn(hi));
    h[i] = *reinterpret_cast<uint32_t*>(&v);
  }
  const int a = (8 * lane) / 64;
  uint8_t* atom = bq + ((tile * nb + b) * 4 + a) * (int64_t)kAtomBytes;
  *reinterpret_cast<uint4*>(atom + sw128_off(rr, (uint32_t)((8 * lane) % 64))) = make_uint4(h[0], h[1], h[2], h[3]);
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
  return (size_t)tiles * nb * 4 * kAtomBytes + (size_t)tiles * nb * kMinBytes + (size_t)n_cols * nb * 4 + 256;
}

int q2k_gemm_tc(const Q2KWeight& w, const void* xq, int64_t n_cols, float* y, int64_t ldy, void* scratch,
                size_t scratch_bytes, cudaStream_t stream) {
  if (!w.tiles || !xq || !y || n_cols <= 0 || ldy < w.n_rows) {
    set_last_error("q2k_gemm_tc: bad arguments");
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
  const size_t smem = gemm_smem_bytes(nb);
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
  uint8_t* bs = bq + (size_t)tiles * nb * 4 * kAtomBytes;
  float* dx = reinterpret_cast<float*>(bs + (size_t)tiles * nb * kMinBytes);
  // padding tokens of the last tile must read as zero
  SMEAI_CUDA_TRY(cudaMemsetAsync(bq, 0, (size_t)tiles * nb * (4 * kAtomBytes + kMinBytes), stream));
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
  p.err = err;
  const dim3 grid((unsigned)((w.n_rows + kTM - 1) / kTM), (unsigned)tiles);
  SMEAI_CUDA_TRY(launch(q2k_gemm_tc_kernel, grid, dim3(kThreads), smem, stream, p));
  return kOk;
}

}  // namespace smeai
