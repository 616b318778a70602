// common.cuh -- shared device/host helpers for the sm_100a kernels.
//
// Every translation unit is compiled with --fmad=false: a fused multiply-add
// appears only where the source writes fmaf()/__fmaf_rn(), so each kernel's
// float rounding is stated in its source and matches the CPU restatement.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>

namespace smeai {

constexpr int QK_K = 256;
constexpr int Q2K_BLOCK_BYTES = 84;   // ggml block_q2_K
constexpr int Q8K_BLOCK_BYTES = 292;  // ggml block_q8_K
constexpr int Q8K_BLOCK_WORDS = Q8K_BLOCK_BYTES / 4;

// Status codes shared by both C entry surfaces (same values as sme_ai_status).
enum Status : int {
  kOk = 0,
  kBadArgument = -1,
  kAllocFailed = -2,
  kUnsupported = -3,
  kWorkspaceTooSmall = -4,
  kCudaError = -5,
};

void set_last_error(const char* fmt, ...);
const char* last_error();

#define SMEAI_CUDA_TRY(expr)                                                   \
  do {                                                                         \
    cudaError_t _e = (expr);                                                   \
    if (_e != cudaSuccess) {                                                   \
      ::smeai::set_last_error("%s:%d %s -> %s", __FILE__, __LINE__, #expr,     \
                              cudaGetErrorString(_e));                         \
      return ::smeai::kCudaError;                                              \
    }                                                                          \
  } while (0)

// Limits of the kernels' bounded waits, read when a kernel is launched and
// passed to it as a parameter.  Waits on this GPU's own work (mbarriers,
// counters of the running grid) default to 2 s; waits on another GPU's rows
// default to 10 s.  set_wait_timeouts(local, peer) overrides them for later
// launches (0 keeps the default): tests use a short limit to make a wait run
// out on purpose.
constexpr uint64_t kDefaultWaitNs = 2000000000ull;
constexpr uint64_t kDefaultPeerWaitNs = 10000000000ull;
void set_wait_timeouts(uint64_t local_ns, uint64_t peer_ns);
uint64_t wait_timeout_ns();
uint64_t peer_wait_timeout_ns();

// True when programmatic dependent launch is enabled (default on; the
// environment variable SMEAI_PDL=0 turns it off for A/B timing).
bool pdl_enabled();

// Launch `kernel` with an optional programmatic-stream-serialization
// attribute so that its prologue (weight loads) may overlap the tail of the
// previous kernel in the stream.  Kernels call pdl_wait() before touching
// data written by earlier kernels.
template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                   cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// The same with a thread-block cluster of `cluster_x` CTAs along x (1 = none).
template <typename... KArgs, typename... Args>
cudaError_t launch_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                           unsigned cluster_x, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ---- device helpers -------------------------------------------------------
// Split cluster barrier: arrive early (relaxed), wait before touching another
// CTA's shared memory; the release/acquire pair publishes DSMEM writes.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared variable in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t cluster_map_shared(const void* p, unsigned rank) {
  uint32_t local = static_cast<uint32_t>(__cvta_generic_to_shared(p)), remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(rank));
  return remote;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// ---- mbarrier + bulk-copy (TMA) primitives ---------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
// One arrival for the whole warp (barriers initialised with a count of warps):
// the lanes meet at __syncwarp, which orders their earlier shared-memory
// accesses before lane 0's release arrive.  `dep` must be computed from every
// register the lanes loaded from the guarded buffer, so those loads have
// completed when the warp arrives (use 0 when nothing was loaded).
__device__ __forceinline__ void mbar_arrive_warp(uint64_t* bar, unsigned dep = 0u) {
  asm volatile("" ::"r"(dep));
  __syncwarp();
  if ((threadIdx.x & 31) == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Wait for phase `parity` of an mbarrier, giving up after ~timeout_ns of wall
// time.  Returns false on timeout (the caller records an error and leaves).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, unsigned parity, uint64_t timeout_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > timeout_ns) return false;
  }
}
// The same, also giving up as soon as the device error word is set: a
// producer whose consumers left early (a wait of theirs gave up) stops
// instead of waiting out its own limit for slots nobody will free.
__device__ __forceinline__ bool mbar_wait_or_error(uint64_t* bar, unsigned parity, uint64_t timeout_ns,
                                                   const unsigned* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*reinterpret_cast<const volatile unsigned*>(err)) return false;
    if (global_timer_ns() - t0 > timeout_ns) return false;
  }
}
// Ask the TMA engine to bring [src, src + bytes) into L2 (a hint: nothing
// completes, nothing is written).  src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
// Contiguous global -> shared copy by the TMA engine, completing on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Device-side error word: a kernel whose bounded wait expires ORs a code
// into it and returns instead of hanging or trapping; the host reads and
// clears it with device_error_take().  Kernels receive its address
// (device_error_ptr(), one word per device) as a parameter.
enum DeviceError : unsigned { kDevErrTimeout = 1u };
__device__ __forceinline__ void raise_device_error(unsigned* err, unsigned code) { atomicOr(err, code); }
unsigned* device_error_ptr();
int device_error_take(unsigned* code);

__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ggml's nearest_int: the float adder rounds v + 1.5*2^23 to an integer
// (round half to even); the integer sits in the low mantissa bits.
__device__ __forceinline__ int magic_round_bits(float v_plus_magic) {
  return (__float_as_int(v_plus_magic) & 0x007fffff) - 0x00400000;
}
constexpr float kMagic = 12582912.0f;

// 4 unsigned bytes of a times 4 signed bytes of b, summed into c.
__device__ __forceinline__ int dp4a_us(unsigned a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// Two signed 16-bit lanes of a times unsigned bytes 0,1 (lo) or 2,3 (hi) of b.
__device__ __forceinline__ int dp2a_lo_su(int a, unsigned b, int c) {
  int d;
  asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp2a_hi_su(int a, unsigned b, int c) {
  int d;
  asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ unsigned ldg_stream(const unsigned* p) {
  unsigned v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

}  // namespace smeai
