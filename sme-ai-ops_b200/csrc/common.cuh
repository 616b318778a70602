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

// ---- device helpers -------------------------------------------------------
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
