// runtime.cu -- error text, feature switches and small host utilities shared
// by both C entry surfaces.
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>

#include "common.cuh"
#include "runtime.h"

namespace smeai {

namespace {
thread_local char g_last_error[512] = {0};
}

void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

const char* last_error() { return g_last_error; }

namespace {
std::atomic<int> g_fail_allocs{0};
std::atomic<uint64_t> g_wait_ns{0}, g_peer_wait_ns{0};
}  // namespace

void fail_next_allocs(int n) { g_fail_allocs.store(n < 0 ? 0 : n); }

cudaError_t device_malloc(void** p, size_t bytes) {
  int left = g_fail_allocs.load();
  while (left > 0 && !g_fail_allocs.compare_exchange_weak(left, left - 1)) {
  }
  if (left > 0) {
    *p = nullptr;
    return cudaErrorMemoryAllocation;
  }
  return cudaMalloc(p, bytes);
}

void set_wait_timeouts(uint64_t local_ns, uint64_t peer_ns) {
  g_wait_ns.store(local_ns);
  g_peer_wait_ns.store(peer_ns);
}
uint64_t wait_timeout_ns() {
  const uint64_t v = g_wait_ns.load();
  return v ? v : kDefaultWaitNs;
}
uint64_t peer_wait_timeout_ns() {
  const uint64_t v = g_peer_wait_ns.load();
  return v ? v : kDefaultPeerWaitNs;
}

bool pdl_enabled() {
  static int enabled = -1;
  if (enabled < 0) {
    const char* v = getenv("SMEAI_PDL");
    enabled = (v && v[0] == '0') ? 0 : 1;
  }
  return enabled == 1;
}

namespace {
__device__ unsigned g_device_error = 0;
}

unsigned* device_error_ptr() {
  static unsigned* cached[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!cached[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    cached[dev] = static_cast<unsigned*>(p);
  }
  return cached[dev];
}

int device_error_take(unsigned* code) {
  unsigned v = 0, zero = 0;
  SMEAI_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)));
  if (v) SMEAI_CUDA_TRY(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero)));
  *code = v;
  return kOk;
}

bool device_ready() {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    return false;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  int major = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return major == 10;
}

bool is_device_pointer(const void* p) {
  if (!p) return false;
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// ---- DeviceBuffer ----------------------------------------------------------
int DeviceBuffer::reserve(size_t bytes) {
  if (bytes <= cap) return kOk;
  if (ptr) cudaFree(ptr);
  ptr = nullptr;
  cap = 0;
  size_t want = bytes < 256 ? 256 : bytes;
  if (device_malloc(&ptr, want) != cudaSuccess) {
    cudaGetLastError();
    ptr = nullptr;
    set_last_error("cudaMalloc of %zu bytes failed", want);
    return kAllocFailed;
  }
  cap = want;
  return kOk;
}

void DeviceBuffer::release() {
  if (ptr) cudaFree(ptr);
  ptr = nullptr;
  cap = 0;
}

// ---- Staged: a host-or-device argument mirrored on the device ---------------
int Staged::in(const void* src, size_t bytes, cudaStream_t s) {
  host = nullptr;
  n = bytes;
  if (!src) {
    dev = nullptr;
    return kOk;
  }
  if (is_device_pointer(src)) {
    dev = const_cast<void*>(src);
    return kOk;
  }
  int st = buf.reserve(bytes);
  if (st != kOk) return st;
  SMEAI_CUDA_TRY(cudaMemcpyAsync(buf.ptr, src, bytes, cudaMemcpyHostToDevice, s));
  dev = buf.ptr;
  return kOk;
}

int Staged::out(void* dst, size_t bytes) {
  n = bytes;
  if (is_device_pointer(dst)) {
    dev = dst;
    host = nullptr;
    return kOk;
  }
  int st = buf.reserve(bytes);
  if (st != kOk) return st;
  dev = buf.ptr;
  host = dst;
  return kOk;
}

int Staged::finish(cudaStream_t s) {
  if (host) SMEAI_CUDA_TRY(cudaMemcpyAsync(host, dev, n, cudaMemcpyDeviceToHost, s));
  return kOk;
}

}  // namespace smeai
