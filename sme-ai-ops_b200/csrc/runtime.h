// runtime.h -- host utilities shared by the C entry surfaces (internal).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

namespace smeai {

bool device_ready();
bool is_device_pointer(const void* p);

// Every device allocation of the library goes through device_malloc.  The
// test hook fail_next_allocs(n) makes the next n calls fail as cudaMalloc
// does when the device is out of memory, so the entry points' ALLOC_FAILED
// paths can be exercised without exhausting a real GPU.
cudaError_t device_malloc(void** p, size_t bytes);
void fail_next_allocs(int n);

// A growable device allocation (never shrinks).
struct DeviceBuffer {
  void* ptr = nullptr;
  size_t cap = 0;
  int reserve(size_t bytes);
  void release();
  ~DeviceBuffer() { release(); }
};

// One argument of a host-pointer entry point: device pointers are used in
// place, host pointers are copied through a device staging buffer.
struct Staged {
  DeviceBuffer buf;
  void* dev = nullptr;
  void* host = nullptr;
  size_t n = 0;
  int in(const void* src, size_t bytes, cudaStream_t s);  // H2D (if host)
  int out(void* dst, size_t bytes);                       // prepare
  int finish(cudaStream_t s);                             // D2H (if host)
};

}  // namespace smeai
