// Shared host/device helpers for libds_kernels_sm100.so.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stddef.h>

#include "ds_kernels.h"

namespace ds {

// ---- host-side error reporting --------------------------------------------------------
void set_last_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* where);

// Per-device facts cached on first use (SM count, ...).
struct DeviceInfo {
  int device;
  int num_sms;
  int clock_khz;  // maximum SM clock: converts wall-time bounds to clock64() cycles
};
int device_info(DeviceInfo* out);

// A second stream per device (with a fork and a join event) for work that overlaps the
// caller's stream inside one entry point: forked from and joined back into the caller's
// stream, so the entry point stays stream-ordered.  Created on first use; entry points that
// use it must not run concurrently on one device from several host threads.
struct SideStream {
  cudaStream_t stream;
  cudaEvent_t fork, join;
};
int side_stream(int device, SideStream* out);

// Programmatic dependent launch for the layer kernels (each lets its successor launch early
// and waits for its predecessor with griddepcontrol): off unless DS_PDL=1 -- measured 2-5 %
// slower per MoE layer step at 1024-8192 tokens, single-GPU and expert-parallel alike.
bool pdl_enabled();
// Fills attrs[n++] with the programmatic-serialization attribute when it is enabled.
void add_pdl_attr(cudaLaunchAttribute* attrs, unsigned int& n);

// Launch `kernel` on `s` with the programmatic-serialization attribute when enabled.
template <typename... ExpT, typename... ActT>
cudaError_t launch_pdl(void (*kernel)(ExpT...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, ActT&&... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 0;
  add_pdl_attr(attr, cfg.numAttrs);
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<ActT&&>(args)...);
}

// Device status word (one per device, lives in this library's module).
int* device_status_ptr();

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// A bump allocator over a caller-provided workspace.
struct Carve {
  uint8_t* base;
  size_t cap;
  size_t used;
  explicit Carve(void* b, size_t c) : base(static_cast<uint8_t*>(b)), cap(c), used(0) {}
  template <typename T>
  T* take(size_t count) {
    used = align_up(used, 256);
    T* p = reinterpret_cast<T*>(base ? base + used : nullptr);
    used += count * sizeof(T);
    return p;
  }
  bool ok() const { return base != nullptr && used <= cap; }
};

}  // namespace ds

#define DS_REQUIRE(cond, ...)                                    \
  do {                                                           \
    if (!(cond)) return ::ds::fail(DS_ERR_INVALID_ARG, __VA_ARGS__); \
  } while (0)

#define DS_CUDA(expr)                                            \
  do {                                                           \
    cudaError_t _e = (expr);                                     \
    if (_e != cudaSuccess) return ::ds::cuda_fail(_e, #expr);    \
  } while (0)

#define DS_LAUNCH_CHECK(name)                                    \
  do {                                                           \
    cudaError_t _e = cudaGetLastError();                         \
    if (_e != cudaSuccess) return ::ds::cuda_fail(_e, name);     \
  } while (0)

#define DS_TRY(expr)                                             \
  do {                                                           \
    int _s = (expr);                                             \
    if (_s != DS_OK) return _s;                                  \
  } while (0)
