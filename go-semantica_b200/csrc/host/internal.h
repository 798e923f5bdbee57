// Host-side internals of libsemantica_b200: contexts, device buffers, errors.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <exception>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "../../../include/semantica_b200.h"
#include "../kernels.h"

namespace sem {

// ---- thread-local error message ----
int set_error(int code, const char* fmt, ...);
const char* last_error();

// Runs the body of a C entry point so that no C++ exception crosses the C
// ABI (unwinding into a cgo or C caller ends its process): a failed host
// allocation returns SEM_ENOMEM, any other exception SEM_EINTERNAL, each with
// its message in sem_last_error.
template <class F>
int guarded(F&& body) noexcept {
  try {
    return body();
  } catch (const std::bad_alloc&) {
    return set_error(SEM_ENOMEM, "host allocation failed");
  } catch (const std::exception& e) {
    return set_error(SEM_EINTERNAL, "%s", e.what());
  } catch (...) {
    return set_error(SEM_EINTERNAL, "unknown exception");
  }
}

// The model's current faithful-mode setting (sem_model_set_faithful).
sem_faithful_config model_faithful_get(const sem_model* m);

// sem_embed's host checks in the reference's order (model_int8.go:149-178):
// fills dims (NULL dims_in = embed_dim) and the total output floats.
int validate_embed_request(const sem_model_config& c, const int32_t* ids, const int32_t* offsets, int32_t B,
                           const int32_t* dims_in, float* out, std::vector<int32_t>* dims, int64_t* out_floats);

#define SEM_CUDA(call)                                                                             \
  do {                                                                                             \
    cudaError_t e_ = (call);                                                                       \
    if (e_ != cudaSuccess) return ::sem::set_error(SEM_EDEVICE, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

// A device allocation that only grows.
struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
  DevBuf() = default;
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  ~DevBuf() { release(); }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
  }
  cudaError_t ensure(size_t n) {
    if (n <= bytes) return cudaSuccess;
    release();
    cudaError_t e = cudaMalloc(&p, n);
    if (e == cudaSuccess) bytes = n;
    else p = nullptr;
    return e;
  }
  template <class T>
  T* as() const { return static_cast<T*>(p); }
};

// Pinned host staging that only grows.
struct HostBuf {
  void* p = nullptr;
  size_t bytes = 0;
  HostBuf() = default;
  HostBuf(const HostBuf&) = delete;
  HostBuf& operator=(const HostBuf&) = delete;
  ~HostBuf() { if (p) cudaFreeHost(p); }
  cudaError_t ensure(size_t n) {
    if (n <= bytes) return cudaSuccess;
    if (p) cudaFreeHost(p);
    p = nullptr;
    bytes = 0;
    cudaError_t e = cudaMallocHost(&p, n);
    if (e == cudaSuccess) bytes = n;
    return e;
  }
  template <class T>
  T* as() const { return static_cast<T*>(p); }
};

// Makes ctx's device current for the lifetime of the guard.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace sem

struct sem_context {
  int device = 0;
  cudaStream_t stream = nullptr;
  std::mutex mu;
  sem::DevBuf scratch;  // shared device scratch (candidate lists, staging)
  sem::HostBuf pinned;
};

// A Q8_0 weight repacked for the device: fp16 codes [n_out][k_in] (exact
// integers) and fp32 block scales [n_out][k_in/32].
struct sem_q8_weight {
  sem_context* ctx = nullptr;
  int32_t k_in = 0, n_out = 0;
  sem::DevBuf codes, scales;   // fp16 codes [n_out][k_in], block scales [n_out][k_in/32]
  sem::DevBuf planes, rscale;  // split planes hi then lo [2][n_out][k_in], row scales [n_out]
  sem::DevBuf lanes;           // int8 plane [n_out][k_in], lane-major rows (CUDA-core kernel)
  sem::Q8Proj proj() const {
    const __half* hi = static_cast<const __half*>(planes.p);
    return sem::Q8Proj{static_cast<const __half*>(codes.p), static_cast<const float*>(scales.p), hi,
                       hi ? hi + (size_t)n_out * k_in : nullptr, static_cast<const float*>(rscale.p),
                       static_cast<const int8_t*>(lanes.p)};
  }
};
