// Test-only kernels: the product's device helpers (common.cuh, sm100.cuh)
// applied element by element, so tests can compare them with the CPU oracle
// on many inputs, and a pipeline wait that nothing completes, so a test can
// check that the bounded wait gives up, reports its error bit and returns.
// Built into tests/_build/libsemantica_testkernels.so; the product library
// never links it.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../go-semantica_b200/csrc/common.cuh"
#include "../../go-semantica_b200/csrc/sm100.cuh"

namespace {

__global__ void fast_exp_kernel(const float* x, float* y, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = sem::fast_exp_ref(x[i]);
}

__global__ void gelu_quick_kernel(const float* x, float* y, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = sem::gelu_quick_ref(x[i]);
}

// RMSNorm of each row (norm.go:8-36): 8 lanes per row, the reference's lane
// order for the sum of squares, x * inv then * w.
__global__ void rmsnorm_kernel(const float* x, const float* w, float* y, int rows, int n, float eps) {
  const int g = (blockIdx.x * blockDim.x + threadIdx.x) >> 3, sub = threadIdx.x & 7;
  const int row = g < rows ? g : rows - 1;  // whole groups of 8 take part in the shuffles
  const float* xr = x + (int64_t)row * n;
  const float inv = sem::rms_inv_ref(sem::row_sumsq_ref(xr, n, sub), n, eps);
  if (g >= rows) return;
  for (int i = sub; i < n; i += 8) y[(int64_t)row * n + i] = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
}

// One thread waits on an mbarrier that expects one arrival and gets none:
// the bounded wait must give up after its limit, set the abort flag and the
// error bit, and return.
__global__ void bounded_wait_kernel(uint32_t* err, uint32_t* returned) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    sem::mbar_init(&bar, 1);
    abort_flag = 0;
    sem::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool ok = sem::mbar_wait(&bar, 0, &abort_flag, err, 0x10u);
    returned[0] = ok ? 2u : 1u;
    returned[1] = (uint32_t)abort_flag;
  }
}

int run_elementwise(int op, const float* hx, float* hy, int64_t n) {
  float *dx = nullptr, *dy = nullptr;
  if (cudaMalloc(&dx, n * 4) != cudaSuccess || cudaMalloc(&dy, n * 4) != cudaSuccess) return 1;
  cudaMemcpy(dx, hx, n * 4, cudaMemcpyHostToDevice);
  const unsigned blocks = (unsigned)((n + 255) / 256);
  if (op == 0) fast_exp_kernel<<<blocks, 256>>>(dx, dy, n);
  else gelu_quick_kernel<<<blocks, 256>>>(dx, dy, n);
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(hy, dy, n * 4, cudaMemcpyDeviceToHost);
  cudaFree(dx);
  cudaFree(dy);
  return e == cudaSuccess ? 0 : 2;
}

}  // namespace

extern "C" {

int tk_fast_exp(const float* x, float* y, int64_t n) { return run_elementwise(0, x, y, n); }
int tk_gelu_quick(const float* x, float* y, int64_t n) { return run_elementwise(1, x, y, n); }

int tk_rmsnorm(const float* x, const float* w, float* y, int rows, int n, float eps) {
  if (n % 8) return 3;
  float *dx = nullptr, *dw = nullptr, *dy = nullptr;
  const size_t bytes = (size_t)rows * n * 4;
  if (cudaMalloc(&dx, bytes) != cudaSuccess || cudaMalloc(&dw, n * 4) != cudaSuccess ||
      cudaMalloc(&dy, bytes) != cudaSuccess)
    return 1;
  cudaMemcpy(dx, x, bytes, cudaMemcpyHostToDevice);
  cudaMemcpy(dw, w, n * 4, cudaMemcpyHostToDevice);
  rmsnorm_kernel<<<(unsigned)((rows * 8 + 255) / 256), 256>>>(dx, dw, dy, rows, n, eps);
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(y, dy, bytes, cudaMemcpyDeviceToHost);
  cudaFree(dx);
  cudaFree(dw);
  cudaFree(dy);
  return e == cudaSuccess ? 0 : 2;
}

// err_bits: the error word after the kernel; returned[0]: 1 if the wait gave
// up, 2 if it (wrongly) completed; returned[1]: the abort flag.
int tk_bounded_wait(uint32_t* err_bits, uint32_t* returned) {
  uint32_t* d = nullptr;
  if (cudaMalloc(&d, 16) != cudaSuccess) return 1;
  cudaMemset(d, 0, 16);
  bounded_wait_kernel<<<1, 32>>>(d, d + 1);
  cudaError_t e = cudaDeviceSynchronize();
  uint32_t h[3] = {0, 0, 0};
  if (e == cudaSuccess) e = cudaMemcpy(h, d, 12, cudaMemcpyDeviceToHost);
  cudaFree(d);
  *err_bits = h[0];
  returned[0] = h[1];
  returned[1] = h[2];
  return e == cudaSuccess ? 0 : 2;
}

}  // extern "C"
