// sem_q8_gemm_noalloc: the Q8_0 projection for callers that cannot allocate.
//
// sem_q8_gemm needs two pieces of device scratch besides its input and output:
// the INT8 activation codes (m x k_in of them, held as fp16 for the tensor
// cores) and one absmax word. Its callers
// pass that scratch in. Some callers cannot provide or allocate it: a host
// runtime that reserves all device memory for its own pool and hands out only
// the buffers it manages (input and output), or a request path whose memory
// budget is fixed at start-up and must not grow or fail under load. cudaMalloc
// also synchronises the device, which such a path cannot afford.
//
// This variant keeps the scratch in a file-scope static __device__ array of
// fixed size (256 bytes for the absmax word + room for kNoAllocMaxCodes codes).
// Every GPU that loads the library holds that array until the process exits.
// The call makes no allocation: no cudaMalloc/cudaFree and no allocating
// library routine.
#include <mutex>

#include "common.cuh"
#include "host/internal.h"
#include "kernels.h"

namespace {

constexpr size_t kNoAllocHeaderBytes = 256;          // absmax word, padded to keep codes 256-byte aligned
constexpr size_t kNoAllocMaxCodes = size_t(8) << 20;  // 8 Mi activation codes (m * k_in)
constexpr size_t kNoAllocCodesBytes = kNoAllocMaxCodes * sizeof(__half);
constexpr int kMaxDevices = 64;

// In host code this name is only a host-side stand-in; kernels receive the
// device address obtained from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocHeaderBytes + kNoAllocCodesBytes];

std::mutex g_setup_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Resolves the array's device address once per device (the device must be current).
int scratch_for_device(int device, uint8_t** out) {
  if (device < 0 || device >= kMaxDevices)
    return sem::set_error(SEM_EINVAL, "sem_q8_gemm_noalloc: device %d beyond the %d supported", device, kMaxDevices);
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (!g_scratch_ptr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return sem::set_error(SEM_EDEVICE, "sem_q8_gemm_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_scratch_ptr[device] = p;
  }
  *out = static_cast<uint8_t*>(g_scratch_ptr[device]);
  return SEM_OK;
}

}  // namespace

extern "C" int sem_q8_gemm_noalloc(sem_q8_weight* w, const float* d_a, int32_t m, float* d_c, void* stream) {
  return sem::guarded([&]() -> int {
    if (!w || !d_a || !d_c) return sem::set_error(SEM_EINVAL, "null argument");
    if (m < 0) return sem::set_error(SEM_EINVAL, "sem_q8_gemm_noalloc: negative row count %d", m);
    if (m == 0) return SEM_OK;  // an empty batch, as sem_q8_gemm treats it
    const size_t need = (size_t)m * (size_t)w->k_in;
    if (need > kNoAllocMaxCodes)
      return sem::set_error(SEM_EINVAL,
                            "sem_q8_gemm_noalloc: %d rows x %d inputs need %zu activation codes of scratch, above the "
                            "static maximum of %zu (at most %zu rows for this weight)",
                            m, w->k_in, need, kNoAllocMaxCodes, kNoAllocMaxCodes / (size_t)w->k_in);
    sem::DeviceGuard dg(w->ctx->device);
    uint8_t* scratch = nullptr;
    int rc = scratch_for_device(w->ctx->device, &scratch);
    if (rc) return rc;
    uint32_t* absmax = reinterpret_cast<uint32_t*>(scratch);
    __half* codes = reinterpret_cast<__half*>(scratch + kNoAllocHeaderBytes);
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : w->ctx->stream;
    // The array keeps the previous call's contents: the absmax word must start at zero.
    SEM_CUDA(cudaMemsetAsync(absmax, 0, sizeof(uint32_t), st));
    SEM_CUDA(sem::launch_absmax(d_a, (int64_t)need, absmax, st));
    sem::SeqMeta meta{nullptr, nullptr, nullptr, m, 1};
    SEM_CUDA(sem::launch_quantize(d_a, nullptr, nullptr, w->k_in, meta, absmax, codes, st));
    // the kernel sem_q8_gemm would take for this m (sem_q8_path)
    SEM_CUDA(sem::launch_q8_proj(codes, w->proj(), m, w->n_out, w->k_in, absmax, nullptr, d_c, sem::kEpiStore, nullptr,
                                 nullptr, st));
    return SEM_OK;
  });
}
