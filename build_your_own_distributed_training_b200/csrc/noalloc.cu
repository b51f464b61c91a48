// Allocation-free RMSNorm backward (see noalloc.h for who calls it and why).
// This entry point has no counterpart in the reference implementation.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "noalloc.h"

// The launch helper shared with the allocating entry point (elementwise.cu);
// it takes the partial-sum workspace as an argument and allocates nothing.
void rmsnorm_bwd_launch(const __nv_bfloat16* dy, const __nv_bfloat16* x, const void* w, bool w_f32,
                        const float* rstd, __nv_bfloat16* dx, float* dw_acc, float* part, int M, int D,
                        int rows_per_cta, cudaStream_t st);

// Per-CTA partial sums of the weight gradient: [num_ctas, dim] floats.
static __device__ __align__(256) float g_noalloc_scratch[DTB_NOALLOC_SCRATCH_FLOATS];

namespace {
constexpr int kMaxDevices = 64;
constexpr int kMaxCtas = 256;
float* g_scratch_addr[kMaxDevices] = {nullptr};
std::mutex g_mu;

// Device address of the scratch array on the current device.  In host code
// the array's name is only a host-side stand-in, so the address must come
// from cudaGetSymbolAddress, once per device, with that device current.
int scratch_for_current_device(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return DTB_NOALLOC_CUDA_ERROR;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return DTB_NOALLOC_CUDA_ERROR;
    g_scratch_addr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_addr[dev];
  return DTB_NOALLOC_OK;
}
}  // namespace

extern "C" int dtb_rmsnorm_bwd_noalloc(const void* dy, const void* x, const void* w, int w_is_fp32,
                                       const float* rstd, void* dx, float* dw_acc, int rows, int dim,
                                       void* stream) {
  if (!dy || !x || !w || !rstd || !dx || !dw_acc || rows <= 0 || dim <= 0 || dim % 8 != 0)
    return DTB_NOALLOC_BAD_ARGUMENT;
  // the kernels move dy, x, dx and w in 16-byte vectors
  const auto misaligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; };
  if (misaligned(dy) || misaligned(x) || misaligned(dx) || misaligned(w)) return DTB_NOALLOC_BAD_ARGUMENT;
  if (dim > DTB_NOALLOC_MAX_DIM) return DTB_NOALLOC_TOO_LARGE;
  // as many CTAs as both the scratch array and kMaxCtas allow
  const long max_ctas = DTB_NOALLOC_SCRATCH_FLOATS / dim < kMaxCtas ? DTB_NOALLOC_SCRATCH_FLOATS / dim : kMaxCtas;
  const int rows_per_cta = (int)((rows + max_ctas - 1) / max_ctas);
  const long ctas = (rows + rows_per_cta - 1) / rows_per_cta;
  if (ctas * (long)dim > DTB_NOALLOC_SCRATCH_FLOATS) return DTB_NOALLOC_TOO_LARGE;
  float* part = nullptr;
  const int rc = scratch_for_current_device(&part);
  if (rc != DTB_NOALLOC_OK) return rc;
  // An error left pending by the caller's own earlier work is reported and left
  // in place for the caller, not consumed here.
  if (cudaPeekAtLastError() != cudaSuccess) return DTB_NOALLOC_CUDA_ERROR;
  rmsnorm_bwd_launch(static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(x), w,
                     w_is_fp32 != 0, rstd, static_cast<__nv_bfloat16*>(dx), dw_acc, part, rows, dim, rows_per_cta,
                     static_cast<cudaStream_t>(stream));
  return cudaGetLastError() == cudaSuccess ? DTB_NOALLOC_OK : DTB_NOALLOC_CUDA_ERROR;
}

extern "C" const char* dtb_noalloc_error_string(int code) {
  switch (code) {
    case DTB_NOALLOC_OK: return "ok";
    case DTB_NOALLOC_BAD_ARGUMENT: return "bad argument: null pointer, a dy/x/dx/w pointer not 16-byte aligned, rows < 1, or dim not a positive multiple of 8";
    case DTB_NOALLOC_TOO_LARGE: return "dim above DTB_NOALLOC_MAX_DIM (12288): the fixed scratch/shared-memory limit";
    case DTB_NOALLOC_CUDA_ERROR: return "CUDA error (an error already pending on entry, scratch address lookup or kernel launch failed)";
    default: return "unknown code";
  }
}
