// Host runtime pieces shared by the kernels: the per-device error word.
#include <c10/cuda/CUDAException.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <mutex>

static int* g_err_words[64] = {nullptr};
static std::mutex g_err_mu;

// 4-byte device word that kernels set to a non-zero code when a bounded wait
// gives up or an argument is invalid; allocated once per device.
int* dtb_error_word() {
  int dev = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_err_mu);
  if (!g_err_words[dev]) {
    C10_CUDA_CHECK(cudaMalloc(&g_err_words[dev], sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(g_err_words[dev], 0, sizeof(int)));
  }
  return g_err_words[dev];
}

// Read and clear the current device's error word (synchronises the device).
int64_t device_error() {
  int* w = dtb_error_word();
  int v = 0;
  C10_CUDA_CHECK(cudaDeviceSynchronize());
  C10_CUDA_CHECK(cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost));
  if (v) C10_CUDA_CHECK(cudaMemset(w, 0, sizeof(int)));
  return v;
}
