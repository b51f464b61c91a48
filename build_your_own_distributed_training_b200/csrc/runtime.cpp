// Host runtime pieces shared by the kernels: the per-device error word.
#include <c10/cuda/CUDAException.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <execinfo.h>
#include <signal.h>
#include <unistd.h>

#include <cstdio>
#include <cstdlib>
#include <mutex>

// Opt-in (DTB_SEGV_TRACE=1): print the native stack of a SIGSEGV to stderr,
// then re-raise it with the default action.
static void segv_trace(int sig) {
  void* frames[64];
  const int n = backtrace(frames, 64);
  static const char msg[] = "\n[dtb] native backtrace:\n";
  (void)!write(2, msg, sizeof(msg) - 1);
  backtrace_symbols_fd(frames, n, 2);
  signal(sig, SIG_DFL);
  raise(sig);
}

static int install_segv_trace() {
  const char* e = std::getenv("DTB_SEGV_TRACE");
  if (e && e[0] == '1') signal(SIGSEGV, segv_trace);
  return 0;
}
static int g_trace_installed = install_segv_trace();

bool dtb_debug_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = std::getenv("DTB_DEBUG");
    on = (e && e[0] == '1') ? 1 : 0;
  }
  return on == 1;
}

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
