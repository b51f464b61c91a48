// Allocation-free C entry point for the RMSNorm backward.
//
// This entry point has no counterpart in the reference implementation.
//
// Who it is for: callers that cannot allocate device memory at the moment
// they run the backward, such as a C or C++ host program (or a plugin inside
// another runtime) that links this library without PyTorch and its caching
// allocator, code that has reserved all device memory up front and may not
// grow it, or code issuing work where a cudaMalloc would synchronise the
// device or is not permitted.
// They pass their own inputs and outputs; the per-block partial sums of the
// weight gradient, which the allocating entry point keeps in a temporary
// buffer, live here in a fixed device array inside the library.
//
// The scratch array holds DTB_NOALLOC_SCRATCH_FLOATS floats (8 MiB); every GPU
// that loads the library keeps it until the process exits.  Limits: `dim` a
// multiple of 8 and at most DTB_NOALLOC_MAX_DIM; any `rows` >= 1.
//
// The first call on a device looks up the array's device address on that
// device (cudaGetSymbolAddress), so make that first call before any stream
// capture begins.  Every call on a device shares the one array: calls whose
// executions overlap on the GPU (different streams without ordering between
// them) race on it.  Each call overwrites every scratch value it later reads,
// so nothing needs clearing between calls.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

#define DTB_NOALLOC_SCRATCH_FLOATS (1L << 21)
#define DTB_NOALLOC_MAX_DIM 12288

#define DTB_NOALLOC_OK 0
#define DTB_NOALLOC_BAD_ARGUMENT 1
#define DTB_NOALLOC_TOO_LARGE 2
#define DTB_NOALLOC_CUDA_ERROR 3

// dy, x, dx: bf16 [rows, dim] row-major; w: [dim] bf16 (w_is_fp32 = 0) or fp32;
// rstd: fp32 [rows] saved by the forward; dw_acc: fp32 [dim], the weight
// gradient is ADDED to it.  Runs on `stream` (a cudaStream_t, may be 0).
// Returns one of the DTB_NOALLOC_* codes; allocates nothing.  If a CUDA error
// is already pending on entry (cudaPeekAtLastError), nothing is launched, the
// call returns DTB_NOALLOC_CUDA_ERROR and the error stays pending.
int dtb_rmsnorm_bwd_noalloc(const void* dy, const void* x, const void* w, int w_is_fp32, const float* rstd,
                            void* dx, float* dw_acc, int rows, int dim, void* stream);

// Text for a return code of dtb_rmsnorm_bwd_noalloc.
const char* dtb_noalloc_error_string(int code);

#ifdef __cplusplus
}
#endif
