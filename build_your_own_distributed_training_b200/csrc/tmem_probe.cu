// Self-check of the tcgen05 MMA form that takes its A operand from tensor
// memory instead of shared memory (the layout a softmax warp produces: thread
// = row = TMEM lane, consecutive bf16 pairs in consecutive 32-bit columns).
// Kernels that keep P or dS in TMEM between the elementwise stage and the next
// product rely on that layout; tmem_a_operand_check runs one such MMA,
// D[128, 128] = A[128, 128] x B[128, 128]^T, so a test can compare it with the
// fp32 product before any kernel depends on it.  One CTA, bounded waits.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace dtb {
namespace probe {

__device__ __forceinline__ void umma_bf16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_st32_u(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

constexpr int N = 128, K = 128;

__global__ void __launch_bounds__(128, 1) tmem_a_probe_kernel(const __nv_bfloat16* __restrict__ A,
                                                              const __nv_bfloat16* __restrict__ B,
                                                              float* __restrict__ D, int* err) {
  __shared__ __align__(1024) uint8_t sb[K / 64][N * 128];  // B, K-major, 128-byte swizzle
  __shared__ uint64_t bar;
  __shared__ uint32_t holder;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = threadIdx.x;  // row of A / D == TMEM lane
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&holder, 256);
    tmem_relinquish();
  }
  // B rows into the swizzled layout the MMA descriptors expect
  for (int i = threadIdx.x; i < N * (K / 8); i += blockDim.x) {
    const int n = i / (K / 8), c = i % (K / 8);  // 16-byte chunk c of row n
    const uint4 v = *reinterpret_cast<const uint4*>(B + (long)n * K + c * 8);
    *reinterpret_cast<uint4*>(&sb[c / 8][n * 128 + (((c % 8) ^ (n & 7)) << 4)]) = v;
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = holder;
  const uint32_t t_d = tmem, t_a = tmem + 128;  // D: 128 fp32 columns; A: K/2 = 64 columns of bf16 pairs
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  // A row r: bf16 pairs (k, k+1) in column k/2, element k in the low half
#pragma unroll
  for (int c = 0; c < K / 2; c += 32) {
    uint32_t v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = *reinterpret_cast<const uint32_t*>(A + (long)r * K + 2 * (c + i));
    tmem_st32_u(t_a + lane_off + c, v);
  }
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0) {
    constexpr uint32_t ID = idesc_bf16(128, N, false, false);
    const uint32_t b0 = smem_u32(&sb[0][0]);
#pragma unroll
    for (int kk = 0; kk < K / 16; ++kk) {
      const uint32_t boff = (kk >> 2) * (N * 128) + (kk & 3) * 32;
      umma_bf16_tmem_a(t_d, t_a + kk * 8, sdesc_sw128(b0 + boff, 16, 1024), ID, kk != 0);
    }
    umma_commit(&bar);
  }
  const bool ok = mbar_wait(&bar, 0, err);
  tc_fence_after();
  if (ok) {
#pragma unroll 1
    for (int c = 0; c < N; c += 32) {
      float v[32];
      tmem_ld32(t_d + lane_off + c, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) D[(long)r * N + c + i] = v[i];
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

}  // namespace probe
}  // namespace dtb

// D = A x B^T for A, B bf16 [128, 128] through one A-from-TMEM MMA (see the file comment).
torch::Tensor tmem_a_operand_check(torch::Tensor A, torch::Tensor B) {
  TORCH_CHECK(A.is_cuda() && A.scalar_type() == at::kBFloat16 && A.is_contiguous() && A.size(0) == 128 &&
                  A.size(1) == dtb::probe::K && B.sizes() == A.sizes() && B.is_contiguous() &&
                  B.scalar_type() == at::kBFloat16,
              "tmem_a_operand_check: bf16 [128, 128] operands");
  const c10::cuda::CUDAGuard g(A.device());
  auto D = torch::empty({128, dtb::probe::N}, A.options().dtype(at::kFloat));
  dtb::probe::tmem_a_probe_kernel<<<1, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(A.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(B.data_ptr()),
      D.data_ptr<float>(), dtb_error_word());
  DTB_LAUNCH_CHECK();
  return D;
}
