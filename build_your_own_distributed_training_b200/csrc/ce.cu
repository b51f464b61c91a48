// Fused LM-head cross-entropy: the reductions between the two GEMM halves.
//
// The head GEMM with EPI_CE_STATS (gemm.cu) leaves, per row and 128/256-column
// block of the vocabulary, the pair (max, sum exp(x - max)) and the label's
// logit; no [tokens, vocab] logits exist.  These kernels turn that into the
// per-row log-sum-exp and the mean loss:
//
//   ce_stats_reduce_kernel   one warp per row combines its column blocks in a
//                            fixed order -> (m, s), then either
//                            lse = m + log s (whole vocabulary on this GPU), or
//                            writes (m, s, target logit if owned) into this
//                            rank's slot of the TP symmetric heap;
//   ce_peer_combine_kernel   vocabulary split over the TP group: after a device
//                            barrier every rank reads every rank's (m, s, t) in
//                            rank order, so all ranks hold the same lse bits;
//   ce_loss_finish_kernel    one CTA: fixed-order sum of the row losses and the
//                            count of valid labels -> loss, 1 / n_valid.
//
// The backward recomputes the logits chunk by chunk with EPI_CE_GRAD, which
// needs only lse, the labels and the device scalar 1 / n_valid.
// Reference semantics: src/model/transformer.py:184-191 (F.cross_entropy,
// mean over labels != -100) and, for the vocabulary split,
// src/parallelism/tensor_parallel.py:396-400 (loss_parallel).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace dtb {
namespace ce {

constexpr int MAX_PEERS = 8;

struct PeerPtrs {
  uint8_t* base[MAX_PEERS];
};

__device__ __forceinline__ void lse_merge(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;  // both empty
  s = s * expf(m - mn) + s2 * expf(m2 - mn);
  m = mn;
}

__device__ __forceinline__ bool label_valid(long lab, long ignore, long vocab_total) {
  return lab != ignore && lab >= 0 && lab < vocab_total;
}

// stats: [M, nblk] float2; tgt: [M].  Labels in [vocab_off, vocab_off + v_local) are owned here.
__global__ void ce_stats_reduce_kernel(const float2* __restrict__ stats, const float* __restrict__ tgt,
                                       const int64_t* __restrict__ labels, int M, int nblk, long vocab_off,
                                       long v_local, long vocab_total, long ignore, float* __restrict__ lse,
                                       float* __restrict__ row_loss, float4* __restrict__ xchg) {
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  float m = -INFINITY, s = 0.f;
  for (int j = lane; j < nblk; j += 32) {
    const float2 p = stats[(long)row * nblk + j];
    lse_merge(m, s, p.x, p.y);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    lse_merge(m, s, m2, s2);
  }
  if (lane != 0) return;
  const long lab = labels[row];
  const bool valid = label_valid(lab, ignore, vocab_total);
  const bool mine = valid && lab >= vocab_off && lab < vocab_off + v_local;
  const float t = mine ? tgt[row] : 0.f;
  if (xchg != nullptr) {
    xchg[row] = make_float4(m, s, t, 0.f);
    return;
  }
  const float l = m + logf(s);
  lse[row] = l;
  row_loss[row] = valid ? l - t : 0.f;
}

__global__ void ce_peer_combine_kernel(PeerPtrs peers, long off, int size, const int64_t* __restrict__ labels, int M,
                                       long vocab_total, long ignore, float* __restrict__ lse,
                                       float* __restrict__ row_loss) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= M) return;
  float4 v[MAX_PEERS];
#pragma unroll
  for (int p = 0; p < MAX_PEERS; ++p) {
    if (p < size) {
      const uint4 u = ld_cg_v4(peers.base[p] + off + (long)row * 16);
      v[p] = make_float4(__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z), __uint_as_float(u.w));
    }
  }
  float m = -INFINITY, s = 0.f, t = 0.f;
#pragma unroll
  for (int p = 0; p < MAX_PEERS; ++p) {
    if (p < size) {
      lse_merge(m, s, v[p].x, v[p].y);
      t += v[p].z;
    }
  }
  const float l = m + logf(s);
  lse[row] = l;
  row_loss[row] = label_valid(labels[row], ignore, vocab_total) ? l - t : 0.f;
}

template <int NT>
__global__ void __launch_bounds__(NT) ce_loss_finish_kernel(const float* __restrict__ row_loss,
                                                            const int64_t* __restrict__ labels, int M,
                                                            long vocab_total, long ignore, float* __restrict__ loss,
                                                            float* __restrict__ inv_n) {
  __shared__ float red[32];
  __shared__ int cnt[32];
  float s = 0.f;
  int c = 0;
  for (int i = threadIdx.x; i < M; i += NT) {
    s += row_loss[i];
    c += label_valid(labels[i], ignore, vocab_total) ? 1 : 0;
  }
  s = warp_sum(s);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    red[w] = s;
    cnt[w] = c;
  }
  __syncthreads();
  if (w == 0) {
    float t = l < NT / 32 ? red[l] : 0.f;
    int k = l < NT / 32 ? cnt[l] : 0;
    t = warp_sum(t);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) k += __shfl_xor_sync(0xffffffffu, k, o);
    if (l == 0) {
      *loss = k > 0 ? t / (float)k : __int_as_float(0x7fc00000);
      *inv_n = k > 0 ? 1.f / (float)k : 0.f;
    }
  }
}

}  // namespace ce
}  // namespace dtb

using namespace dtb;

static cudaStream_t ce_stream() { return at::cuda::getCurrentCUDAStream(); }

// Reduce the head GEMM's statistics.  Without `xchg_bases` (vocabulary on this
// GPU): fills lse and row_loss.  With them (vocabulary split over the TP
// group): writes this rank's (m, s, t) rows at byte offset `xchg_off` of its
// heap; the caller runs a device barrier and then ce_peer_combine.
void ce_stats_reduce(torch::Tensor stats, torch::Tensor tgt, torch::Tensor labels, int64_t vocab_off, int64_t v_local,
                     int64_t vocab_total, int64_t ignore, torch::Tensor lse, torch::Tensor row_loss,
                     c10::optional<torch::Tensor> xchg) {
  TORCH_CHECK(stats.scalar_type() == at::kFloat && stats.is_contiguous() && stats.dim() == 2 && stats.size(1) % 2 == 0,
              "ce_stats_reduce: fp32 [M, 2 * blocks]");
  const c10::cuda::CUDAGuard g(stats.device());
  const int M = (int)stats.size(0), nblk = (int)(stats.size(1) / 2);
  TORCH_CHECK(labels.numel() == M && tgt.numel() == M && lse.numel() == M && row_loss.numel() == M,
              "ce_stats_reduce: row counts differ");
  if (M == 0) return;
  float4* x = nullptr;
  if (xchg.has_value()) {
    TORCH_CHECK(xchg->numel() * xchg->element_size() >= (long)M * 16 && (reinterpret_cast<uintptr_t>(xchg->data_ptr()) & 15) == 0,
                "ce_stats_reduce: exchange rows must hold M x 16 bytes, 16-byte aligned");
    x = reinterpret_cast<float4*>(xchg->data_ptr());
  }
  constexpr int kWarps = 8;
  ce::ce_stats_reduce_kernel<<<(M + kWarps - 1) / kWarps, 32 * kWarps, 0, ce_stream()>>>(
      reinterpret_cast<const float2*>(stats.data_ptr<float>()), tgt.data_ptr<float>(), labels.data_ptr<int64_t>(), M,
      nblk, (long)vocab_off, (long)v_local, (long)vocab_total, (long)ignore, lse.data_ptr<float>(),
      row_loss.data_ptr<float>(), x);
  DTB_LAUNCH_CHECK();
}

void ce_peer_combine(std::vector<int64_t> bases, int64_t off, torch::Tensor labels, int64_t vocab_total, int64_t ignore,
                     torch::Tensor lse, torch::Tensor row_loss) {
  DTB_CHECK(bases.size() >= 1 && bases.size() <= (size_t)ce::MAX_PEERS, "ce_peer_combine: group size %zu", bases.size());
  DTB_CHECK(off % 16 == 0, "ce_peer_combine: offset must be 16-byte aligned");
  const c10::cuda::CUDAGuard g(lse.device());
  const int M = (int)labels.numel();
  if (M == 0) return;
  ce::PeerPtrs p{};
  for (size_t i = 0; i < bases.size(); ++i) p.base[i] = reinterpret_cast<uint8_t*>(bases[i]);
  ce::ce_peer_combine_kernel<<<(M + 255) / 256, 256, 0, ce_stream()>>>(
      p, (long)off, (int)bases.size(), labels.data_ptr<int64_t>(), M, (long)vocab_total, (long)ignore,
      lse.data_ptr<float>(), row_loss.data_ptr<float>());
  DTB_LAUNCH_CHECK();
}

// loss = sum(row_loss) / n_valid (NaN when no label is valid), inv_n = 1 / n_valid (0 then).
void ce_loss_finish(torch::Tensor row_loss, torch::Tensor labels, int64_t vocab_total, int64_t ignore,
                    torch::Tensor loss, torch::Tensor inv_n) {
  const c10::cuda::CUDAGuard g(row_loss.device());
  const int M = (int)row_loss.numel();
  TORCH_CHECK(labels.numel() == M, "ce_loss_finish: row counts differ");
  ce::ce_loss_finish_kernel<1024><<<1, 1024, 0, ce_stream()>>>(row_loss.data_ptr<float>(), labels.data_ptr<int64_t>(),
                                                              M, (long)vocab_total, (long)ignore,
                                                              loss.data_ptr<float>(), inv_n.data_ptr<float>());
  DTB_LAUNCH_CHECK();
}
