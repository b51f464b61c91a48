// NVLink peer-memory transport: symmetric heaps, device barriers and the
// ZeRO collectives, as this package's own kernels (sm_100a).
//
// A symmetric heap is one cudaMalloc per rank of the same size, exported with
// cudaIpcGetMemHandle and mapped into every peer of the group
// (cudaIpcOpenMemHandle), so every rank holds a device pointer to every
// peer's heap.  NVSwitch gives each GPU full bandwidth to every peer, so the
// collectives are one-step pulls: rank r reads what it needs straight from the
// peers (16-byte loads that bypass L1) instead of rotating chunks around a ring.
//
// Ordering: data is published with a system-scope release store of a flag
// (epoch numbers, monotonically increasing per channel, so nothing is ever
// reset) and consumed after an acquire load of that flag.  Every spin is
// bounded by %globaltimer: past the limit the kernel records
// ERR_PEER_TIMEOUT in the device error word and returns.
//
// No TMA, no multicast, no multimem: plain loads and stores over NVLink.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace dtb {
namespace comm {

constexpr int MAX_PEERS = 8;

struct PeerPtrs {
  uint8_t* base[MAX_PEERS];  // heap base of every rank (base[rank] is local)
};

// ---------------------------------------------------------------- barrier
// flags: [MAX_PEERS] u32 per channel at `flag_off` inside every heap; rank r
// writes slot r of every peer, then waits for all slots of its own.
__global__ void peer_barrier_kernel(PeerPtrs peers, long flag_off, int rank, int size, uint32_t epoch,
                                    uint64_t timeout_ns, int* err) {
  const int p = threadIdx.x;
  if (p < size) {
    __threadfence_system();
    st_release_sys(reinterpret_cast<uint32_t*>(peers.base[p] + flag_off) + rank, epoch);
  }
  __syncwarp();
  if (p < size) wait_flag(reinterpret_cast<const uint32_t*>(peers.base[rank] + flag_off) + p, epoch, timeout_ns, err);
  __syncwarp();
  __threadfence_system();
}

// ---------------------------------------------------------------- all-gather
// out[p * shard_bytes : (p+1) * shard_bytes] = heap_p[src_off : src_off + shard_bytes]
__global__ void peer_all_gather_kernel(PeerPtrs peers, long src_off, long shard_bytes, int size, uint8_t* out) {
  const long nv = shard_bytes / 16;
  for (int p = 0; p < size; ++p) {
    const uint8_t* src = peers.base[p] + src_off;
    uint8_t* dst = out + p * shard_bytes;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < nv; i += (long)gridDim.x * blockDim.x)
      *reinterpret_cast<uint4*>(dst + i * 16) = ld_cg_v4(src + i * 16);
  }
}

// ---------------------------------------------------------------- reduce-scatter
// out[i] = scale * sum_{p = 0..size-1} grad_p[rank * n + i]   (fp32, fixed order)
// and, for the gradient norm, part[blockIdx.x] = sum_i w_i * out[i]^2 with
// w_i = 1 below `split` (TP-sharded entries) and rep_w from there on
// (TP-replicated entries, which every TP rank holds: rep_w = 1/tp), so the
// norm needs no second pass over the shard.
template <int NT>
__global__ void __launch_bounds__(NT) peer_reduce_scatter_kernel(PeerPtrs peers, long grad_off, long n, int rank,
                                                                int size, float scale, float* out, float* part,
                                                                long split, float rep_w) {
  __shared__ float red[32];
  float ss = 0.f;
  const long nv = n / 4;
  for (long i = blockIdx.x * (long)NT + threadIdx.x; i < nv; i += (long)gridDim.x * NT) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = 0; p < size; ++p) {
      const float* g = reinterpret_cast<const float*>(peers.base[p] + grad_off) + (long)rank * n;
      const uint4 v = ld_cg_v4(g + i * 4);
      acc.x += __uint_as_float(v.x);
      acc.y += __uint_as_float(v.y);
      acc.z += __uint_as_float(v.z);
      acc.w += __uint_as_float(v.w);
    }
    acc.x *= scale; acc.y *= scale; acc.z *= scale; acc.w *= scale;
    reinterpret_cast<float4*>(out)[i] = acc;
    const long e = i * 4;
    if (e + 4 <= split) {
      ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
    } else if (e >= split) {
      ss += rep_w * (acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w);
    } else {
      ss += (e < split ? 1.f : rep_w) * acc.x * acc.x + (e + 1 < split ? 1.f : rep_w) * acc.y * acc.y +
            (e + 2 < split ? 1.f : rep_w) * acc.z * acc.z + (e + 3 < split ? 1.f : rep_w) * acc.w * acc.w;
    }
  }
  // per-block partial of sum(out^2), fixed order
  float v = warp_sum(ss);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    float t = l < NT / 32 ? red[l] : 0.f;
    t = warp_sum(t);
    if (l == 0 && part) part[blockIdx.x] = t;
  }
}

// ---------------------------------------------------------------- all-reduce
// out = sum_p heap_p[src_off ...] (+ residual), bf16, fixed rank order, so all
// ranks produce identical bits.  One-shot: every rank reads every peer.
__global__ void peer_all_reduce_bf16_kernel(PeerPtrs peers, long src_off, long n, int size,
                                            const __nv_bfloat16* residual, __nv_bfloat16* out) {
  const long nv = n / 8;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < nv; i += (long)gridDim.x * blockDim.x) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int p = 0; p < size; ++p) {
      const uint4 v = ld_cg_v4(peers.base[p] + src_off + i * 16);
      const uint32_t* u = &v.x;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = unpack_bf16x2(u[k]);
        acc[2 * k] += f.x;
        acc[2 * k + 1] += f.y;
      }
    }
    if (residual) {
      const uint4 r = *reinterpret_cast<const uint4*>(residual + i * 8);
      const uint32_t* u = &r.x;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = unpack_bf16x2(u[k]);
        acc[2 * k] += f.x;
        acc[2 * k + 1] += f.y;
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + i * 8) = o;
  }
}

// rows [row0, row0 + rows) of a [*, cols] bf16 matrix: out = sum over peers (reduce-scatter by rows)
__global__ void peer_reduce_rows_bf16_kernel(PeerPtrs peers, long src_off, long row0, long rows, long cols, int size,
                                             __nv_bfloat16* out) {
  const long nv = rows * cols / 8;
  const long base = row0 * cols * 2;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < nv; i += (long)gridDim.x * blockDim.x) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int p = 0; p < size; ++p) {
      const uint4 v = ld_cg_v4(peers.base[p] + src_off + base + i * 16);
      const uint32_t* u = &v.x;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = unpack_bf16x2(u[k]);
        acc[2 * k] += f.x;
        acc[2 * k + 1] += f.y;
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + i * 8) = o;
  }
}

// Bounded wait on a flag that nothing sets: the timeout path of every peer
// wait, exercised by the tests without involving a second GPU.
__global__ void wait_flag_probe_kernel(const uint32_t* flag, uint32_t target, uint64_t timeout_ns, int* err) {
  if (threadIdx.x == 0) wait_flag(flag, target, timeout_ns, err);
}

static PeerPtrs make_peers(const std::vector<int64_t>& bases) {
  DTB_CHECK(bases.size() >= 1 && bases.size() <= MAX_PEERS, "peer group size %zu not in [1, %d]", bases.size(),
            MAX_PEERS);
  PeerPtrs p{};
  for (size_t i = 0; i < bases.size(); ++i) p.base[i] = reinterpret_cast<uint8_t*>(bases[i]);
  return p;
}

static int blocks_for(long work_items, int nt) {
  long b = (work_items + nt - 1) / nt;
  return (int)std::max<long>(1, std::min<long>(b, 8L * device_sm_count()));
}

// The gradient reduce-scatter overlaps the backward GEMMs on a side stream:
// DTB_RS_CTAS caps its grid (default 2 per SM) so it leaves the SMs' issue
// slots mostly to the GEMM that shares them.
static int rs_blocks_for(long work_items, int nt) {
  static long cap = -1;
  if (cap < 0) {
    const char* e = getenv("DTB_RS_CTAS");
    cap = (e != nullptr && atol(e) > 0) ? atol(e) : 2L * device_sm_count();
  }
  long b = (work_items + nt - 1) / nt;
  return (int)std::max<long>(1, std::min<long>(b, cap));
}

}  // namespace comm
}  // namespace dtb

using namespace dtb::comm;
static cudaStream_t cs() { return at::cuda::getCurrentCUDAStream(); }

// ------------------------------------------------------------------ heaps
// Raw device allocation (not from the caching allocator: IPC handles name
// whole allocations) wrapped in a uint8 tensor that frees it.
torch::Tensor sym_malloc(int64_t nbytes) {
  void* p = nullptr;
  DTB_CUDA(cudaMalloc(&p, nbytes));
  DTB_CUDA(cudaMemset(p, 0, nbytes));
  int dev = 0;
  DTB_CUDA(cudaGetDevice(&dev));
  return torch::from_blob(
      p, {nbytes}, [](void* q) { cudaFree(q); }, torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, dev));
}

torch::Tensor ipc_handle(torch::Tensor heap) {
  cudaIpcMemHandle_t h;
  DTB_CUDA(cudaIpcGetMemHandle(&h, heap.data_ptr()));
  auto out = torch::empty({(long)sizeof(h)}, torch::kUInt8);
  std::memcpy(out.data_ptr(), &h, sizeof(h));
  return out;
}

int64_t ipc_open(torch::Tensor handle) {
  DTB_CHECK(handle.numel() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data_ptr(), sizeof(h));
  void* p = nullptr;
  DTB_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr) { DTB_CUDA(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr))); }

// ------------------------------------------------------------------ collectives
void peer_barrier(std::vector<int64_t> bases, int64_t flag_off, int64_t rank, int64_t epoch, double timeout_s) {
  auto peers = make_peers(bases);
  peer_barrier_kernel<<<1, 32, 0, cs()>>>(peers, flag_off, (int)rank, (int)bases.size(), (uint32_t)epoch,
                                          (uint64_t)(timeout_s * 1e9), dtb_error_word());
  DTB_LAUNCH_CHECK();
}

// flag word `rank` at flag_off of every rank's heap := epoch (release, system scope),
// after everything earlier on the stream (e.g. the copy that staged this rank's rows)
__global__ void peer_signal_kernel(PeerPtrs peers, long flag_off, int rank, int size, uint32_t epoch) {
  const int p = threadIdx.x;
  if (p < size) {
    __threadfence_system();
    dtb::st_release_sys(reinterpret_cast<uint32_t*>(peers.base[p] + flag_off) + rank, epoch);
  }
}

void peer_signal(std::vector<int64_t> bases, int64_t flag_off, int64_t rank, int64_t epoch) {
  auto peers = make_peers(bases);
  peer_signal_kernel<<<1, 32, 0, cs()>>>(peers, flag_off, (int)rank, (int)bases.size(), (uint32_t)epoch);
  DTB_LAUNCH_CHECK();
}

void peer_all_gather(std::vector<int64_t> bases, int64_t src_off, int64_t shard_bytes, torch::Tensor out) {
  DTB_CHECK(shard_bytes % 16 == 0 && src_off % 16 == 0, "all-gather needs 16-byte aligned shards");
  DTB_CHECK(out.numel() * out.element_size() >= shard_bytes * (long)bases.size(), "all-gather output too small");
  auto peers = make_peers(bases);
  peer_all_gather_kernel<<<blocks_for(shard_bytes / 16, 256), 256, 0, cs()>>>(
      peers, src_off, shard_bytes, (int)bases.size(), reinterpret_cast<uint8_t*>(out.data_ptr()));
  DTB_LAUNCH_CHECK();
}

// All-gather on the copy engines: one cudaMemcpyAsync per rank from its heap
// (peer memory through the IPC mapping) into this rank's output, on the
// current stream.  No SM runs it, so a gather overlapped with GEMMs takes no
// issue slots or registers from them.  Valid when every source shard is final
// before the stream reaches the copies (ZeRO parameter shards: written by the
// optimizer step, followed by a device barrier).
// Rank p's piece is read at bases[p] + src_off + p * src_stride (src_stride 0:
// every rank's piece at the same offset); skip_rank's piece is not copied (it
// is already in place when `out` is that rank's own heap buffer).
void peer_all_gather_ce(std::vector<int64_t> bases, int64_t src_off, int64_t shard_bytes, torch::Tensor out,
                        int64_t src_stride, int64_t skip_rank) {
  DTB_CHECK(out.numel() * out.element_size() >= shard_bytes * (long)bases.size(), "all-gather output too small");
  auto* dst = reinterpret_cast<uint8_t*>(out.data_ptr());
  for (size_t p = 0; p < bases.size(); ++p) {
    if ((int64_t)p == skip_rank) continue;
    DTB_CUDA(cudaMemcpyAsync(dst + p * shard_bytes,
                             reinterpret_cast<const uint8_t*>(bases[p]) + src_off + (long)p * src_stride, shard_bytes,
                             cudaMemcpyDeviceToDevice, cs()));
  }
}

// Reduce-scatter (mean over the group) of an fp32 gradient buffer.  `part`
// (optional, fp32, at least reduce_scatter_blocks(n) entries) receives the
// per-block weighted sums of squares of the result (see the kernel); entries
// past the blocks used are left untouched.
int64_t reduce_scatter_blocks(int64_t n) { return rs_blocks_for(n / 4, 256); }

void peer_reduce_scatter(std::vector<int64_t> bases, int64_t grad_off, int64_t rank, double scale, torch::Tensor out,
                         c10::optional<torch::Tensor> part, int64_t split, double rep_w) {
  DTB_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous(), "reduce-scatter: fp32 shard");
  const long n = out.numel();
  DTB_CHECK(n % 4 == 0 && grad_off % 16 == 0, "reduce-scatter needs 16-byte aligned shards");
  auto peers = make_peers(bases);
  const int nb = rs_blocks_for(n / 4, 256);
  float* pp = nullptr;
  if (part.has_value()) {
    DTB_CHECK(part->scalar_type() == at::kFloat && part->is_contiguous() && part->numel() >= nb,
              "reduce-scatter: partials need %d fp32 entries", nb);
    pp = part->data_ptr<float>();
  }
  peer_reduce_scatter_kernel<256><<<nb, 256, 0, cs()>>>(peers, grad_off, n, (int)rank, (int)bases.size(), (float)scale,
                                                        out.data_ptr<float>(), pp, (long)split, (float)rep_w);
  DTB_LAUNCH_CHECK();
}

void peer_all_reduce_bf16(std::vector<int64_t> bases, int64_t src_off, c10::optional<torch::Tensor> residual,
                          torch::Tensor out) {
  DTB_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() % 8 == 0, "all-reduce: bf16");
  auto peers = make_peers(bases);
  const long n = out.numel();
  peer_all_reduce_bf16_kernel<<<blocks_for(n / 8, 256), 256, 0, cs()>>>(
      peers, src_off, n, (int)bases.size(),
      residual.has_value() ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr()) : nullptr,
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  DTB_LAUNCH_CHECK();
}

void peer_reduce_rows_bf16(std::vector<int64_t> bases, int64_t src_off, int64_t row0, int64_t cols, torch::Tensor out) {
  DTB_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && cols % 8 == 0, "reduce rows: bf16");
  auto peers = make_peers(bases);
  const long rows = out.numel() / cols;
  peer_reduce_rows_bf16_kernel<<<blocks_for(rows * cols / 8, 256), 256, 0, cs()>>>(
      peers, src_off, row0, rows, cols, (int)bases.size(), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  DTB_LAUNCH_CHECK();
}

void wait_flag_probe(torch::Tensor flag, int64_t target, double timeout_s) {
  wait_flag_probe_kernel<<<1, 32, 0, cs()>>>(reinterpret_cast<const uint32_t*>(flag.data_ptr()), (uint32_t)target,
                                             (uint64_t)(timeout_s * 1e9), dtb_error_word());
  DTB_LAUNCH_CHECK();
}
