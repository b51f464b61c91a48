// Persistent warp-specialised tcgen05 GEMM for sm_100a with fused epilogues.
//
//   C[M,N] = sum_k A(m,k) * B(n,k)      bf16 inputs, fp32 accumulation in TMEM
//
// A and B are each K-major (reduction axis contiguous) or MN-major, so the
// three products of a linear layer (forward x.W^T, input grad dy.W, weight
// grad dy^T.x) all run without transposing anything in memory.
//
// CTA = 10 warps, one CTA per SM, grid = min(#tiles, #SMs), static tile stride:
//   warp 0      TMA producer: one elected thread streams 128x64 A and BNx64 B
//               tiles (128-byte swizzle) into a STAGES-deep smem ring;
//   warp 1      owns the TMEM allocation (2 x BN fp32 columns: the accumulator
//               is double buffered) and one thread issues tcgen05.mma
//               128xBNx16 instructions; tcgen05.commit releases smem stages
//               and publishes finished accumulators;
//   warps 2-9   epilogue, two warpgroups taking alternate tiles (one per TMEM
//               accumulator buffer): tcgen05.ld the accumulator (warp w reads TMEM lanes
//               32*(w%4)..+31 = tile rows), apply the fused epilogue and store,
//               while the MMA warp already accumulates the next tile into the
//               other TMEM buffer.
//
// Epilogues: bf16 / fp32 store (optional device-scalar alpha), fp32
// accumulate into an existing buffer (weight gradients), residual add,
// rotate-half RoPE on the q/k columns, SwiGLU (B rows n and F+n of the
// stacked [W_gate; W_up] land in one 256-wide tile, the epilogue writes
// silu(g)*u plus g and u for the backward), and the two halves of the fused
// LM-head cross-entropy: per (row, column block) log-sum-exp statistics and
// the target logit with no logits written (forward), and the logit gradient
// (softmax - onehot) * coef recomputed from the accumulator (backward).
//
// No TMA multicast anywhere: each CTA loads its own tiles.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include <cmath>

#include "common.cuh"

bool dtb_debug_enabled();

namespace dtb {

enum Epi : int {
  EPI_STORE_BF16 = 0,
  EPI_STORE_F32 = 1,
  EPI_ACC_F32 = 2,
  EPI_RESIDUAL = 3,
  EPI_ROPE = 4,
  EPI_SWIGLU = 5,
  EPI_PEER_AR = 6,  // D = sum over the TP group of every rank's tile (+ R), through NVLink peer memory
  EPI_CE_STATS = 7,     // per (row, column block): (max, sum exp(x - max)) -> ce_stats; x[label] -> ce_tgt
  EPI_CE_GRAD = 8,      // D(bf16) = (exp(x - lse[row]) - [col == label]) * coef, coef = *alpha * *ce_inv_n
  EPI_ACC_BF16OUT = 9,  // D(bf16) = acc + F[row, col], F an fp32 matrix (last step of a K-chunked GEMM)
};

constexpr int MAX_PEERS = 8;

struct GemmArgs {
  int M, N, K;          // N: output columns (for SwiGLU: F)
  void* D;
  long ldd;
  const __nv_bfloat16* R;
  long ldr;
  const float* alpha;
  const float* cos_t;
  const float* sin_t;
  int rope_cols, head_dim, seqlen;
  __nv_bfloat16* D2;
  long ldd2;
  int ffn;
  int m_blocks, n_blocks, k_iters, num_tiles;
  int flag_tiles;       // EPI_PEER_AR: flag slots per rank (one per 128-row slab x column block)
  int* err;
  // EPI_PEER_AR: symmetric heaps of the group, staging area and flags inside them
  uint8_t* peer_base[MAX_PEERS];
  int peer_n, peer_rank;
  int rs_row0, rs_rows;  // rs_rows > 0: reduce-scatter, this rank sums rows [rs_row0, rs_row0 + rs_rows) only
  int two_shot;          // all-reduce in two steps: each tile's owner sums it, the others copy the sum
  long stage_off, flag_off;
  uint32_t epoch;
  uint64_t timeout_ns;
  // EPI_CE_STATS / EPI_CE_GRAD: labels of the rows, global vocabulary index of
  // output column 0, vocabulary size, ignored label
  const int64_t* labels;
  long vocab_off, vocab_total, ignore;
  float* ce_stats;        // [M, n_blocks] float2
  float* ce_tgt;          // [M]
  const float* ce_lse;    // [M]
  const float* ce_inv_n;  // device scalar 1 / (number of valid labels)
  const float* acc_in;    // EPI_ACC_BF16OUT: fp32 [M, N] with row stride ld_acc
  long ld_acc;
  // fp32 outputs: the K range split over `ksplit` work units per tile (see splitk_wait)
  int ksplit;
  int* sk_flags;
  uint32_t sk_epoch;
  int d_v8;               // fp32 D: base 32-byte aligned and ldd % 8 == 0 (256-bit stores)
  int d_tma;              // tma_store_epi epilogues: D (and R or D2) go through tensor maps
  // AG (all-gather fused in front of the GEMM, sequence parallelism): A is the
  // gathered [M, K] buffer `ag_out`, filled by the kernel's copier warps from this
  // rank's rows `ag_local` and the peers' staged rows (peer_base[p] + stage_off)
  const __nv_bfloat16* ag_local;
  __nv_bfloat16* ag_out;
  int ag_rows;            // rows per rank (a multiple of the tile height)
  int ag_mrot;            // m-blocks of this rank's rows: tiles start there
  long ag_staged_off;     // per-rank "rows staged" flags inside every heap
  uint32_t ag_epoch;      // this call's epoch (staged flags)
  uint32_t* ag_count;     // per-128-row chunk: rows copied, cumulative over launches
  uint32_t ag_target;     // count a chunk reaches once this launch has copied it
};

constexpr int BM = 128;
constexpr int BK = 64;
// ring depth when a stage is 32 KB per CTA (CTA pairs, or 128-column tiles):
// (7 stages measured no faster: 1256 vs 1267 TFLOP/s at 4096^3, so 6 leave room)
constexpr int kStages32K = 6;
constexpr int GROUP_M = 16;

__device__ __forceinline__ void tile_coords(int tile, int mblocks, int nblocks, int& mb, int& nb) {
  const int per_group = GROUP_M * nblocks;
  const int g = tile / per_group;
  const int first = g * GROUP_M;
  const int gm = min(GROUP_M, mblocks - first);
  const int r = tile - g * per_group;
  mb = first + r % gm;
  nb = r / gm;
}

// epilogues whose output leaves through TMA bulk stores (when args.d_tma is set)
__host__ __device__ constexpr bool tma_store_epi(int epi) {
  return epi == EPI_STORE_BF16 || epi == EPI_STORE_F32 || epi == EPI_ACC_F32 || epi == EPI_RESIDUAL ||
         epi == EPI_ROPE || epi == EPI_SWIGLU;
}

// TSTORE: 4 KB of shared memory per epilogue warp for the TMA-store epilogues
template <int BN, int STAGES, bool PAIR = false, bool TSTORE = false>
struct SmemLayout {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = (PAIR ? BN / 2 : BN) * BK * 2;  // a CTA pair splits B by columns
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STG_OFF = STAGES * STAGE_BYTES;
  static constexpr int STG_BYTES = TSTORE ? 8 * 4096 : 0;
  static constexpr int BAR_OFF = STG_OFF + STG_BYTES;
  static constexpr int RBAR_OFF = BAR_OFF + (2 * STAGES + 4) * 8 + 16;  // TSTORE: one barrier per epilogue warp
  static constexpr int TOTAL = RBAR_OFF + (TSTORE ? 8 * 8 : 0) + 1024;   // + alignment slack
  static_assert(TOTAL <= 232448, "shared memory per CTA");
};

// ---------------------------------------------------------------- epilogue
template <int EPI>
__device__ __forceinline__ void store_chunk(const GemmArgs& a, int row, int col, float (&v)[32], int ncols_valid) {
  if (a.alpha != nullptr) {
    const float s = *a.alpha;
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] *= s;
  }
  if (EPI == EPI_STORE_F32 || EPI == EPI_ACC_F32) {
    float* p = reinterpret_cast<float*>(a.D) + (long)row * a.ldd + col;
    if (ncols_valid >= 32 && a.d_v8) {
      if (EPI == EPI_ACC_F32) {
        float c[32];
#pragma unroll
        for (int i = 0; i < 32; i += 8) ld_global_v8f(p + i, c + i);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] += c[i];
      }
#pragma unroll
      for (int i = 0; i < 32; i += 8) st_global_v8f(p + i, v + i);
    } else if (ncols_valid >= 32) {
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        float4 o = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        if (EPI == EPI_ACC_F32) {
          float4 c = *reinterpret_cast<float4*>(p + i);
          o.x += c.x; o.y += c.y; o.z += c.z; o.w += c.w;
        }
        *reinterpret_cast<float4*>(p + i) = o;
      }
    } else {
      for (int i = 0; i < ncols_valid; ++i) p[i] = (EPI == EPI_ACC_F32 ? p[i] : 0.f) + v[i];
    }
    return;
  }
  // bf16 outputs
  __nv_bfloat16* p = reinterpret_cast<__nv_bfloat16*>(a.D) + (long)row * a.ldd + col;
  if (EPI == EPI_RESIDUAL) {
    const __nv_bfloat16* r = a.R + (long)row * a.ldr + col;
    if (ncols_valid >= 32) {
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        uint4 q = *reinterpret_cast<const uint4*>(r + i);
        float2 f0 = unpack_bf16x2(q.x), f1 = unpack_bf16x2(q.y), f2 = unpack_bf16x2(q.z), f3 = unpack_bf16x2(q.w);
        v[i] += f0.x; v[i + 1] += f0.y; v[i + 2] += f1.x; v[i + 3] += f1.y;
        v[i + 4] += f2.x; v[i + 5] += f2.y; v[i + 6] += f3.x; v[i + 7] += f3.y;
      }
    } else {
      for (int i = 0; i < ncols_valid; ++i) v[i] += __bfloat162float(r[i]);
    }
  }
  if (ncols_valid >= 32) {
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
      uint4 o;
      o.x = pack_bf16x2(v[i], v[i + 1]);
      o.y = pack_bf16x2(v[i + 2], v[i + 3]);
      o.z = pack_bf16x2(v[i + 4], v[i + 5]);
      o.w = pack_bf16x2(v[i + 6], v[i + 7]);
      *reinterpret_cast<uint4*>(p + i) = o;
    }
  } else {
    for (int i = 0; i < ncols_valid; ++i) p[i] = __float2bfloat16_rn(v[i]);
  }
}

__device__ __forceinline__ void store_bf16_32(__nv_bfloat16* p, const float (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    uint4 o;
    o.x = pack_bf16x2(v[i], v[i + 1]);
    o.y = pack_bf16x2(v[i + 2], v[i + 3]);
    o.z = pack_bf16x2(v[i + 4], v[i + 5]);
    o.w = pack_bf16x2(v[i + 6], v[i + 7]);
    *reinterpret_cast<uint4*>(p + i) = o;
  }
}

// rotate-half RoPE of the pair (x1, x2) = (column p, column p + hd/2) of a head,
// each product rounded on its own (no contraction) so every epilogue gives the same bits
__device__ __forceinline__ float rope_lo(float x1, float x2, float c, float s) {
  return __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
}
__device__ __forceinline__ float rope_hi(float x1, float x2, float c, float s) {
  return __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
}
__device__ __forceinline__ float swiglu_h(float gr, float ur) { return __fdividef(gr, 1.f + __expf(-gr)) * ur; }

template <int BN, int EPI>
__device__ __forceinline__ void epilogue_tile(const GemmArgs& a, uint32_t tbase, int mb, int nb, int quad,
                                              int lane) {
  const int row = mb * BM + quad * 32 + lane;
  const bool row_ok = row < a.M;
  const uint32_t trow = tbase + ((uint32_t)(quad * 32) << 16);
  if (EPI == EPI_SWIGLU) {
    // TMEM columns [0,128): gate, [128,256): up, for output columns nb*128 + [0,128)
    const int c0 = nb * 128;
#pragma unroll 1
    for (int c = 0; c < 128; c += 32) {
      uint32_t rg[32], ru[32];
      tmem_ld32_async(trow + c, rg);
      tmem_ld32_async(trow + 128 + c, ru);
      tmem_wait_ld();
      tmem_regs(rg);
      tmem_regs(ru);
      if (row_ok) {
        float g[32], u[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) g[i] = __uint_as_float(rg[i]), u[i] = __uint_as_float(ru[i]);
        __nv_bfloat16* gp = a.D2 + (long)row * a.ldd2 + c0 + c;
        __nv_bfloat16* up = gp + a.ffn;
        // the backward recomputes from the rounded g/u, so round first
        float gr[32], ur[32], h[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          gr[i] = __bfloat162float(__float2bfloat16_rn(g[i]));
          ur[i] = __bfloat162float(__float2bfloat16_rn(u[i]));
          h[i] = swiglu_h(gr[i], ur[i]);
        }
        store_bf16_32(gp, gr);
        store_bf16_32(up, ur);
        store_bf16_32(reinterpret_cast<__nv_bfloat16*>(a.D) + (long)row * a.ldd + c0 + c, h);
      }
    }
    return;
  }
  constexpr float kLog2e = 1.4426950408889634f;
  if (EPI == EPI_CE_STATS) {
    // online log-sum-exp over this tile's columns of the row, base 2
    const int n0 = nb * BN;
    const long lab = row_ok ? a.labels[row] : a.ignore;
    const long tc = (lab == a.ignore) ? -1 : lab - a.vocab_off - n0;  // target column inside this tile
    float m = -INFINITY, s = 0.f, t = 0.f;
    bool hit = false;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      if (n0 + c >= a.N) break;
      float v[32];
      tmem_ld32(trow + c, v);
      const int nv = min(32, a.N - (n0 + c));
      float cm = -INFINITY;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < nv) cm = fmaxf(cm, v[i]);
      if (tc >= c && tc < c + 32) {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (tc == c + i) t = v[i];
        hit = true;
      }
      const float mn = fmaxf(m, cm);
      const float mb = mn * kLog2e;
      float cs = 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (i < nv) cs += ex2_approx(fmaf(v[i], kLog2e, -mb));
      s = s * ex2_approx((m - mn) * kLog2e) + cs;
      m = mn;
    }
    if (row_ok) {
      reinterpret_cast<float2*>(a.ce_stats)[(long)row * a.n_blocks + nb] = make_float2(m, s);
      if (hit) a.ce_tgt[row] = t;
    }
    return;
  }
  if (EPI == EPI_CE_GRAD) {
    const int n0 = nb * BN;
    const long lab = row_ok ? a.labels[row] : a.ignore;
    const bool valid = row_ok && lab != a.ignore && lab >= 0 && lab < a.vocab_total;
    const long tc = valid ? lab - a.vocab_off - n0 : -1;
    const float coef = valid ? (*a.alpha) * (*a.ce_inv_n) : 0.f;
    const float lse2 = row_ok ? a.ce_lse[row] * kLog2e : 0.f;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      if (n0 + c >= a.N) break;
      float v[32];
      tmem_ld32(trow + c, v);
      if (row_ok) {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          v[i] = (ex2_approx(fmaf(v[i], kLog2e, -lse2)) - (tc == c + i ? 1.f : 0.f)) * coef;
        const int nv = min(32, a.N - (n0 + c));
        __nv_bfloat16* p = reinterpret_cast<__nv_bfloat16*>(a.D) + (long)row * a.ldd + n0 + c;
        if (nv >= 32) store_bf16_32(p, v);
        else
          for (int i = 0; i < nv; ++i) p[i] = __float2bfloat16_rn(v[i]);
      }
    }
    return;
  }
  if (EPI == EPI_ACC_BF16OUT) {
    const int n0 = nb * BN;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      if (n0 + c >= a.N) break;
      float v[32];
      tmem_ld32(trow + c, v);
      if (row_ok) {
        const int nv = min(32, a.N - (n0 + c));
        const float* f = a.acc_in + (long)row * a.ld_acc + n0 + c;
        __nv_bfloat16* p = reinterpret_cast<__nv_bfloat16*>(a.D) + (long)row * a.ldd + n0 + c;
        if (nv >= 32) {
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            const float4 q = *reinterpret_cast<const float4*>(f + i);
            v[i] += q.x; v[i + 1] += q.y; v[i + 2] += q.z; v[i + 3] += q.w;
          }
          store_bf16_32(p, v);
        } else {
          for (int i = 0; i < nv; ++i) p[i] = __float2bfloat16_rn(v[i] + f[i]);
        }
      }
    }
    return;
  }
  const int n0 = nb * BN;
  if (EPI == EPI_ROPE) {
    const int hd = a.head_dim, half = hd >> 1;
    // this row's table rows (pos < seqlen also for rows past M, which are not stored)
    const int pos = row % a.seqlen;
    const float4* crow = reinterpret_cast<const float4*>(a.cos_t + (long)pos * hd);
    const float4* srow = reinterpret_cast<const float4*>(a.sin_t + (long)pos * hd);
#pragma unroll 1
    for (int h0 = 0; h0 < BN; h0 += hd) {
      const int col = n0 + h0;
      if (col >= a.N) break;
      if (col < a.rope_cols) {
#pragma unroll 1
        for (int j = 0; j < half; j += 32) {
          // table loads first, then both TMEM loads under one wait: the L2 and
          // TMEM latencies overlap instead of adding up
          float4 c4[8], s4[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            c4[q] = __ldg(crow + (j >> 2) + q);
            s4[q] = __ldg(srow + (j >> 2) + q);
          }
          uint32_t r1[32], r2[32];
          tmem_ld32_async(trow + h0 + j, r1);
          tmem_ld32_async(trow + h0 + half + j, r2);
          tmem_wait_ld();
          tmem_regs(r1);
          tmem_regs(r2);
          if (row_ok) {
            const float* cs = reinterpret_cast<const float*>(c4);
            const float* sn = reinterpret_cast<const float*>(s4);
            float y1[32], y2[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float x1 = __uint_as_float(r1[i]), x2 = __uint_as_float(r2[i]);
              y1[i] = rope_lo(x1, x2, cs[i], sn[i]);
              y2[i] = rope_hi(x1, x2, cs[i], sn[i]);
            }
            __nv_bfloat16* p = reinterpret_cast<__nv_bfloat16*>(a.D) + (long)row * a.ldd + col + j;
            store_bf16_32(p, y1);
            store_bf16_32(p + half, y2);
          }
        }
      } else {
#pragma unroll 1
        for (int j = 0; j < hd; j += 64) {
          uint32_t r1[32], r2[32];
          tmem_ld32_async(trow + h0 + j, r1);
          tmem_ld32_async(trow + h0 + j + 32, r2);
          tmem_wait_ld();
          tmem_regs(r1);
          tmem_regs(r2);
          if (row_ok) {
            float v1[32], v2[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v1[i] = __uint_as_float(r1[i]), v2[i] = __uint_as_float(r2[i]);
            __nv_bfloat16* p = reinterpret_cast<__nv_bfloat16*>(a.D) + (long)row * a.ldd + col + j;
            store_bf16_32(p, v1);
            store_bf16_32(p + 32, v2);
          }
        }
      }
    }
    return;
  }
  if (EPI == EPI_RESIDUAL) {
    // residual rows are loaded before each TMEM read, so the global-load and
    // TMEM latencies overlap instead of adding up
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      if (n0 + c >= a.N) break;
      const int nv = min(32, a.N - (n0 + c));
      uint4 q[4];
      const bool vec = row_ok && nv >= 32;
      if (vec) {
        const uint4* rp = reinterpret_cast<const uint4*>(a.R + (long)row * a.ldr + n0 + c);
#pragma unroll
        for (int i = 0; i < 4; ++i) q[i] = __ldg(rp + i);
      }
      float v[32];
      tmem_ld32(trow + c, v);
      if (!row_ok) continue;
      if (!vec) {
        store_chunk<EPI_RESIDUAL>(a, row, n0 + c, v, nv);
        continue;
      }
      if (a.alpha != nullptr) {
        const float sc = *a.alpha;
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __fmul_rn(v[i], sc);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t* u = &q[i].x;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = unpack_bf16x2(u[k]);
          v[8 * i + 2 * k] = __fadd_rn(v[8 * i + 2 * k], f.x);
          v[8 * i + 2 * k + 1] = __fadd_rn(v[8 * i + 2 * k + 1], f.y);
        }
      }
      store_bf16_32(reinterpret_cast<__nv_bfloat16*>(a.D) + (long)row * a.ldd + n0 + c, v);
    }
    return;
  }
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    if (n0 + c >= a.N) break;
    float v[32];
    tmem_ld32(trow + c, v);
    if (row_ok) store_chunk<EPI>(a, row, n0 + c, v, min(32, a.N - (n0 + c)));
  }
}

// ---------------------------------------------------------------- TMA-store epilogue (bf16 D)
// Each epilogue warp converts 32 rows x 64 columns of its accumulator rows to
// bf16, writes them into its 4 KB staging slot in the 128-byte-swizzled layout
// of the D tensor map's [32 x 64] box, and one lane issues a bulk tensor store.
// The global writes then go out as whole 128-byte lines from the TMA unit
// instead of one 16-byte piece per thread and row from the load/store unit
// (measured: the row-per-thread stores held the tensor pipe at ~77% busy where
// an epilogue without stores reached ~91%).  Rows past M are clipped by the
// tensor map; before a slot is rewritten its previous store must have read it.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* m, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(m),
               "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_group0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

template <int BN>
__device__ __forceinline__ void epilogue_tma_store(const GemmArgs& a, const CUtensorMap* tmD, uint8_t* stg,
                                                   uint32_t tbase, int mb, int nb, int quad, int lane) {
  const uint32_t trow = tbase + ((uint32_t)(quad * 32) << 16);
  const int n0 = nb * BN;
  const int grow0 = mb * BM + quad * 32;
  const float sc = a.alpha != nullptr ? *a.alpha : 1.f;
#pragma unroll 1
  for (int c = 0; c < BN; c += 64) {
    if (n0 + c >= a.N) break;
    uint32_t r1[32], r2[32];
    tmem_ld32_async(trow + c, r1);
    tmem_ld32_async(trow + c + 32, r2);
    tmem_wait_ld();
    tmem_regs(r1);
    tmem_regs(r2);
    uint32_t pk[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      pk[i] = pack_bf16x2(__uint_as_float(r1[2 * i]) * sc, __uint_as_float(r1[2 * i + 1]) * sc);
      pk[16 + i] = pack_bf16x2(__uint_as_float(r2[2 * i]) * sc, __uint_as_float(r2[2 * i + 1]) * sc);
    }
    // the slot's previous store has read it
    if (lane == 0) bulk_wait_group_read0();
    __syncwarp();
    uint8_t* rowp = stg + lane * 128;
#pragma unroll
    for (int cc = 0; cc < 8; ++cc)
      *reinterpret_cast<uint4*>(rowp + ((cc ^ (lane & 7)) << 4)) =
          make_uint4(pk[4 * cc], pk[4 * cc + 1], pk[4 * cc + 2], pk[4 * cc + 3]);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tmD, stg, n0 + c, grow0);
      bulk_commit_group();
    }
  }
}

// fp32 D: a [32 rows x 32 columns] box (128 bytes per row) per store.  With
// ACC the box is added to D by the TMA unit (cp.reduce.async.bulk.tensor .add):
// the weight-gradient accumulation never reads D into the SM.  Each element is
// added once per launch, in the same fp32 operation as a load-add-store, so the
// result is the same bits.
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* m, const void* src, int c0, int c1) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(m),
               "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
}

template <int BN, bool ACC>
__device__ __forceinline__ void epilogue_tma_f32(const GemmArgs& a, const CUtensorMap* tmD, uint8_t* stg,
                                                 uint32_t tbase, int mb, int nb, int quad, int lane) {
  const uint32_t trow = tbase + ((uint32_t)(quad * 32) << 16);
  const int n0 = nb * BN;
  const int grow0 = mb * BM + quad * 32;
  const float sc = a.alpha != nullptr ? *a.alpha : 1.f;
  uint32_t r[32];
  if (n0 < a.N) tmem_ld32_async(trow, r);
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    if (n0 + c >= a.N) break;
    tmem_wait_ld();
    tmem_regs(r);
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * sc;
    // next chunk's TMEM read overlaps this chunk's staging
    if (c + 32 < BN && n0 + c + 32 < a.N) tmem_ld32_async(trow + c + 32, r);
    if (lane == 0) bulk_wait_group_read0();
    __syncwarp();
    uint8_t* rowp = stg + lane * 128;
#pragma unroll
    for (int cc = 0; cc < 8; ++cc)
      *reinterpret_cast<float4*>(rowp + ((cc ^ (lane & 7)) << 4)) =
          make_float4(v[4 * cc], v[4 * cc + 1], v[4 * cc + 2], v[4 * cc + 3]);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      if constexpr (ACC) tma_reduce_add_2d(tmD, stg, n0 + c, grow0);
      else tma_store_2d(tmD, stg, n0 + c, grow0);
      bulk_commit_group();
    }
  }
}

// D = alpha * acc + R (bf16): the residual's [32 x 64] box is brought into the
// staging slot by TMA (issued before the accumulator is read, so both latencies
// overlap), summed in place and stored from the same slot.  `rbar` is this
// warp's barrier, `rphase` its phase.
template <int BN>
__device__ __forceinline__ void epilogue_tma_residual(const GemmArgs& a, const CUtensorMap* tmD,
                                                      const CUtensorMap* tmR, uint8_t* stg, uint64_t* rbar,
                                                      uint32_t& rphase, uint32_t tbase, int mb, int nb, int quad,
                                                      int lane, volatile int* abort_flag) {
  const uint32_t trow = tbase + ((uint32_t)(quad * 32) << 16);
  const int n0 = nb * BN;
  const int grow0 = mb * BM + quad * 32;
  const float sc = a.alpha != nullptr ? *a.alpha : 1.f;
#pragma unroll 1
  for (int c = 0; c < BN; c += 64) {
    if (n0 + c >= a.N) break;
    if (lane == 0) {
      bulk_wait_group_read0();  // the slot's previous store has read it
      mbar_arrive_expect_tx(rbar, 4096);
      tma_load_2d(stg, tmR, rbar, n0 + c, grow0);
    }
    uint32_t r1[32], r2[32];
    tmem_ld32_async(trow + c, r1);
    tmem_ld32_async(trow + c + 32, r2);
    tmem_wait_ld();
    tmem_regs(r1);
    tmem_regs(r2);
    const bool ok = mbar_wait(rbar, rphase, a.err);
    rphase ^= 1;
    if (!ok) {
      *abort_flag = 1;  // the residual never arrived: leave the tile unwritten, the error word is set
      return;
    }
    uint8_t* rowp = stg + lane * 128;
#pragma unroll
    for (int cc = 0; cc < 8; ++cc) {
      uint4* q = reinterpret_cast<uint4*>(rowp + ((cc ^ (lane & 7)) << 4));
      const uint4 in = *q;
      const uint32_t* rr = cc < 4 ? r1 : r2;
      const int b = (cc & 3) * 8;
      const float2 f0 = unpack_bf16x2(in.x), f1 = unpack_bf16x2(in.y), f2 = unpack_bf16x2(in.z),
                   f3 = unpack_bf16x2(in.w);
      uint4 o;
      // (alpha * acc) + r rounded twice, as in the row-per-thread epilogue
#define DTB_AR(i, f) __fadd_rn(__fmul_rn(__uint_as_float(rr[b + (i)]), sc), f)
      o.x = pack_bf16x2(DTB_AR(0, f0.x), DTB_AR(1, f0.y));
      o.y = pack_bf16x2(DTB_AR(2, f1.x), DTB_AR(3, f1.y));
      o.z = pack_bf16x2(DTB_AR(4, f2.x), DTB_AR(5, f2.y));
      o.w = pack_bf16x2(DTB_AR(6, f3.x), DTB_AR(7, f3.y));
#undef DTB_AR
      *q = o;
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tmD, stg, n0 + c, grow0);
      bulk_commit_group();
    }
  }
}

// Writes 64 bf16 (packed pairs) as this lane's row of a 128-byte-swizzled
// [32 x 64] box in the warp's staging slot, then one lane stores the box at
// (x, y) through `m`.  The slot's previous store must have read it: checked here.
__device__ __forceinline__ void stage_and_store_row64(const CUtensorMap* m, uint8_t* stg, const uint32_t (&pk)[32],
                                                      int x, int y, int lane) {
  if (lane == 0) bulk_wait_group_read0();
  __syncwarp();
  uint8_t* rowp = stg + lane * 128;
#pragma unroll
  for (int cc = 0; cc < 8; ++cc)
    *reinterpret_cast<uint4*>(rowp + ((cc ^ (lane & 7)) << 4)) =
        make_uint4(pk[4 * cc], pk[4 * cc + 1], pk[4 * cc + 2], pk[4 * cc + 3]);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(m, stg, x, y);
    bulk_commit_group();
  }
}

// QKV projection with RoPE on the first rope_cols columns: each 64-column box of
// the output is produced in two 32-column halves; a rotated half needs both
// members of its pairs (columns p and p + hd/2 of the head), so the TMEM
// columns are read once per output half instead of once per pair.
template <int BN>
__device__ __forceinline__ void epilogue_tma_rope(const GemmArgs& a, const CUtensorMap* tmD, uint8_t* stg,
                                                  uint32_t tbase, int mb, int nb, int quad, int lane) {
  const uint32_t trow = tbase + ((uint32_t)(quad * 32) << 16);
  const int n0 = nb * BN;
  const int grow0 = mb * BM + quad * 32;
  const int hd = a.head_dim, half = hd >> 1;
  const int pos = (grow0 + lane) % a.seqlen;  // rows past M read valid table rows and are clipped on store
  const float4* crow = reinterpret_cast<const float4*>(a.cos_t + (long)pos * hd);
  const float4* srow = reinterpret_cast<const float4*>(a.sin_t + (long)pos * hd);
#pragma unroll 1
  for (int c = 0; c < BN; c += 64) {
    const int col = n0 + c;
    if (col >= a.N) break;
    uint32_t pk[32];
    if (col < a.rope_cols) {
      const int h0 = (c / hd) * hd;  // head start inside the tile (hd % 64 == 0)
#pragma unroll
      for (int j = 0; j < 64; j += 32) {
        const int e = c - h0 + j;  // element of the head
        const bool lo = e < half;
        const int p = lo ? e : e - half;
        float4 c4[8], s4[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          c4[q] = __ldg(crow + (p >> 2) + q);
          s4[q] = __ldg(srow + (p >> 2) + q);
        }
        uint32_t r1[32], r2[32];
        tmem_ld32_async(trow + h0 + p, r1);
        tmem_ld32_async(trow + h0 + half + p, r2);
        tmem_wait_ld();
        tmem_regs(r1);
        tmem_regs(r2);
        const float* cs = reinterpret_cast<const float*>(c4);
        const float* sn = reinterpret_cast<const float*>(s4);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float x1a = __uint_as_float(r1[2 * i]), x2a = __uint_as_float(r2[2 * i]);
          const float x1b = __uint_as_float(r1[2 * i + 1]), x2b = __uint_as_float(r2[2 * i + 1]);
          const float ya = lo ? rope_lo(x1a, x2a, cs[2 * i], sn[2 * i]) : rope_hi(x1a, x2a, cs[2 * i], sn[2 * i]);
          const float yb = lo ? rope_lo(x1b, x2b, cs[2 * i + 1], sn[2 * i + 1])
                              : rope_hi(x1b, x2b, cs[2 * i + 1], sn[2 * i + 1]);
          pk[(j >> 1) + i] = pack_bf16x2(ya, yb);
        }
      }
    } else {
      uint32_t r1[32], r2[32];
      tmem_ld32_async(trow + c, r1);
      tmem_ld32_async(trow + c + 32, r2);
      tmem_wait_ld();
      tmem_regs(r1);
      tmem_regs(r2);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        pk[i] = pack_bf16x2(__uint_as_float(r1[2 * i]), __uint_as_float(r1[2 * i + 1]));
        pk[16 + i] = pack_bf16x2(__uint_as_float(r2[2 * i]), __uint_as_float(r2[2 * i + 1]));
      }
    }
    stage_and_store_row64(tmD, stg, pk, col, grow0, lane);
  }
}

// Gate/up projection with SwiGLU: TMEM columns [0,128) hold g and [128,256) u
// for output columns nb*128 + [0,128).  Per 64 output columns three boxes leave
// through the one staging slot: round(g) and round(u) into D2 = [g | u] (at
// column c and ffn + c), then silu(g) * u into D, from the rounded values.
template <int BN>
__device__ __forceinline__ void epilogue_tma_swiglu(const GemmArgs& a, const CUtensorMap* tmD,
                                                    const CUtensorMap* tmD2, uint8_t* stg, uint32_t tbase, int mb,
                                                    int nb, int quad, int lane) {
  const uint32_t trow = tbase + ((uint32_t)(quad * 32) << 16);
  const int c0 = nb * 128;
  const int grow0 = mb * BM + quad * 32;
#pragma unroll 1
  for (int c = 0; c < 128; c += 64) {
    uint32_t pk[32];
#pragma unroll 1
    for (int which = 0; which < 2; ++which) {  // 0: g, 1: u
      uint32_t r1[32], r2[32];
      tmem_ld32_async(trow + which * 128 + c, r1);
      tmem_ld32_async(trow + which * 128 + c + 32, r2);
      tmem_wait_ld();
      tmem_regs(r1);
      tmem_regs(r2);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        pk[i] = pack_bf16x2(__uint_as_float(r1[2 * i]), __uint_as_float(r1[2 * i + 1]));
        pk[16 + i] = pack_bf16x2(__uint_as_float(r2[2 * i]), __uint_as_float(r2[2 * i + 1]));
      }
      stage_and_store_row64(tmD2, stg, pk, which * a.ffn + c0 + c, grow0, lane);
    }
#pragma unroll
    for (int j = 0; j < 64; j += 32) {
      uint32_t rg[32], ru[32];
      tmem_ld32_async(trow + c + j, rg);
      tmem_ld32_async(trow + 128 + c + j, ru);
      tmem_wait_ld();
      tmem_regs(rg);
      tmem_regs(ru);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float ga = __bfloat162float(__float2bfloat16_rn(__uint_as_float(rg[2 * i])));
        const float gb = __bfloat162float(__float2bfloat16_rn(__uint_as_float(rg[2 * i + 1])));
        const float ua = __bfloat162float(__float2bfloat16_rn(__uint_as_float(ru[2 * i])));
        const float ub = __bfloat162float(__float2bfloat16_rn(__uint_as_float(ru[2 * i + 1])));
        pk[(j >> 1) + i] = pack_bf16x2(swiglu_h(ga, ua), swiglu_h(gb, ub));
      }
    }
    stage_and_store_row64(tmD, stg, pk, c0 + c, grow0, lane);
  }
}

// ---------------------------------------------------------------- split-K (fp32 outputs)
// When the output has too few tiles to fill the SMs evenly (e.g. 256 CTA-pair
// tiles on 74 pairs is 3.46 waves), each tile's K range is cut into `ksplit`
// parts, work unit u = split * num_tiles + tile.  Split 0 stores (or
// accumulates, EPI_ACC_F32) its partial product as usual; split s > 0 waits
// until split s-1 of the same (tile, quadrant) has published, then adds its
// partial into D.  The additions happen in split order, so the result is the
// same on every run.  Flags are per (CTA-tile, quadrant) in a device buffer;
// split s publishes sk_epoch + s (the host advances sk_epoch by ksplit per
// launch, so old values never satisfy a wait).  Split s waits on a unit with a
// smaller index, which every CTA reaches first, so the waits always end.
__device__ __forceinline__ void splitk_publish(const GemmArgs& a, int ftile, int quad, int lane, int split) {
  __syncwarp();
  if (lane == 0) {
    __threadfence();
    st_release_sys(reinterpret_cast<uint32_t*>(a.sk_flags) + (long)ftile * 4 + quad, a.sk_epoch + split);
  }
}

__device__ __forceinline__ bool splitk_wait(const GemmArgs& a, int ftile, int quad, int split) {
  return wait_flag(reinterpret_cast<const uint32_t*>(a.sk_flags) + (long)ftile * 4 + quad, a.sk_epoch + split - 1,
                   a.timeout_ns, a.err);
}

// split s > 0: D += this split's partial (D read around L1: other SMs wrote it)
template <int BN>
__device__ __forceinline__ void splitk_accumulate(const GemmArgs& a, uint32_t tbase, int mb, int nb, int quad,
                                                  int lane) {
  const int row = mb * BM + quad * 32 + lane;
  const uint32_t trow = tbase + ((uint32_t)(quad * 32) << 16);
  const int n0 = nb * BN;
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    if (n0 + c >= a.N) break;
    float v[32];
    tmem_ld32(trow + c, v);
    if (row < a.M) {
      if (a.alpha != nullptr) {
        const float sc = *a.alpha;
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] *= sc;
      }
      float* p = reinterpret_cast<float*>(a.D) + (long)row * a.ldd + n0 + c;
      const int nv = min(32, a.N - (n0 + c));
      if (nv >= 32) {
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          const float4 q = __ldcg(reinterpret_cast<const float4*>(p + i));
          *reinterpret_cast<float4*>(p + i) = make_float4(q.x + v[i], q.y + v[i + 1], q.z + v[i + 2], q.w + v[i + 3]);
        }
      } else {
        for (int i = 0; i < nv; ++i) p[i] = __ldcg(p + i) + v[i];
      }
    }
  }
}

// ---------------------------------------------------------------- GEMM -> all-reduce
// Phase 1 (TMEM still held): this thread's row of the tile -> bf16 in the
// local staging area of the symmetric heap (same [M, N] layout as D).
template <int BN>
__device__ __forceinline__ void peer_ar_stage(const GemmArgs& a, uint32_t tbase, int mb, int nb, int quad, int lane) {
  const int row = mb * BM + quad * 32 + lane;
  const uint32_t trow = tbase + ((uint32_t)(quad * 32) << 16);
  const int n0 = nb * BN;
  __nv_bfloat16* stage = reinterpret_cast<__nv_bfloat16*>(a.peer_base[a.peer_rank] + a.stage_off);
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    if (n0 + c >= a.N) break;
    float v[32];
    tmem_ld32(trow + c, v);
    if (row < a.M) {
      if (a.alpha != nullptr) {
        const float s = *a.alpha;
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] *= s;
      }
      store_bf16_32(stage + (long)row * a.ldd + n0 + c, v);
    }
  }
}

// Phase 2: publish this (tile, quadrant) to every peer.  bar.warp.sync orders
// the other lanes' staging stores before the releasing lane's flag store, and
// release is cumulative, so one system-scope release per peer suffices.
__device__ __forceinline__ void peer_ar_publish(const GemmArgs& a, int tile, int quad, int lane) {
  const long nflags = (long)a.flag_tiles * 4;
  const long f = (long)tile * 4 + quad;
  __syncwarp();
  if (lane < a.peer_n)
    st_release_sys(reinterpret_cast<uint32_t*>(a.peer_base[lane] + a.flag_off) + (long)a.peer_rank * nflags + f,
                   a.epoch);
}

// The warp owns rows [row0, row0 + 32) of a tile; lane l covers columns
// [c, c + 8) (c = 8l), so each load instruction reads one contiguous 512-byte
// row segment.  Per step the loads of RU rows from every rank (NP >= peer_n)
// and of the residual are all issued before any is used (NP * RU + RU 16-byte
// loads in flight per lane), so a step costs one NVLink round trip; the sum
// then runs in rank order, which keeps every rank's result bitwise equal.
template <int NP, int RU, bool WRITEBACK = false>
__device__ __forceinline__ void peer_sum_rows(const GemmArgs& a, int row0, int n0, int c) {
#pragma unroll 1
  for (int r = 0; r < 32; r += RU) {
    uint4 v[NP][RU], q[RU];
#pragma unroll
    for (int p = 0; p < NP; ++p)
#pragma unroll
      for (int i = 0; i < RU; ++i) {
        const int rr = row0 + r + i;
        v[p][i] = (p < a.peer_n && rr < a.M)
                      ? ld_cg_v4(a.peer_base[p] + a.stage_off + ((long)rr * a.ldd + n0 + c) * 2)
                      : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
    for (int i = 0; i < RU; ++i) {
      const int rr = row0 + r + i;
      q[i] = (a.R != nullptr && rr < a.M) ? *reinterpret_cast<const uint4*>(a.R + (long)(rr - a.rs_row0) * a.ldr + n0 + c)
                                          : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < RU; ++i) {
      const int rr = row0 + r + i;
      if (rr >= a.M) continue;
      float acc[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] = 0.f;
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        if (p >= a.peer_n) break;
        const uint32_t* u = &v[p][i].x;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 t = unpack_bf16x2(u[k]);
          acc[2 * k] += t.x;
          acc[2 * k + 1] += t.y;
        }
      }
      if (a.R != nullptr) {
        const uint32_t* u = &q[i].x;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 t = unpack_bf16x2(u[k]);
          acc[2 * k] += t.x;
          acc[2 * k + 1] += t.y;
        }
      }
      uint4 o;
      o.x = pack_bf16x2(acc[0], acc[1]);
      o.y = pack_bf16x2(acc[2], acc[3]);
      o.z = pack_bf16x2(acc[4], acc[5]);
      o.w = pack_bf16x2(acc[6], acc[7]);
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.D) + (long)(rr - a.rs_row0) * a.ldd + n0 + c) = o;
      if (WRITEBACK)  // two-shot owner: the sum replaces this rank's staged partial, for the peers to copy
        *reinterpret_cast<uint4*>(a.peer_base[a.peer_rank] + a.stage_off + ((long)rr * a.ldd + n0 + c) * 2) = o;
    }
  }
}

// Phase 3 (one tile later, so the flag round trip overlaps the next tile):
// wait for every peer's copy of the tile, then sum the staged tiles in rank
// order (+ residual) into D.  All ranks add the same bf16 partials in the same
// order, so they agree bitwise.
template <int BN>
__device__ __forceinline__ bool peer_ar_finish(const GemmArgs& a, int tile, int mb, int nb, int quad, int lane) {
  // reduce-scatter: tiles outside this rank's rows are summed by their owners
  if (a.rs_rows > 0 && (mb * BM < a.rs_row0 || mb * BM >= a.rs_row0 + a.rs_rows)) return true;
  const int row = mb * BM + quad * 32 + lane;
  const int n0 = nb * BN;
  const long nflags = (long)a.flag_tiles * 4;
  const long f = (long)tile * 4 + quad;
  const uint32_t* mine = reinterpret_cast<const uint32_t*>(a.peer_base[a.peer_rank] + a.flag_off);
  bool ok = true;
  for (int p = 0; p < a.peer_n && ok; ++p) ok = wait_flag(mine + (long)p * nflags + f, a.epoch, a.timeout_ns, a.err);
  if (!ok) return false;
  (void)row;
  const int row0 = mb * BM + quad * 32;
  const int cols = min(BN, a.N - n0);
  const int c = lane * 8;
  if (c >= cols) return true;
  if (a.peer_n <= 2) peer_sum_rows<2, 8>(a, row0, n0, c);
  else if (a.peer_n <= 4) peer_sum_rows<4, 4>(a, row0, n0, c);
  else peer_sum_rows<8, 2>(a, row0, n0, c);
  return true;
}

// ---------------------------------------------------------------- two-shot all-reduce
// For larger TP groups the one-shot finish above pulls (tp - 1) copies of every
// tile into every rank.  Two-shot: the (tile, quadrant) flag unit `f` belongs
// to rank f % tp.  Its owner waits for every rank's staged partial, sums them in
// rank order (+ residual) into D and back into its own staging slot, then
// raises a "done" flag in every peer's heap; the other ranks copy the sum from
// the owner.  Per-rank NVLink ingress drops from (tp-1) to 2(tp-1)/tp payloads.
// Done flags follow the partial flags: done_off = flag_off + peer_n * nflags * 4.
__device__ __forceinline__ int two_shot_owner(const GemmArgs& a, int tile, int quad) {
  return (int)(((long)tile * 4 + quad) % a.peer_n);
}

template <int BN>
__device__ __forceinline__ bool peer_ar_reduce_own(const GemmArgs& a, int tile, int mb, int nb, int quad, int lane) {
  const long nflags = (long)a.flag_tiles * 4;
  const long f = (long)tile * 4 + quad;
  const uint32_t* mine = reinterpret_cast<const uint32_t*>(a.peer_base[a.peer_rank] + a.flag_off);
  bool ok = true;
  for (int p = 0; p < a.peer_n && ok; ++p) ok = wait_flag(mine + (long)p * nflags + f, a.epoch, a.timeout_ns, a.err);
  if (!ok) return false;
  const int row0 = mb * BM + quad * 32;
  const int n0 = nb * BN;
  const int cols = min(BN, a.N - n0);
  const int c = lane * 8;
  if (c < cols) {
    if (a.peer_n <= 4) peer_sum_rows<4, 4, true>(a, row0, n0, c);
    else peer_sum_rows<8, 2, true>(a, row0, n0, c);
  }
  const long done_off = a.flag_off + (long)a.peer_n * nflags * 4;
  __syncwarp();
  if (lane < a.peer_n && lane != a.peer_rank)
    st_release_sys(reinterpret_cast<uint32_t*>(a.peer_base[lane] + done_off) + f, a.epoch);
  return true;
}

template <int BN>
__device__ __forceinline__ bool peer_ar_fetch(const GemmArgs& a, int tile, int mb, int nb, int quad, int lane) {
  const long nflags = (long)a.flag_tiles * 4;
  const long f = (long)tile * 4 + quad;
  const int owner = two_shot_owner(a, tile, quad);
  const long done_off = a.flag_off + (long)a.peer_n * nflags * 4;
  if (!wait_flag(reinterpret_cast<const uint32_t*>(a.peer_base[a.peer_rank] + done_off) + f, a.epoch, a.timeout_ns,
                 a.err))
    return false;
  const int row0 = mb * BM + quad * 32;
  const int n0 = nb * BN;
  const int cols = min(BN, a.N - n0);
  const int c = lane * 8;
  if (c >= cols) return true;
  const uint8_t* src = a.peer_base[owner] + a.stage_off;
  constexpr int RU = 8;
#pragma unroll 1
  for (int r = 0; r < 32; r += RU) {
    uint4 v[RU];
#pragma unroll
    for (int i = 0; i < RU; ++i) {
      const int rr = row0 + r + i;
      v[i] = rr < a.M ? ld_cg_v4(src + ((long)rr * a.ldd + n0 + c) * 2) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < RU; ++i) {
      const int rr = row0 + r + i;
      if (rr < a.M) *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.D) + (long)rr * a.ldd + n0 + c) = v[i];
    }
  }
  return true;
}

// ---------------------------------------------------------------- all-gather -> GEMM
// Copier warps (AG launches only: warps 10 and 11) pull the gathered A rows in
// the order the tiles need them (this rank's rows first, then the following
// ranks'), one 8 KB-class row per warp step, 16-byte loads that bypass L1 (a
// peer's rows come over NVLink), all issued before any store.  After a row is
// stored each lane fences its generic stores against the async (TMA) proxy,
// and lane 0 adds 1 to the row's 128-row chunk counter with release
// semantics; the producer warp waits (acquire, bounded) until the chunks of a
// tile's A rows have all their rows, then loads them by TMA.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void red_release_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bool ag_copy_rows(const GemmArgs& a, int copier, int ncopiers, int lane) {
  const int M = a.M, K = a.K;
  const int R = a.ag_rows;
  const int nranks = a.peer_n;
  uint32_t staged_seen = 0;  // bit p: rank p's rows are staged
  const uint32_t* staged = reinterpret_cast<const uint32_t*>(a.peer_base[a.peer_rank] + a.ag_staged_off);
  for (int rr = copier; rr < M; rr += ncopiers) {
    // rotated row order: rank r's rows first
    const int row = (rr + a.peer_rank * R) % M;
    const int p = row / R;
    const __nv_bfloat16* src;
    if (p == a.peer_rank) {
      src = a.ag_local + (long)(row - p * R) * K;
    } else {
      if (!(staged_seen & (1u << p))) {
        if (!wait_flag(staged + p, a.ag_epoch, a.timeout_ns, a.err)) return false;
        staged_seen |= 1u << p;
      }
      src = reinterpret_cast<const __nv_bfloat16*>(a.peer_base[p] + a.stage_off) + (long)(row - p * R) * K;
    }
    __nv_bfloat16* dst = a.ag_out + (long)row * K;
    // K bf16 = K/8 16-byte pieces per row; 32 lanes, up to 8 pieces each in flight
    for (int c0 = lane * 8; c0 < K; c0 += 32 * 8 * 8) {
      uint4 v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c = c0 + i * 256;
        v[i] = c < K ? ld_cg_v4(src + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c = c0 + i * 256;
        if (c < K) *reinterpret_cast<uint4*>(dst + c) = v[i];
      }
    }
    fence_proxy_async_global();
    __syncwarp();
    if (lane == 0) red_release_add(a.ag_count + row / 128, 1u);
  }
  return true;
}

// Tile order.  Normal launches: groups of GROUP_M row blocks (L2 reuse of B).
// All-gather launches: one row block at a time across all column blocks,
// starting at this rank's own rows, so the tiles consume gathered rows in the
// order and at about the rate the copier warps deliver them (B, the weight, is
// small enough to stay in L2 across row blocks).
template <bool AG>
__device__ __forceinline__ void ag_or_grouped_coords(const GemmArgs& a, int tile, int& mb, int& nb) {
  if constexpr (AG) {
    mb = (tile / a.n_blocks + a.ag_mrot) % a.m_blocks;
    nb = tile % a.n_blocks;
  } else {
    tile_coords(tile, a.m_blocks, a.n_blocks, mb, nb);
  }
}

// producer side: every 128-row chunk of rows [row0, row0 + rows) complete
__device__ __forceinline__ bool ag_wait_rows(const GemmArgs& a, int row0, int rows) {
  for (int c = row0 / 128; c < (row0 + rows + 127) / 128 && c * 128 < a.M; ++c) {
    const uint32_t* p = a.ag_count + c;
    if ((int32_t)(ld_acquire_gpu(p) - a.ag_target) < 0) {
      const uint64_t t0 = globaltimer_ns();
      while ((int32_t)(ld_acquire_gpu(p) - a.ag_target) < 0) {
        if (globaltimer_ns() - t0 > a.timeout_ns) {
          atomicExch(a.err, ERR_PEER_TIMEOUT);
          return false;
        }
        __nanosleep(128);
      }
    }
  }
  fence_proxy_async_global();
  return true;
}

// ---------------------------------------------------------------- kernel
// PAIR = false: one CTA per 128 x BN tile.
// PAIR = true (BN = 256): a (2,1,1) cluster computes a 256 x 256 tile with
// cta_group::2 MMAs: CTA r loads rows [128r, 128r+128) of the A tile and
// columns [128r, 128r+128) of the B tile into its own shared memory, the
// leader (r = 0) issues M=256 MMAs that read both CTAs' operands, and CTA r's
// TMEM receives output rows [128r, 128r+128).  Each SM then streams half of
// B per tile, which halves its shared-memory operand traffic.  Both CTAs'
// loads count on the leader's "full" barrier; the leader's commits arrive on
// both CTAs' "empty" / "accumulator full" barriers; both CTAs' epilogue warps
// arrive on the leader's "accumulator empty" barrier.
template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI, bool PAIR, bool AG = false>
__global__ void __launch_bounds__(AG ? 384 : 320, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmR,
                        const GemmArgs args) {
  static_assert(!AG || (!A_MN && !B_MN), "all-gather mode gathers K-major A rows");
  static_assert(!PAIR || BN == 256, "CTA pairs use 256-column tiles");
  constexpr bool TSTORE = tma_store_epi(EPI);
  using L = SmemLayout<BN, STAGES, PAIR, TSTORE>;
  constexpr int TILE_M = PAIR ? 2 * BM : BM;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t cta = PAIR ? cluster_ctarank() : 0;   // rank within the pair
  const bool leader = cta == 0;
  const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;      // tile-walker id
  const int units = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], PAIR ? 8 : 4);  // one arrival per epilogue warp of each CTA
    }
    if constexpr (TSTORE)
      for (int i = 0; i < 8; ++i) mbar_init(reinterpret_cast<uint64_t*>(smem + L::RBAR_OFF) + i, 1);
    *abort_flag = 0;
    if constexpr (PAIR) fence_mbar_init_cluster();
    else fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_holder, 2 * BN);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_holder, 2 * BN);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // the peer's barriers exist before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  constexpr uint32_t IDESC = idesc_bf16(TILE_M, BN, A_MN, B_MN);

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_phase[STAGES];
      bool issued[STAGES];
      for (int s = 0; s < STAGES; ++s) issued[s] = false, issued_phase[s] = 0;
      bool ok = true;
      const int kper = (args.k_iters + args.ksplit - 1) / args.ksplit;
      for (int u = unit; u < args.num_tiles * args.ksplit && ok; u += units) {
        const int tile = u % args.num_tiles, split = u / args.num_tiles;
        int mb, nb;
        ag_or_grouped_coords<AG>(args, tile, mb, nb);
        const int arow = mb * TILE_M + (int)cta * BM;  // first A row this CTA loads
        const int k_end = min(args.k_iters, (split + 1) * kper);
        if constexpr (AG) {
          if (!ag_wait_rows(args, arow, BM)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
        }
        for (int k = split * kper; k < k_end; ++k) {
          if (*abort_flag || !mbar_wait(&empty[stage], phase ^ 1, args.err)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * L::STAGE_BYTES;
          uint8_t* sb = sa + L::A_BYTES;
          if constexpr (PAIR) {
            // both CTAs' bytes complete on the leader's barrier; only the leader expects them
            if (leader) mbar_arrive_expect_tx(&full[stage], 2 * L::STAGE_BYTES);
            const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
            if (!A_MN) {
              tma_load_2d_pair(sa, &tmA, fb, k * BK, arow);
            } else {
              tma_load_2d_pair(sa, &tmA, fb, arow, k * BK);
              tma_load_2d_pair(sa + 8192, &tmA, fb, arow + 64, k * BK);
            }
            if (!B_MN) {
              const int r = (EPI == EPI_SWIGLU) ? (cta == 0 ? nb * 128 : args.ffn + nb * 128) : nb * BN + (int)cta * 128;
              tma_load_2d_pair(sb, &tmB, fb, k * BK, r);
            } else {
#pragma unroll
              for (int j = 0; j < 2; ++j) tma_load_2d_pair(sb + j * 8192, &tmB, fb, nb * BN + (int)cta * 128 + j * 64, k * BK);
            }
          } else {
            mbar_arrive_expect_tx(&full[stage], L::STAGE_BYTES);
            if (!A_MN) {
              tma_load_2d(sa, &tmA, &full[stage], k * BK, arow);
            } else {
              tma_load_2d(sa, &tmA, &full[stage], arow, k * BK);
              tma_load_2d(sa + 8192, &tmA, &full[stage], arow + 64, k * BK);
            }
            if (!B_MN) {
#pragma unroll
              for (int j = 0; j < BN / 128; ++j) {
                int r = (EPI == EPI_SWIGLU) ? (j == 0 ? nb * 128 : args.ffn + nb * 128) : nb * BN + j * 128;
                tma_load_2d(sb + j * 16384, &tmB, &full[stage], k * BK, r);
              }
            } else {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j) tma_load_2d(sb + j * 8192, &tmB, &full[stage], nb * BN + j * 64, k * BK);
            }
          }
          issued[stage] = true;
          issued_phase[stage] = phase;
          if (++stage == STAGES) stage = 0, phase ^= 1;
        }
      }
      if (!ok && leader) {
        // drain copies still in flight before the CTA's shared memory goes away
        // (a pair's follower has no barrier of its own for them: its bounded
        // waits outlast its last copy by far)
        for (int s = 0; s < STAGES; ++s)
          if (issued[s]) mbar_wait(&full[s], issued_phase[s], args.err);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      int t = 0;
      bool ok = true;
      const int kper = (args.k_iters + args.ksplit - 1) / args.ksplit;
      for (int u = unit; u < args.num_tiles * args.ksplit && ok; u += units, ++t) {
        const int split = u / args.num_tiles;
        const int k_begin = split * kper, k_end = min(args.k_iters, (split + 1) * kper);
        const int acc = t & 1;
        const uint32_t acc_phase = (t >> 1) & 1;
        if (*abort_flag || !mbar_wait(&acc_empty[acc], acc_phase ^ 1, args.err)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        for (int k = k_begin; k < k_end; ++k) {
          if (*abort_flag || !mbar_wait(&full[stage], phase, args.err)) {
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + stage * L::STAGE_BYTES);
          const uint32_t b0 = a0 + L::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = A_MN ? sdesc_sw128(a0 + kk * 2048, 8192, 1024) : sdesc_sw128(a0 + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? sdesc_sw128(b0 + kk * 2048, 8192, 1024) : sdesc_sw128(b0 + kk * 32, 16, 1024);
            if constexpr (PAIR) umma_bf16_pair(d, ad, bd, IDESC, (k != k_begin) || kk != 0);
            else umma_bf16(d, ad, bd, IDESC, (k != k_begin) || kk != 0);
          }
          if constexpr (PAIR) umma_commit_pair(&empty[stage]);
          else umma_commit(&empty[stage]);
          if (++stage == STAGES) stage = 0, phase ^= 1;
        }
        if constexpr (PAIR) umma_commit_pair(&acc_full[acc]);
        else umma_commit(&acc_full[acc]);
      }
    }
  } else if (AG && warp >= 10) {
    if (!ag_copy_rows(args, (int)blockIdx.x * 2 + (warp - 10), (int)gridDim.x * 2, lane)) *abort_flag = 1;
  } else {
    // two epilogue warpgroups (warps 2-9): group g drains the tiles that land
    // in TMEM buffer g, so each group has two tiles of time for its stores
    // and twice as many memory requests are in flight per SM
    const int quad = warp & 3;
    const int wg = (warp - 2) >> 2;
    int t = 0;
    int pend_tile = -1, pend_mb = 0, pend_nb = 0;  // EPI_PEER_AR: tile published, not yet reduced
    int pend2_tile = -1, pend2_mb = 0, pend2_nb = 0;  // two-shot: reduced by its owner, not yet copied
    uint32_t rphase = 0;                               // TMA residual epilogue: this warp's barrier phase
    for (int u = unit; u < args.num_tiles * args.ksplit; u += units, ++t) {
      const int tile = u % args.num_tiles, split = u / args.num_tiles;
      const int acc = t & 1;
      if (acc != wg) continue;
      const uint32_t acc_phase = (t >> 1) & 1;
      int mb, nb;
      ag_or_grouped_coords<AG>(args, tile, mb, nb);
      const int slab = PAIR ? 2 * mb + (int)cta : mb;     // this CTA's 128-row block of the output
      const int ftile = PAIR ? 2 * tile + (int)cta : tile;
      if (*abort_flag || !mbar_wait(&acc_full[acc], acc_phase, args.err)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      if constexpr (EPI == EPI_PEER_AR) {
        peer_ar_stage<BN>(args, tmem_base + acc * BN, slab, nb, quad, lane);
      } else if (TSTORE && args.d_tma) {
        uint8_t* stg = smem + L::STG_OFF + (warp - 2) * 4096;
        const uint32_t tb = tmem_base + acc * BN;
        if constexpr (EPI == EPI_STORE_BF16) {
          epilogue_tma_store<BN>(args, &tmD, stg, tb, slab, nb, quad, lane);
        } else if constexpr (EPI == EPI_RESIDUAL) {
          epilogue_tma_residual<BN>(args, &tmD, &tmR, stg, reinterpret_cast<uint64_t*>(smem + L::RBAR_OFF) + (warp - 2),
                                    rphase, tb, slab, nb, quad, lane, abort_flag);
        } else if constexpr (EPI == EPI_STORE_F32 || EPI == EPI_ACC_F32) {
          epilogue_tma_f32<BN, EPI == EPI_ACC_F32>(args, &tmD, stg, tb, slab, nb, quad, lane);
        } else if constexpr (EPI == EPI_ROPE) {
          epilogue_tma_rope<BN>(args, &tmD, stg, tb, slab, nb, quad, lane);
        } else if constexpr (EPI == EPI_SWIGLU) {
          if constexpr (BN == 256) epilogue_tma_swiglu<BN>(args, &tmD, &tmR, stg, tb, slab, nb, quad, lane);
        }
      } else if constexpr (EPI == EPI_STORE_F32 || EPI == EPI_ACC_F32) {
        if (split == 0) {
          epilogue_tile<BN, EPI>(args, tmem_base + acc * BN, slab, nb, quad, lane);
        } else if (splitk_wait(args, ftile, quad, split)) {
          splitk_accumulate<BN>(args, tmem_base + acc * BN, slab, nb, quad, lane);
        } else {
          *abort_flag = 1;
        }
        if (args.ksplit > 1) splitk_publish(args, ftile, quad, lane, split);
      } else {
        epilogue_tile<BN, EPI>(args, tmem_base + acc * BN, slab, nb, quad, lane);
      }
      // the MMA warp may reuse this accumulator buffer
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR) mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[acc]), 0));
        else mbar_arrive(&acc_empty[acc]);
      }
      if constexpr (EPI == EPI_PEER_AR) {
        peer_ar_publish(args, ftile, quad, lane);
        if (args.two_shot) {
          // tile k-1: its owner sums it; tile k-2: the others copy the owner's sum
          bool ok = true;
          if (pend_tile >= 0 && two_shot_owner(args, pend_tile, quad) == args.peer_rank)
            ok = peer_ar_reduce_own<BN>(args, pend_tile, pend_mb, pend_nb, quad, lane);
          if (ok && pend2_tile >= 0 && two_shot_owner(args, pend2_tile, quad) != args.peer_rank)
            ok = peer_ar_fetch<BN>(args, pend2_tile, pend2_mb, pend2_nb, quad, lane);
          if (!ok) {
            *abort_flag = 1;
            pend_tile = pend2_tile = -1;
            break;
          }
          pend2_tile = pend_tile;
          pend2_mb = pend_mb;
          pend2_nb = pend_nb;
        } else if (pend_tile >= 0 && !peer_ar_finish<BN>(args, pend_tile, pend_mb, pend_nb, quad, lane)) {
          *abort_flag = 1;
          pend_tile = -1;
          break;
        }
        pend_tile = ftile;
        pend_mb = slab;
        pend_nb = nb;
      }
    }
    if constexpr (EPI == EPI_PEER_AR) {
      if (args.two_shot) {
        bool ok = true;
        if (pend_tile >= 0 && two_shot_owner(args, pend_tile, quad) == args.peer_rank)
          ok = peer_ar_reduce_own<BN>(args, pend_tile, pend_mb, pend_nb, quad, lane);
        if (ok && pend2_tile >= 0 && two_shot_owner(args, pend2_tile, quad) != args.peer_rank)
          ok = peer_ar_fetch<BN>(args, pend2_tile, pend2_mb, pend2_nb, quad, lane);
        if (ok && pend_tile >= 0 && two_shot_owner(args, pend_tile, quad) != args.peer_rank)
          ok = peer_ar_fetch<BN>(args, pend_tile, pend_mb, pend_nb, quad, lane);
        if (!ok) *abort_flag = 1;
      } else if (pend_tile >= 0 && !peer_ar_finish<BN>(args, pend_tile, pend_mb, pend_nb, quad, lane)) {
        *abort_flag = 1;
      }
    }
    if constexpr (TSTORE) {
      if (lane == 0) bulk_wait_group0();  // this warp's stores are done before its staging slot goes away
      __syncwarp();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // no remote arrive or MMA operand read targets a CTA that has left
  tc_fence_after();
  if (warp == 1) {
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, 2 * BN);
    else tmem_dealloc(tmem_base, 2 * BN);
  }
}

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    DTB_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    DTB_CHECK(q == cudaDriverEntryPointSuccess && p, "cuTensorMapEncodeTiled not available");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// cuTensorMapEncodeTiled is a driver-API call and needs a current context on
// the calling thread; autograd's worker threads may not have bound one yet
// (the runtime binds the primary context lazily), so do it once per thread.
static void bind_context_once() {
  static thread_local bool bound = false;
  if (!bound) {
    DTB_CUDA(cudaFree(nullptr));
    bound = true;
  }
}

// 2-D bf16 tensor map over a row-major [rows, inner] matrix, box [box_rows, 64].
static CUtensorMap make_map(const void* base, long inner, long rows, long row_stride_elems, int box_rows) {
  bind_context_once();
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_stride_elems * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  DTB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (%d): inner=%ld rows=%ld stride=%ld box_rows=%d base=%p", (int)r, inner, rows, row_stride_elems, box_rows, base);
  return m;
}

// Output / residual map for the TMA-store epilogues: [32 rows x 128 bytes] boxes
// (64 bf16 or 32 fp32 columns), 128-byte swizzle.  Returns false (the caller then
// keeps the row-per-thread epilogue) when the base or the row stride is not
// 16-byte aligned, which a tensor map cannot describe.
static bool make_out_map(CUtensorMap* m, const void* base, bool f32, long inner, long rows, long row_stride_elems) {
  const int es = f32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (row_stride_elems * es) % 16 != 0 || inner <= 0 || rows <= 0)
    return false;
  bind_context_once();
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(row_stride_elems * es)};
  cuuint32_t box[2] = {(cuuint32_t)(128 / es), 32};
  cuuint32_t estr[2] = {1, 1};
  return encode_fn()(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                     const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int num_sms() { return device_sm_count(); }

template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI, bool PAIR, bool AG = false>
static void launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td, const CUtensorMap& tr, GemmArgs& g,
                   cudaStream_t st) {
  using L = SmemLayout<BN, STAGES, PAIR, tma_store_epi(EPI)>;
  auto kern = gemm_tcgen05_kernel<BN, STAGES, A_MN, B_MN, EPI, PAIR, AG>;
  constexpr int NT = AG ? 384 : 320;
  static bool configured = false;
  if (!configured) {
    DTB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL));
    configured = true;
  }
  if (g.num_tiles == 0) return;
  const int work = g.num_tiles * std::max(1, g.ksplit);
  if constexpr (PAIR) {
    // persistent (2,1,1) clusters, one per pair of SMs
    const int pairs = std::min(work, num_sms() / 2);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * pairs, 1, 1);
    cfg.blockDim = dim3(NT, 1, 1);
    cfg.dynamicSmemBytes = L::TOTAL;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    DTB_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, td, tr, g));
  } else {
    const int grid = std::min(work, num_sms());
    kern<<<grid, NT, L::TOTAL, st>>>(ta, tb, td, tr, g);
  }
  DTB_LAUNCH_CHECK();
}

template <int BN, bool A_MN, bool B_MN, bool PAIR>
static void dispatch_epi(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td, const CUtensorMap& tr, GemmArgs& g,
                         cudaStream_t st) {
  // per-CTA stage: 16 KB of A + 32 KB (BN=256), 16 KB (BN=128 or a pair's half of 256) of B
  constexpr int ST = (BN == 256 && !PAIR) ? 4 : kStages32K;
  switch (epi) {
    case EPI_STORE_BF16: launch<BN, ST, A_MN, B_MN, EPI_STORE_BF16, PAIR>(ta, tb, td, tr, g, st); break;
    case EPI_STORE_F32: launch<BN, ST, A_MN, B_MN, EPI_STORE_F32, PAIR>(ta, tb, td, tr, g, st); break;
    case EPI_ACC_F32: launch<BN, ST, A_MN, B_MN, EPI_ACC_F32, PAIR>(ta, tb, td, tr, g, st); break;
    case EPI_RESIDUAL:
      if constexpr (!A_MN && !B_MN) { launch<BN, ST, A_MN, B_MN, EPI_RESIDUAL, PAIR>(ta, tb, td, tr, g, st); break; }
      TORCH_CHECK(false, "residual epilogue needs K-major operands");
    case EPI_ROPE:
      if constexpr (!A_MN && !B_MN) { launch<BN, ST, A_MN, B_MN, EPI_ROPE, PAIR>(ta, tb, td, tr, g, st); break; }
      TORCH_CHECK(false, "rope epilogue needs K-major operands");
    case EPI_SWIGLU:
      if constexpr (!A_MN && !B_MN && BN == 256) { launch<BN, ST, A_MN, B_MN, EPI_SWIGLU, PAIR>(ta, tb, td, tr, g, st); break; }
      TORCH_CHECK(false, "swiglu epilogue needs K-major operands and BN=256");
    case EPI_PEER_AR:
      if constexpr (!A_MN) { launch<BN, ST, A_MN, B_MN, EPI_PEER_AR, PAIR>(ta, tb, td, tr, g, st); break; }
      TORCH_CHECK(false, "peer all-reduce epilogue needs a K-major A operand");
    case EPI_CE_STATS:
      if constexpr (!A_MN && !B_MN) { launch<BN, ST, A_MN, B_MN, EPI_CE_STATS, PAIR>(ta, tb, td, tr, g, st); break; }
      TORCH_CHECK(false, "cross-entropy epilogues need K-major operands");
    case EPI_CE_GRAD:
      if constexpr (!A_MN && !B_MN) { launch<BN, ST, A_MN, B_MN, EPI_CE_GRAD, PAIR>(ta, tb, td, tr, g, st); break; }
      TORCH_CHECK(false, "cross-entropy epilogues need K-major operands");
    case EPI_ACC_BF16OUT:
      if constexpr (!A_MN && B_MN) { launch<BN, ST, A_MN, B_MN, EPI_ACC_BF16OUT, PAIR>(ta, tb, td, tr, g, st); break; }
      TORCH_CHECK(false, "fp32-accumulator epilogue is built for the input-gradient layout (A K-major, B MN-major)");
    default: DTB_CHECK(false, "unknown epilogue %d", epi);
  }
}

// all-gather -> GEMM launches (K-major operands; the epilogues the column-parallel
// layers use)
template <int BN, bool PAIR>
static void dispatch_epi_ag(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td, const CUtensorMap& tr,
                            GemmArgs& g, cudaStream_t st) {
  constexpr int ST = (BN == 256 && !PAIR) ? 4 : kStages32K;
  switch (epi) {
    case EPI_STORE_BF16: launch<BN, ST, false, false, EPI_STORE_BF16, PAIR, true>(ta, tb, td, tr, g, st); break;
    case EPI_ROPE: launch<BN, ST, false, false, EPI_ROPE, PAIR, true>(ta, tb, td, tr, g, st); break;
    case EPI_SWIGLU:
      if constexpr (BN == 256) { launch<BN, ST, false, false, EPI_SWIGLU, PAIR, true>(ta, tb, td, tr, g, st); break; }
      TORCH_CHECK(false, "swiglu epilogue needs BN=256");
    default: DTB_CHECK(false, "all-gather GEMM: epilogue %d not built", epi);
  }
}

// Split-K for fp32 outputs: the number of K parts per tile.  Off unless
// DTB_GEMM_KSPLIT=n asks for n parts.  Measured on B200 (weight-gradient GEMMs,
// 4096-12288 x 4096-11008, K = 4096): two parts ran at 0.68-0.72x and four at
// 0.35-0.42x the one-part speed even where one part leaves the last wave 46%
// full; each extra part's fp32 read-modify-write of D in the epilogue, with
// half the MMA work per unit to hide it behind, outweighs the filled wave.
static int choose_ksplit(int tiles, int units_per_wave, int k_iters) {
  (void)tiles;
  (void)units_per_wave;
  static int forced = -2;
  if (forced == -2) {
    const char* e = getenv("DTB_GEMM_KSPLIT");
    forced = (e != nullptr && atoi(e) > 0) ? atoi(e) : 1;
  }
  int ks = std::max(1, std::min(forced, k_iters));
  while (ks > 1 && (long)(ks - 1) * ((k_iters + ks - 1) / ks) >= k_iters) --ks;  // no empty part
  return ks;
}

// Per-device flag words of the split-K handshake (allocated once, never freed)
// and the launch epoch.
static int* splitk_flags(long needed, uint32_t* epoch_out, int ks) {
  constexpr long kFlags = 1L << 20;
  static int* flags[64] = {nullptr};
  static uint32_t epoch[64] = {0};
  int dev = 0;
  DTB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64 || needed > kFlags) return nullptr;
  if (flags[dev] == nullptr) {
    DTB_CUDA(cudaMalloc(&flags[dev], kFlags * sizeof(int)));
    DTB_CUDA(cudaMemset(flags[dev], 0, kFlags * sizeof(int)));
    epoch[dev] = 1;
  }
  *epoch_out = epoch[dev];
  epoch[dev] += (uint32_t)ks;
  return flags[dev];
}

// Per-device chunk counters of the all-gather GEMM (allocated once, never freed;
// cleared on the stream before each launch).
static uint32_t* ag_counters(long chunks) {
  constexpr long kMax = 1L << 16;
  static uint32_t* cnt[64] = {nullptr};
  int dev = 0;
  DTB_CUDA(cudaGetDevice(&dev));
  DTB_CHECK(dev >= 0 && dev < 64 && chunks <= kMax, "all-gather GEMM: %ld row chunks (max %ld)", chunks, kMax);
  if (cnt[dev] == nullptr) DTB_CUDA(cudaMalloc(&cnt[dev], kMax * sizeof(uint32_t)));
  return cnt[dev];
}

// CTA pairs for 256-column tiles unless DTB_GEMM_PAIR=0 (single-CTA tiles)
static bool pair_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("DTB_GEMM_PAIR");
    v = (e == nullptr || e[0] != '0') ? 1 : 0;
  }
  return v == 1;
}

// TMA-store epilogues: level 1 (default) for store / accumulate / residual, level 2
// also for RoPE and SwiGLU, 0 for none (DTB_GEMM_TMA_EPI=0/1/2).  The level-2 set is
// built and checked against the row-per-thread path by its test, which runs it in
// a child process; it becomes the default once that has passed on a B200.
// gemm_tma_epilogue() sets the level at run time (tests compare the paths).
static int g_tma_epi = -1;
static int tma_epi_level() {
  if (g_tma_epi < 0) {
    const char* e = getenv("DTB_GEMM_TMA_EPI");
    g_tma_epi = (e == nullptr) ? 1 : (e[0] == '0' ? 0 : (e[0] == '2' ? 2 : 1));
  }
  return g_tma_epi;
}

}  // namespace dtb

int64_t gemm_tma_epilogue(int64_t level) {
  const int prev = dtb::tma_epi_level();
  dtb::g_tma_epi = (int)std::max<int64_t>(0, std::min<int64_t>(2, level));
  return prev;
}

// Python entry: see ops/gemm.py for the operand conventions.
//   A: [M,K] (a_mn=false) or [K,M] (a_mn=true); B: [N,K] or [K,N]; D: [M,N]
//   (SwiGLU: B = [2F,K], D = [M,F], D2 = [M,2F]; p0 = F).
struct PeerCfg {
  std::vector<int64_t> bases;
  int rank;
  long stage_off, flag_off;
  uint32_t epoch;
  double timeout_s;
  int rs_row0 = 0, rs_rows = 0;  // reduce-scatter: this rank's output rows
  bool two_shot = false;
};

// All-gather fused in front of the GEMM (sequence parallelism, column-parallel layers).
struct AgCfg {
  std::vector<int64_t> bases;
  int rank;
  long stage_off, staged_off;
  uint32_t epoch;
  double timeout_s;
  const __nv_bfloat16* local;
  int rows;  // rows per rank
};

// Fused LM-head cross-entropy epilogues (EPI_CE_STATS / EPI_CE_GRAD).
struct CeCfg {
  const int64_t* labels;
  long vocab_off, vocab_total, ignore;
  float* stats;
  float* tgt;
  const float* lse;
  const float* inv_n;
};

static void gemm_impl(torch::Tensor A, torch::Tensor B, torch::Tensor D, bool a_mn, bool b_mn, int64_t epi,
                      c10::optional<torch::Tensor> R, c10::optional<torch::Tensor> alpha,
                      c10::optional<torch::Tensor> cos_t, c10::optional<torch::Tensor> sin_t,
                      c10::optional<torch::Tensor> D2, int64_t p0, int64_t p1, const PeerCfg* peer,
                      const CeCfg* ce = nullptr, const AgCfg* ag = nullptr) {
  using namespace dtb;
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && D.is_cuda(), "gemm: CUDA tensors expected");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm: bf16 operands expected");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.is_contiguous() && B.is_contiguous(), "gemm: 2-D contiguous operands");
  const c10::cuda::CUDAGuard guard(A.device());
  const long M = a_mn ? A.size(1) : A.size(0);
  const long K = a_mn ? A.size(0) : A.size(1);
  const long Kb = b_mn ? B.size(0) : B.size(1);
  long NB = b_mn ? B.size(1) : B.size(0);
  DTB_CHECK(K == Kb, "gemm: reduction sizes differ (%ld vs %ld)", K, Kb);
  TORCH_CHECK(A.size(1) % 8 == 0 && B.size(1) % 8 == 0, "gemm: row strides must be multiples of 16 bytes");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(A.data_ptr()) & 15) == 0 && (reinterpret_cast<uintptr_t>(B.data_ptr()) & 15) == 0,
              "gemm: operands must be 16-byte aligned");
  GemmArgs g{};
  g.M = (int)M;
  g.K = (int)K;
  g.D = D.data_ptr();
  g.ldd = D.stride(0);
  g.err = dtb_error_word();
  if (peer != nullptr) {
    DTB_CHECK(epi == EPI_PEER_AR && peer->bases.size() >= 1 && peer->bases.size() <= (size_t)MAX_PEERS,
              "peer GEMM: bad group");
    for (size_t i = 0; i < peer->bases.size(); ++i) g.peer_base[i] = reinterpret_cast<uint8_t*>(peer->bases[i]);
    g.peer_n = (int)peer->bases.size();
    g.peer_rank = peer->rank;
    g.stage_off = peer->stage_off;
    g.flag_off = peer->flag_off;
    g.epoch = peer->epoch;
    g.timeout_ns = (uint64_t)(peer->timeout_s * 1e9);
    g.rs_row0 = peer->rs_row0;
    g.rs_rows = peer->rs_rows;
    g.two_shot = peer->two_shot && peer->rs_rows == 0 && g.peer_n > 1 ? 1 : 0;
    if (g.rs_rows > 0)
      DTB_CHECK(g.rs_row0 % BM == 0 && g.rs_rows % BM == 0 && g.rs_row0 + g.rs_rows <= M && D.size(0) == g.rs_rows,
                "peer GEMM reduce-scatter: row block [%d, %d) must be 128-row aligned and match D", g.rs_row0,
                g.rs_row0 + g.rs_rows);
    DTB_CHECK(peer->stage_off % 16 == 0 && D.size(1) % 8 == 0, "peer GEMM: staging must be 16-byte aligned");
  } else {
    DTB_CHECK(epi != EPI_PEER_AR, "peer all-reduce epilogue needs a peer group");
  }
  const bool f32out = D.scalar_type() == at::kFloat;
  int e = (int)epi;
  if (e == EPI_STORE_BF16 && f32out) e = EPI_STORE_F32;
  if (e == EPI_ACC_F32) TORCH_CHECK(f32out, "gemm: accumulate epilogue needs an fp32 output");
  g.d_v8 = f32out && (reinterpret_cast<uintptr_t>(D.data_ptr()) & 31) == 0 && D.stride(0) % 8 == 0;
  if (e == EPI_STORE_BF16 || e == EPI_RESIDUAL || e == EPI_ROPE || e == EPI_SWIGLU || e == EPI_PEER_AR ||
      e == EPI_CE_GRAD || e == EPI_ACC_BF16OUT)
    TORCH_CHECK(D.scalar_type() == at::kBFloat16, "gemm: bf16 output expected");
  TORCH_CHECK((e == EPI_CE_STATS || e == EPI_CE_GRAD) == (ce != nullptr), "gemm: cross-entropy epilogue config");
  if (ce != nullptr) {
    g.labels = ce->labels;
    g.vocab_off = ce->vocab_off;
    g.vocab_total = ce->vocab_total;
    g.ignore = ce->ignore;
    g.ce_stats = ce->stats;
    g.ce_tgt = ce->tgt;
    g.ce_lse = ce->lse;
    g.ce_inv_n = ce->inv_n;
    if (e == EPI_CE_GRAD) TORCH_CHECK(alpha.has_value() && ce->lse && ce->inv_n, "gemm: ce grad needs alpha, lse, 1/n");
  }
  if (e == EPI_ACC_BF16OUT) {
    TORCH_CHECK(R.has_value() && R->scalar_type() == at::kFloat && R->stride(1) == 1 && R->size(0) == M &&
                    (reinterpret_cast<uintptr_t>(R->data_ptr()) & 15) == 0 && R->stride(0) % 4 == 0,
                "gemm: fp32 accumulator input [M, N], rows 16-byte aligned");
    g.acc_in = R->data_ptr<float>();
    g.ld_acc = R->stride(0);
  }
  TORCH_CHECK(D.stride(1) == 1 && (D.stride(0) % 8 == 0 || e == EPI_CE_STATS),
              "gemm: output rows must be contiguous and 16B aligned");
  if (alpha.has_value()) {
    TORCH_CHECK(alpha->scalar_type() == at::kFloat && alpha->is_cuda(), "gemm: alpha must be a CUDA fp32 scalar");
    g.alpha = alpha->data_ptr<float>();
  }
  int BN = NB > 128 ? 256 : 128;
  if (e == EPI_PEER_AR && R.has_value()) {
    DTB_CHECK(R->scalar_type() == at::kBFloat16 && R->stride(1) == 1, "gemm: bad residual");
    g.R = reinterpret_cast<const __nv_bfloat16*>(R->data_ptr());
    g.ldr = R->stride(0);
  }
  if (e == EPI_RESIDUAL) {
    TORCH_CHECK(R.has_value() && R->scalar_type() == at::kBFloat16 && R->stride(1) == 1, "gemm: bad residual");
    g.R = reinterpret_cast<const __nv_bfloat16*>(R->data_ptr());
    g.ldr = R->stride(0);
  }
  if (e == EPI_ROPE) {
    g.rope_cols = (int)p0;
    g.head_dim = (int)(p1 >> 16);
    g.seqlen = (int)(p1 & 0xFFFF);
    TORCH_CHECK(g.head_dim % 64 == 0 && BN % g.head_dim == 0, "gemm: rope epilogue needs head_dim in {64,128,256}");
    TORCH_CHECK(cos_t.has_value() && sin_t.has_value(), "gemm: rope tables missing");
    g.cos_t = cos_t->data_ptr<float>();
    g.sin_t = sin_t->data_ptr<float>();
    TORCH_CHECK(((reinterpret_cast<uintptr_t>(g.cos_t) | reinterpret_cast<uintptr_t>(g.sin_t)) & 15) == 0 &&
                    cos_t->is_contiguous() && sin_t->is_contiguous(),
                "gemm: rope tables must be contiguous and 16-byte aligned");
  }
  if (e == EPI_SWIGLU) {
    TORCH_CHECK(D2.has_value(), "gemm: swiglu needs D2");
    g.ffn = (int)p0;
    TORCH_CHECK(g.ffn % 128 == 0 && NB == 2 * g.ffn, "gemm: swiglu needs B=[2F,K] with F % 128 == 0");
    g.D2 = reinterpret_cast<__nv_bfloat16*>(D2->data_ptr());
    g.ldd2 = D2->stride(0);
    BN = 256;
    g.N = g.ffn;
    g.n_blocks = g.ffn / 128;
  } else {
    g.N = (int)NB;
    g.n_blocks = (int)((NB + BN - 1) / BN);
  }
  const bool pair = BN == 256 && M > BM && pair_enabled();
  const int tile_m = pair ? 2 * BM : BM;
  g.m_blocks = (int)((M + tile_m - 1) / tile_m);
  g.k_iters = (int)((K + BK - 1) / BK);
  g.num_tiles = g.m_blocks * g.n_blocks;
  g.flag_tiles = pair ? 2 * g.num_tiles : g.num_tiles;
  if (ag != nullptr) {
    DTB_CHECK(!a_mn && !b_mn && (e == EPI_STORE_BF16 || e == EPI_ROPE || e == EPI_SWIGLU) && peer == nullptr,
              "all-gather GEMM: K-major operands and a store / RoPE / SwiGLU epilogue");
    DTB_CHECK(ag->bases.size() >= 2 && ag->bases.size() <= (size_t)MAX_PEERS && ag->rows > 0 &&
                  (long)ag->rows * (long)ag->bases.size() == M && ag->rows % tile_m == 0 && K % 8 == 0 &&
                  ag->stage_off % 16 == 0,
              "all-gather GEMM: %d rows per rank x %zu ranks must equal M=%ld, in %d-row tiles", ag->rows,
              ag->bases.size(), M, tile_m);
    for (size_t i = 0; i < ag->bases.size(); ++i) g.peer_base[i] = reinterpret_cast<uint8_t*>(ag->bases[i]);
    g.peer_n = (int)ag->bases.size();
    g.peer_rank = ag->rank;
    g.stage_off = ag->stage_off;
    g.ag_staged_off = ag->staged_off;
    g.ag_epoch = ag->epoch;
    g.timeout_ns = (uint64_t)(ag->timeout_s * 1e9);
    g.ag_local = ag->local;
    g.ag_out = reinterpret_cast<__nv_bfloat16*>(A.data_ptr());
    g.ag_rows = ag->rows;
    g.ag_mrot = (int)((long)ag->rank * ag->rows / tile_m);
    g.ag_count = ag_counters((M + 127) / 128);
    g.ag_target = 128;
    DTB_CUDA(cudaMemsetAsync(g.ag_count, 0, ((M + 127) / 128) * sizeof(uint32_t), at::cuda::getCurrentCUDAStream()));
  }
  g.ksplit = 1;
  if ((e == EPI_STORE_F32 || e == EPI_ACC_F32) && peer == nullptr && ce == nullptr && g.num_tiles > 0) {
    const int ks = choose_ksplit(g.num_tiles, pair ? num_sms() / 2 : num_sms(), g.k_iters);
    if (ks > 1) {
      g.sk_flags = splitk_flags((long)g.flag_tiles * 4, &g.sk_epoch, ks);
      if (g.sk_flags != nullptr) {
        g.ksplit = ks;
        g.timeout_ns = 10ull * 1000000000ull;
      }
    }
  }
  if (e == EPI_CE_STATS) {
    TORCH_CHECK(D.scalar_type() == at::kFloat && D.size(0) == M && D.size(1) == 2L * g.n_blocks,
                "gemm: ce stats must be fp32 [M, 2 * n_blocks]");
  } else {
    TORCH_CHECK((g.rs_rows > 0 ? D.size(0) == g.rs_rows : D.size(0) == M) && D.size(1) == g.N,
                "gemm: output shape mismatch");
  }
  // tensor maps: A box = 128 rows (K-major) or 64 K-rows (MN-major); B likewise
  if (dtb_debug_enabled())
    fprintf(stderr, "[dtb] gemm M=%ld N=%d K=%ld a_mn=%d b_mn=%d epi=%d BN=%d A=%p B=%p D=%p alpha=%p\n", M, g.N, K,
            (int)a_mn, (int)b_mn, e, BN, A.data_ptr(), B.data_ptr(), D.data_ptr(), (const void*)g.alpha);
  const CUtensorMap ta = a_mn ? make_map(A.data_ptr(), M, K, A.stride(0), BK) : make_map(A.data_ptr(), K, M, A.stride(0), BM);
  const CUtensorMap tb = b_mn ? make_map(B.data_ptr(), NB, K, B.stride(0), BK) : make_map(B.data_ptr(), K, NB, B.stride(0), 128);
  // store / accumulate / residual / RoPE / SwiGLU epilogues: D (and R or D2) through TMA
  // boxes when each can be described by a tensor map; split-K keeps the row-per-thread epilogue
  CUtensorMap td = ta, tr = ta;
  g.d_tma = 0;
  if (tma_store_epi(e) && g.ksplit == 1 && tma_epi_level() >= ((e == EPI_ROPE || e == EPI_SWIGLU) ? 2 : 1)) {
    bool ok = make_out_map(&td, D.data_ptr(), f32out, g.N, D.size(0), D.stride(0));
    if (ok && e == EPI_RESIDUAL) ok = make_out_map(&tr, R->data_ptr(), false, g.N, R->size(0), R->stride(0));
    // SwiGLU: tr describes D2 = [g | u]
    if (ok && e == EPI_SWIGLU) ok = make_out_map(&tr, D2->data_ptr(), false, 2L * g.ffn, D2->size(0), D2->stride(0));
    g.d_tma = ok ? 1 : 0;
  }
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  if (ag != nullptr) {
    if (BN == 256 && pair) dispatch_epi_ag<256, true>(e, ta, tb, td, tr, g, st);
    else if (BN == 256) dispatch_epi_ag<256, false>(e, ta, tb, td, tr, g, st);
    else dispatch_epi_ag<128, false>(e, ta, tb, td, tr, g, st);
    return;
  }
  if (BN == 256 && pair) {
    if (!a_mn && !b_mn) dispatch_epi<256, false, false, true>(e, ta, tb, td, tr, g, st);
    else if (!a_mn && b_mn) dispatch_epi<256, false, true, true>(e, ta, tb, td, tr, g, st);
    else if (a_mn && b_mn) dispatch_epi<256, true, true, true>(e, ta, tb, td, tr, g, st);
    else TORCH_CHECK(false, "gemm: layout (MN, K) not built");
  } else if (BN == 256) {
    if (!a_mn && !b_mn) dispatch_epi<256, false, false, false>(e, ta, tb, td, tr, g, st);
    else if (!a_mn && b_mn) dispatch_epi<256, false, true, false>(e, ta, tb, td, tr, g, st);
    else if (a_mn && b_mn) dispatch_epi<256, true, true, false>(e, ta, tb, td, tr, g, st);
    else TORCH_CHECK(false, "gemm: layout (MN, K) not built");
  } else {
    if (!a_mn && !b_mn) dispatch_epi<128, false, false, false>(e, ta, tb, td, tr, g, st);
    else if (!a_mn && b_mn) dispatch_epi<128, false, true, false>(e, ta, tb, td, tr, g, st);
    else if (a_mn && b_mn) dispatch_epi<128, true, true, false>(e, ta, tb, td, tr, g, st);
    else TORCH_CHECK(false, "gemm: layout (MN, K) not built");
  }
}

void gemm_entry(torch::Tensor A, torch::Tensor B, torch::Tensor D, bool a_mn, bool b_mn, int64_t epi,
                c10::optional<torch::Tensor> R, c10::optional<torch::Tensor> alpha,
                c10::optional<torch::Tensor> cos_t, c10::optional<torch::Tensor> sin_t,
                c10::optional<torch::Tensor> D2, int64_t p0, int64_t p1) {
  gemm_impl(A, B, D, a_mn, b_mn, epi, R, alpha, cos_t, sin_t, D2, p0, p1, nullptr);
}

// D = sum over the peer group of (A x B) (+ R): the GEMM fused with an
// all-reduce through the symmetric heaps (staging at stage_off, flags at
// flag_off, both inside every rank's heap; epoch increases by one per call).
// two_shot: see peer_ar_reduce_own; the flag area then holds (peer_n + 1) x flag
// slots (the partial flags of every rank, then the done flags).
void gemm_peer_ar(torch::Tensor A, torch::Tensor B, torch::Tensor D, bool b_mn, c10::optional<torch::Tensor> R,
                  c10::optional<torch::Tensor> alpha, std::vector<int64_t> bases, int64_t rank, int64_t stage_off,
                  int64_t flag_off, int64_t epoch, double timeout_s, bool two_shot) {
  PeerCfg pc{bases, (int)rank, (long)stage_off, (long)flag_off, (uint32_t)epoch, timeout_s};
  pc.two_shot = two_shot;
  gemm_impl(A, B, D, false, b_mn, dtb::EPI_PEER_AR, R, alpha, c10::nullopt, c10::nullopt, c10::nullopt, 0, 0, &pc);
}

// D = rows [row0, row0 + rows) of sum over the peer group of (A x B) (+ R, already
// in the reduce-scattered layout): the GEMM fused with a reduce-scatter.  Every
// rank stages its whole product; each rank sums only its own row block.
void gemm_peer_rs(torch::Tensor A, torch::Tensor B, torch::Tensor D, bool b_mn, c10::optional<torch::Tensor> R,
                  std::vector<int64_t> bases, int64_t rank, int64_t stage_off, int64_t flag_off, int64_t epoch,
                  double timeout_s, int64_t row0, int64_t rows) {
  DTB_CHECK(rows > 0, "peer GEMM reduce-scatter: empty row block");
  PeerCfg pc{bases, (int)rank, (long)stage_off, (long)flag_off, (uint32_t)epoch, timeout_s, (int)row0, (int)rows};
  gemm_impl(A, B, D, false, b_mn, dtb::EPI_PEER_AR, R, c10::nullopt, c10::nullopt, c10::nullopt, c10::nullopt, 0, 0,
            &pc);
}

// Column blocks of the CE statistics for an N-column GEMM (same tile width rule as gemm_impl).
int64_t gemm_ce_blocks(int64_t N) {
  const int BN = N > 128 ? 256 : 128;
  return (N + BN - 1) / BN;
}

static void dtb_ce_check_stats_shape(const torch::Tensor& stats, long M, long N) {
  TORCH_CHECK(stats.scalar_type() == at::kFloat && stats.is_contiguous() && stats.dim() == 2 && stats.size(0) == M &&
                  stats.size(1) == 2 * gemm_ce_blocks(N),
              "ce: stats must be fp32 [M, 2 * gemm_ce_blocks(N)]");
}

// Fused LM-head cross-entropy, forward half: statistics of logits = h W^T
// without writing the logits.  stats: fp32 [M, 2 * n_blocks] ((max, sum exp)
// per row and 128/256-column block), tgt: fp32 [M] (logit of the row's label
// where the label falls in this GEMM's columns [vocab_off, vocab_off + N)).
void gemm_ce_stats(torch::Tensor h, torch::Tensor w, torch::Tensor labels, torch::Tensor stats, torch::Tensor tgt,
                   int64_t vocab_off, int64_t vocab_total, int64_t ignore) {
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.is_contiguous() && labels.numel() == h.size(0),
              "ce: int64 labels [M]");
  TORCH_CHECK(tgt.scalar_type() == at::kFloat && tgt.numel() == h.size(0), "ce: fp32 target logits [M]");
  dtb_ce_check_stats_shape(stats, h.size(0), w.size(0));
  CeCfg c{labels.data_ptr<int64_t>(), (long)vocab_off, (long)vocab_total, (long)ignore, stats.data_ptr<float>(),
          tgt.data_ptr<float>(), nullptr, nullptr};
  gemm_impl(h, w, stats, false, false, dtb::EPI_CE_STATS, c10::nullopt, c10::nullopt, c10::nullopt, c10::nullopt,
            c10::nullopt, 0, 0, nullptr, &c);
}

// Fused LM-head cross-entropy, backward half: out[M, N] (bf16) =
// (softmax(h W^T) - onehot(label)) * dloss * inv_n for the vocabulary columns
// [vocab_off, vocab_off + N) of w's rows, with lse the full-vocabulary
// log-sum-exp of each row from the forward.
void gemm_ce_grad(torch::Tensor h, torch::Tensor w, torch::Tensor labels, torch::Tensor lse, torch::Tensor dloss,
                  torch::Tensor inv_n, torch::Tensor out, int64_t vocab_off, int64_t vocab_total, int64_t ignore) {
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.is_contiguous() && labels.numel() == h.size(0),
              "ce: int64 labels [M]");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.numel() == h.size(0), "ce: fp32 lse [M]");
  TORCH_CHECK(inv_n.scalar_type() == at::kFloat && inv_n.is_cuda(), "ce: fp32 device scalar 1/n");
  CeCfg c{labels.data_ptr<int64_t>(), (long)vocab_off, (long)vocab_total, (long)ignore, nullptr, nullptr,
          lse.data_ptr<float>(), inv_n.data_ptr<float>()};
  gemm_impl(h, w, out, false, false, dtb::EPI_CE_GRAD, c10::nullopt, dloss, c10::nullopt, c10::nullopt,
            c10::nullopt, 0, 0, nullptr, &c);
}

// Column-parallel GEMM with the sequence-parallel all-gather fused in front of it:
// A_gathered [size * rows, K] is filled by the kernel (this rank's rows from
// A_local, every peer's from its heap at stage_off once the peer has raised its
// staged flag to `epoch`) and multiplied as it lands; D = A_gathered x B^T with
// the given epilogue (store, RoPE, SwiGLU: as gemm_entry).
void gemm_ag(torch::Tensor A_gathered, torch::Tensor A_local, torch::Tensor B, torch::Tensor D, int64_t epi,
             c10::optional<torch::Tensor> cos_t, c10::optional<torch::Tensor> sin_t, c10::optional<torch::Tensor> D2,
             int64_t p0, int64_t p1, std::vector<int64_t> bases, int64_t rank, int64_t stage_off, int64_t staged_off,
             int64_t epoch, double timeout_s) {
  TORCH_CHECK(A_local.scalar_type() == at::kBFloat16 && A_local.is_contiguous() && A_local.dim() == 2 &&
                  A_local.size(1) == A_gathered.size(1) &&
                  (reinterpret_cast<uintptr_t>(A_local.data_ptr()) & 15) == 0,
              "gemm_ag: bf16 contiguous local rows");
  AgCfg c{bases, (int)rank, (long)stage_off, (long)staged_off, (uint32_t)epoch, timeout_s,
          reinterpret_cast<const __nv_bfloat16*>(A_local.data_ptr()), (int)A_local.size(0)};
  gemm_impl(A_gathered, B, D, false, false, epi, c10::nullopt, c10::nullopt, cos_t, sin_t, D2, p0, p1, nullptr,
            nullptr, &c);
}
