// Causal grouped-query flash attention, forward and backward (sm_100a).
//
// These mma.sync kernels cover every shape the tcgen05 kernels
// (attention_tc.cu, attention_bwd_tc.cu: head_dim 64/128, seq_len % 128 == 0)
// do not: head_dim 16, 32, 64 or 128 and any seq_len.  Rows past the end of
// the sequence are zero-filled on load and never stored; padded query rows get
// lse = +inf in the backward so their probabilities are exactly 0.
//
// Inputs come straight from the packed projection qkv[b*s, (nq + 2 nkv) * hd]
// (q heads, then k heads, then v heads); query head h reads kv head
// h / (nq / nkv), so nothing is repeated or transposed in memory.
//
// Forward: CTA = 4 warps x 16 query rows (64-row query tile); K/V tiles of 64
// rows stream through a double-buffered cp.async ring in XOR-swizzled shared
// memory; S = Q K^T and O += P V run on bf16 m16n8k16 tensor-core MMAs with
// fp32 accumulation; the online softmax (exp2 with the log2(e)-folded scale)
// stays in registers; tiles above the diagonal are skipped.  Saves the
// per-row log-sum-exp for the backward.
//
// Backward, deterministic (no atomics):
//   attn_bwd_dkdv: CTA per (64-row kv tile, batch, kv head); loops over the
//     query heads of its group and the query tiles at or below the diagonal,
//     recomputing P^T = exp(K Q^T - lse) and accumulating dV += P^T dO,
//     dK += dS^T Q in registers;
//   attn_bwd_dq: CTA per (64-row query tile, batch, head); loops over kv
//     tiles, accumulating dQ += dS K.
//   D = rowsum(dO * O) comes from a small pre-pass.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace dtb {
namespace attn {

constexpr float LOG2E = 1.4426950408889634f;

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// 16-byte copy that writes zeros instead when `valid` is false (source not read)
__device__ __forceinline__ void cp_async16_zfill(void* dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// D(16x8, fp32) += A(16x16 bf16, row) * B(16x8 bf16, col)
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Tile [R][HD] bf16 in smem, 16-byte chunks XOR-swizzled by row to keep
// ldmatrix conflict-free.
template <int HD>
__device__ __forceinline__ uint32_t swz(int row, int col) {  // byte offset of element (row, col)
  constexpr int CHR = HD / 8 < 8 ? HD / 8 : 8;              // 16-byte chunks a row's XOR may span
  const int chunk = (col >> 3) ^ (row & (CHR - 1));
  return (uint32_t)(row * HD * 2 + chunk * 16 + (col & 7) * 2);
}

// rows [0, valid) come from g, rows [valid, R) are zero-filled
template <int R, int HD, int NT>
__device__ __forceinline__ void load_tile(uint8_t* s, const __nv_bfloat16* g, long ld, int valid = R) {
  constexpr int CH = HD / 8;
#pragma unroll
  for (int i = threadIdx.x; i < R * CH; i += NT) {
    const int r = i / CH, c = i % CH;
    const bool ok = r < valid;
    cp_async16_zfill(s + swz<HD>(r, c * 8), g + (ok ? (long)r * ld + c * 8 : 0), ok);
  }
}

// A fragment (16 rows x 16 cols at (r0, c0)) of a swizzled [*, HD] tile.
template <int HD>
__device__ __forceinline__ void frag_a(uint32_t base, int r0, int c0, uint32_t (&a)[4]) {
  const int l = threadIdx.x & 31;
  const int r = r0 + (l & 7) + ((l >> 3) & 1) * 8;
  const int c = c0 + (l >> 4) * 8;
  ldsm_x4(base + swz<HD>(r, c), a[0], a[1], a[2], a[3]);
}
// B fragments for two n8 tiles, B(k, n) = T[n][k] (T rows = n): rows n0..n0+15, cols k0..k0+15.
template <int HD>
__device__ __forceinline__ void frag_b_rows(uint32_t base, int n0, int k0, uint32_t& b00, uint32_t& b01, uint32_t& b10,
                                            uint32_t& b11) {
  const int l = threadIdx.x & 31;
  const int r = n0 + (l & 7) + (l >> 4) * 8;
  const int c = k0 + ((l >> 3) & 1) * 8;
  ldsm_x4(base + swz<HD>(r, c), b00, b01, b10, b11);
}
// B fragments for two n8 tiles, B(k, n) = T[k][n] (T rows = k): rows k0..k0+15, cols n0..n0+15.
template <int HD>
__device__ __forceinline__ void frag_b_cols(uint32_t base, int k0, int n0, uint32_t& b00, uint32_t& b01, uint32_t& b10,
                                            uint32_t& b11) {
  const int l = threadIdx.x & 31;
  const int r = k0 + (l & 7) + ((l >> 3) & 1) * 8;
  const int c = n0 + (l >> 4) * 8;
  ldsm_x4_t(base + swz<HD>(r, c), b00, b01, b10, b11);
}

// ---------------------------------------------------------------- forward
template <int HD>
__global__ void __launch_bounds__(128) attn_fwd_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                      __nv_bfloat16* __restrict__ out, float* __restrict__ lse, int S,
                                                      int nq, int nkv, float scale_log2) {
  constexpr int BM = 64, BN = 64;
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* sQ = sm;
  uint8_t* sK = sm + BM * HD * 2;             // [2][BN][HD]
  uint8_t* sV = sK + 2 * BN * HD * 2;         // [2][BN][HD]
  const int nqb = (S + BM - 1) / BM;
  const int qb = nqb - 1 - blockIdx.x;  // heavy tiles first
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (nq / nkv);
  const long ld = (long)(nq + 2 * nkv) * HD;
  const __nv_bfloat16* base = qkv + (long)b * S * ld;
  const __nv_bfloat16* gq = base + (long)qb * BM * ld + h * HD;
  const __nv_bfloat16* gk = base + (long)(nq + hk) * HD;
  const __nv_bfloat16* gv = base + (long)(nq + nkv + hk) * HD;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  load_tile<BM, HD, 128>(sQ, gq, ld, S - qb * BM);
  load_tile<BN, HD, 128>(sK, gk, ld, S);
  load_tile<BN, HD, 128>(sV, gv, ld, S);
  cp_commit();

  float o[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  uint32_t qf[HD / 16][4];
  const int nkb = qb + 1;
  const int row0 = qb * BM + warp * 16 + g, row1 = row0 + 8;

  for (int j = 0; j < nkb; ++j) {
    const int buf = j & 1;
    if (j + 1 < nkb) {
      load_tile<BN, HD, 128>(sK + (buf ^ 1) * BN * HD * 2, gk + (long)(j + 1) * BN * ld, ld, S - (j + 1) * BN);
      load_tile<BN, HD, 128>(sV + (buf ^ 1) * BN * HD * 2, gv + (long)(j + 1) * BN * ld, ld, S - (j + 1) * BN);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) frag_a<HD>(smem_u32(sQ), warp * 16, kk * 16, qf[kk]);
    }
    const uint32_t kb = smem_u32(sK + buf * BN * HD * 2), vb = smem_u32(sV + buf * BN * HD * 2);
    float s[BN / 8][4];
#pragma unroll
    for (int n = 0; n < BN / 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
      for (int n = 0; n < BN / 16; ++n) {
        uint32_t b00, b01, b10, b11;
        frag_b_rows<HD>(kb, n * 16, kk * 16, b00, b01, b10, b11);
        mma16816(s[2 * n], qf[kk], b00, b01);
        mma16816(s[2 * n + 1], qf[kk], b10, b11);
      }
    }
    // scale, mask, online softmax (rows row0 / row1; each quad holds a row)
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int n = 0; n < BN / 8; ++n) {
      const int c = j * BN + n * 8 + 2 * t;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = c + (e & 1);
        const int row = (e < 2) ? row0 : row1;
        float v = s[n][e] * scale_log2;
        if (j == qb && col > row) v = -INFINITY;
        s[n][e] = v;
      }
      mx0 = fmaxf(mx0, fmaxf(s[n][0], s[n][1]));
      mx1 = fmaxf(mx1, fmaxf(s[n][2], s[n][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float c0 = exp2f(m0 - mx0), c1 = exp2f(m1 - mx1);
    m0 = mx0;
    m1 = mx1;
    float rs0 = 0.f, rs1 = 0.f;
    uint32_t pf[BN / 16][4];
#pragma unroll
    for (int n = 0; n < BN / 8; ++n) {
      const float p0 = exp2f(s[n][0] - m0), p1 = exp2f(s[n][1] - m0);
      const float p2 = exp2f(s[n][2] - m1), p3 = exp2f(s[n][3] - m1);
      rs0 += p0 + p1;
      rs1 += p2 + p3;
      pf[n >> 1][(n & 1) * 2 + 0] = pack_bf16x2(p0, p1);
      pf[n >> 1][(n & 1) * 2 + 1] = pack_bf16x2(p2, p3);
    }
    l0 = l0 * c0 + rs0;
    l1 = l1 * c1 + rs1;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      o[i][0] *= c0; o[i][1] *= c0; o[i][2] *= c1; o[i][3] *= c1;
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
      const uint32_t a[4] = {pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3]};
#pragma unroll
      for (int n = 0; n < HD / 16; ++n) {
        uint32_t b00, b01, b10, b11;
        frag_b_cols<HD>(vb, kk * 16, n * 16, b00, b01, b10, b11);
        mma16816(o[2 * n], a, b00, b01);
        mma16816(o[2 * n + 1], a, b10, b11);
      }
    }
    __syncthreads();
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = 1.f / l0, inv1 = 1.f / l1;
  const long ldo = (long)nq * HD;
  __nv_bfloat16* o0 = out + ((long)b * S + row0) * ldo + h * HD;
  __nv_bfloat16* o1 = o0 + 8 * ldo;
#pragma unroll
  for (int n = 0; n < HD / 8; ++n) {
    if (row0 < S) *reinterpret_cast<uint32_t*>(o0 + n * 8 + 2 * t) = pack_bf16x2(o[n][0] * inv0, o[n][1] * inv0);
    if (row1 < S) *reinterpret_cast<uint32_t*>(o1 + n * 8 + 2 * t) = pack_bf16x2(o[n][2] * inv1, o[n][3] * inv1);
  }
  if (t == 0) {
    float* L = lse + ((long)b * nq + h) * S;
    if (row0 < S) L[row0] = (m0 + log2f(l0)) / LOG2E;
    if (row1 < S) L[row1] = (m1 + log2f(l1)) / LOG2E;
  }
}

// ---------------------------------------------------------------- backward
// D[b, h, i] = sum_d dO[i, d] * O[i, d]
template <int HD>
__global__ void attn_bwd_pre_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dO,
                                    float* __restrict__ Dv, int S, int nq, long rows) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const long total = rows * nq;
  if (warp >= total) return;
  const long row = warp / nq;
  const int h = warp % nq;
  const __nv_bfloat16* a = o + row * (long)nq * HD + h * HD;
  const __nv_bfloat16* c = dO + row * (long)nq * HD + h * HD;
  float s = 0.f;
  for (int d = lane * 2; d < HD; d += 64) {
    float2 x = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(a + d));
    float2 y = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(c + d));
    s += x.x * y.x + x.y * y.y;
  }
  s = warp_sum(s);
  if (lane == 0) {
    const long b = row / S, i = row % S;
    Dv[(b * nq + h) * S + i] = s;
  }
}

template <int HD>
__global__ void __launch_bounds__(128) attn_bwd_dkdv_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                           const __nv_bfloat16* __restrict__ dO,
                                                           const float* __restrict__ lse, const float* __restrict__ Dv,
                                                           __nv_bfloat16* __restrict__ dqkv, int S, int nq, int nkv,
                                                           float scale, float scale_log2) {
  constexpr int BN = 64, BQ = 32;
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* sK = sm;                       // [BN][HD]
  uint8_t* sV = sK + BN * HD * 2;         // [BN][HD]
  uint8_t* sQ = sV + BN * HD * 2;         // [2][BQ][HD]
  uint8_t* sO = sQ + 2 * BQ * HD * 2;     // [2][BQ][HD]   (dO)
  float* sL = reinterpret_cast<float*>(sO + 2 * BQ * HD * 2);  // [2][BQ] lse*log2e
  float* sD = sL + 2 * BQ;                                     // [2][BQ]
  const int nkb = (S + BN - 1) / BN;
  const int kb = nkb - 1 - blockIdx.x;  // tiles near the end see the fewest query tiles
  const int hk = blockIdx.y, b = blockIdx.z;
  const int grp = nq / nkv;
  const long ld = (long)(nq + 2 * nkv) * HD;
  const long ldo = (long)nq * HD;
  const __nv_bfloat16* base = qkv + (long)b * S * ld;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int kv0 = kb * BN;

  load_tile<BN, HD, 128>(sK, base + (long)kv0 * ld + (nq + hk) * HD, ld, S - kv0);
  load_tile<BN, HD, 128>(sV, base + (long)kv0 * ld + (nq + nkv + hk) * HD, ld, S - kv0);
  cp_commit();

  float dk[HD / 8][4], dv[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;

  const int q_first = kv0 / BQ;
  const int nqt = (S + BQ - 1) / BQ - q_first;  // query tiles per head
  const int total = nqt * grp;
  auto issue = [&](int it, int buf) {
    const int hh = hk * grp + it / nqt;
    const int q0 = (q_first + it % nqt) * BQ;
    load_tile<BQ, HD, 128>(sQ + buf * BQ * HD * 2, base + (long)q0 * ld + hh * HD, ld, S - q0);
    load_tile<BQ, HD, 128>(sO + buf * BQ * HD * 2, dO + ((long)b * S + q0) * ldo + hh * HD, ldo, S - q0);
    if (threadIdx.x < BQ) {
      // padded query rows: lse = +inf makes their probabilities exactly 0
      const bool in = q0 + (int)threadIdx.x < S;
      const long li = ((long)b * nq + hh) * S + q0 + threadIdx.x;
      sL[buf * BQ + threadIdx.x] = in ? lse[li] * LOG2E : INFINITY;
      sD[buf * BQ + threadIdx.x] = in ? Dv[li] : 0.f;
    }
  };
  issue(0, 0);
  cp_commit();
  const int krow0 = kv0 + warp * 16 + g;  // this thread's kv rows: krow0, krow0 + 8
  for (int it = 0; it < total; ++it) {
    const int buf = it & 1;
    __syncthreads();  // buffer buf^1 free (previous iteration done with it)
    if (it + 1 < total) issue(it + 1, buf ^ 1);
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    const int q0 = (q_first + it % nqt) * BQ;
    const uint32_t qb = smem_u32(sQ + buf * BQ * HD * 2), ob = smem_u32(sO + buf * BQ * HD * 2);
    const float* L = sL + buf * BQ;
    const float* Dd = sD + buf * BQ;
    // S^T = K Q^T  [16 kv x BQ q] per warp
    float s[BQ / 8][4], dp[BQ / 8][4];
#pragma unroll
    for (int n = 0; n < BQ / 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[n][e] = dp[n][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      uint32_t ka[4], va[4];
      frag_a<HD>(smem_u32(sK), warp * 16, kk * 16, ka);
      frag_a<HD>(smem_u32(sV), warp * 16, kk * 16, va);
#pragma unroll
      for (int n = 0; n < BQ / 16; ++n) {
        uint32_t b00, b01, b10, b11;
        frag_b_rows<HD>(qb, n * 16, kk * 16, b00, b01, b10, b11);
        mma16816(s[2 * n], ka, b00, b01);
        mma16816(s[2 * n + 1], ka, b10, b11);
        frag_b_rows<HD>(ob, n * 16, kk * 16, b00, b01, b10, b11);
        mma16816(dp[2 * n], va, b00, b01);
        mma16816(dp[2 * n + 1], va, b10, b11);
      }
    }
    // P^T = exp2(S^T*scale_log2 - lse2[q]); dS^T = P^T (dP^T - D[q])
    uint32_t pa[BQ / 16][4], da[BQ / 16][4];
#pragma unroll
    for (int n = 0; n < BQ / 8; ++n) {
      float p[4], d[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qc = n * 8 + 2 * t + (e & 1);
        const int kr = (e < 2) ? krow0 : krow0 + 8;
        float v = exp2f(s[n][e] * scale_log2 - L[qc]);
        if (q0 + qc < kr) v = 0.f;
        p[e] = v;
        d[e] = v * (dp[n][e] - Dd[qc]);
      }
      pa[n >> 1][(n & 1) * 2 + 0] = pack_bf16x2(p[0], p[1]);
      pa[n >> 1][(n & 1) * 2 + 1] = pack_bf16x2(p[2], p[3]);
      da[n >> 1][(n & 1) * 2 + 0] = pack_bf16x2(d[0], d[1]);
      da[n >> 1][(n & 1) * 2 + 1] = pack_bf16x2(d[2], d[3]);
    }
    // dV += P^T dO ; dK += dS^T Q     (k = q index)
#pragma unroll
    for (int kk = 0; kk < BQ / 16; ++kk) {
#pragma unroll
      for (int n = 0; n < HD / 16; ++n) {
        uint32_t b00, b01, b10, b11;
        frag_b_cols<HD>(ob, kk * 16, n * 16, b00, b01, b10, b11);
        mma16816(dv[2 * n], pa[kk], b00, b01);
        mma16816(dv[2 * n + 1], pa[kk], b10, b11);
        frag_b_cols<HD>(qb, kk * 16, n * 16, b00, b01, b10, b11);
        mma16816(dk[2 * n], da[kk], b00, b01);
        mma16816(dk[2 * n + 1], da[kk], b10, b11);
      }
    }
  }
  const long ldd = ld;
  __nv_bfloat16* gk0 = dqkv + ((long)b * S + krow0) * ldd + (nq + hk) * HD;
  __nv_bfloat16* gv0 = dqkv + ((long)b * S + krow0) * ldd + (nq + nkv + hk) * HD;
#pragma unroll
  for (int n = 0; n < HD / 8; ++n) {
    const int c = n * 8 + 2 * t;
    if (krow0 < S) {
      *reinterpret_cast<uint32_t*>(gk0 + c) = pack_bf16x2(dk[n][0] * scale, dk[n][1] * scale);
      *reinterpret_cast<uint32_t*>(gv0 + c) = pack_bf16x2(dv[n][0], dv[n][1]);
    }
    if (krow0 + 8 < S) {
      *reinterpret_cast<uint32_t*>(gk0 + 8 * ldd + c) = pack_bf16x2(dk[n][2] * scale, dk[n][3] * scale);
      *reinterpret_cast<uint32_t*>(gv0 + 8 * ldd + c) = pack_bf16x2(dv[n][2], dv[n][3]);
    }
  }
}

template <int HD>
__global__ void __launch_bounds__(128) attn_bwd_dq_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                         const __nv_bfloat16* __restrict__ dO,
                                                         const float* __restrict__ lse, const float* __restrict__ Dv,
                                                         __nv_bfloat16* __restrict__ dqkv, int S, int nq, int nkv,
                                                         float scale, float scale_log2) {
  constexpr int BM = 64, BN = 32;
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* sQ = sm;                     // [BM][HD]
  uint8_t* sO = sQ + BM * HD * 2;       // [BM][HD]
  uint8_t* sK = sO + BM * HD * 2;       // [2][BN][HD]
  uint8_t* sV = sK + 2 * BN * HD * 2;   // [2][BN][HD]
  const int nqb = (S + BM - 1) / BM;
  const int qbk = nqb - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (nq / nkv);
  const long ld = (long)(nq + 2 * nkv) * HD;
  const long ldo = (long)nq * HD;
  const __nv_bfloat16* base = qkv + (long)b * S * ld;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int q0 = qbk * BM;
  const __nv_bfloat16* gk = base + (long)(nq + hk) * HD;
  const __nv_bfloat16* gv = base + (long)(nq + nkv + hk) * HD;
  load_tile<BM, HD, 128>(sQ, base + (long)q0 * ld + h * HD, ld, S - q0);
  load_tile<BM, HD, 128>(sO, dO + ((long)b * S + q0) * ldo + h * HD, ldo, S - q0);
  load_tile<BN, HD, 128>(sK, gk, ld, S);
  load_tile<BN, HD, 128>(sV, gv, ld, S);
  cp_commit();
  const int row0 = q0 + warp * 16 + g, row1 = row0 + 8;
  const long li = ((long)b * nq + h) * S;
  const float L0 = row0 < S ? lse[li + row0] * LOG2E : INFINITY;
  const float L1 = row1 < S ? lse[li + row1] * LOG2E : INFINITY;
  const float D0 = row0 < S ? Dv[li + row0] : 0.f, D1 = row1 < S ? Dv[li + row1] : 0.f;
  float dq[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
  uint32_t qf[HD / 16][4], of[HD / 16][4];
  const int nkt = min((q0 + BM) / BN, (S + BN - 1) / BN);
  for (int j = 0; j < nkt; ++j) {
    const int buf = j & 1;
    if (j + 1 < nkt) {
      load_tile<BN, HD, 128>(sK + (buf ^ 1) * BN * HD * 2, gk + (long)(j + 1) * BN * ld, ld, S - (j + 1) * BN);
      load_tile<BN, HD, 128>(sV + (buf ^ 1) * BN * HD * 2, gv + (long)(j + 1) * BN * ld, ld, S - (j + 1) * BN);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        frag_a<HD>(smem_u32(sQ), warp * 16, kk * 16, qf[kk]);
        frag_a<HD>(smem_u32(sO), warp * 16, kk * 16, of[kk]);
      }
    }
    const uint32_t kb = smem_u32(sK + buf * BN * HD * 2), vb = smem_u32(sV + buf * BN * HD * 2);
    float s[BN / 8][4], dp[BN / 8][4];
#pragma unroll
    for (int n = 0; n < BN / 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[n][e] = dp[n][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
      for (int n = 0; n < BN / 16; ++n) {
        uint32_t b00, b01, b10, b11;
        frag_b_rows<HD>(kb, n * 16, kk * 16, b00, b01, b10, b11);
        mma16816(s[2 * n], qf[kk], b00, b01);
        mma16816(s[2 * n + 1], qf[kk], b10, b11);
        frag_b_rows<HD>(vb, n * 16, kk * 16, b00, b01, b10, b11);
        mma16816(dp[2 * n], of[kk], b00, b01);
        mma16816(dp[2 * n + 1], of[kk], b10, b11);
      }
    }
    uint32_t da[BN / 16][4];
#pragma unroll
    for (int n = 0; n < BN / 8; ++n) {
      float d[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int col = j * BN + n * 8 + 2 * t + (e & 1);
        const int row = (e < 2) ? row0 : row1;
        float p = exp2f(s[n][e] * scale_log2 - ((e < 2) ? L0 : L1));
        if (col > row) p = 0.f;
        d[e] = p * (dp[n][e] - ((e < 2) ? D0 : D1));
      }
      da[n >> 1][(n & 1) * 2 + 0] = pack_bf16x2(d[0], d[1]);
      da[n >> 1][(n & 1) * 2 + 1] = pack_bf16x2(d[2], d[3]);
    }
    // dQ += dS K   (k = kv index; B(k, n) = K[kv][d])
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
#pragma unroll
      for (int n = 0; n < HD / 16; ++n) {
        uint32_t b00, b01, b10, b11;
        frag_b_cols<HD>(kb, kk * 16, n * 16, b00, b01, b10, b11);
        mma16816(dq[2 * n], da[kk], b00, b01);
        mma16816(dq[2 * n + 1], da[kk], b10, b11);
      }
    }
    __syncthreads();
  }
  __nv_bfloat16* g0 = dqkv + ((long)b * S + row0) * ld + h * HD;
#pragma unroll
  for (int n = 0; n < HD / 8; ++n) {
    const int c = n * 8 + 2 * t;
    if (row0 < S) *reinterpret_cast<uint32_t*>(g0 + c) = pack_bf16x2(dq[n][0] * scale, dq[n][1] * scale);
    if (row1 < S) *reinterpret_cast<uint32_t*>(g0 + 8 * ld + c) = pack_bf16x2(dq[n][2] * scale, dq[n][3] * scale);
  }
}

template <int HD>
void fwd_launch(const __nv_bfloat16* qkv, __nv_bfloat16* o, float* lse, int B, int S, int nq, int nkv, float scale,
                cudaStream_t st) {
  const int smem = (64 + 4 * 64) * HD * 2;
  static bool cfg = false;
  if (!cfg) {
    DTB_CUDA(cudaFuncSetAttribute(attn_fwd_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    cfg = true;
  }
  dim3 grid((S + 63) / 64, nq, B);
  attn_fwd_kernel<HD><<<grid, 128, smem, st>>>(qkv, o, lse, S, nq, nkv, scale * LOG2E);
}

template <int HD>
void bwd_pre_launch(const __nv_bfloat16* o, const __nv_bfloat16* dO, float* Dv, int B, int S, int nq, cudaStream_t st) {
  const long rows = (long)B * S;
  const long warps = rows * nq;
  attn_bwd_pre_kernel<HD><<<(int)((warps * 32 + 255) / 256), 256, 0, st>>>(o, dO, Dv, S, nq, rows);
}

template <int HD>
void bwd_launch(const __nv_bfloat16* qkv, const __nv_bfloat16* o, const __nv_bfloat16* dO, const float* lse, float* Dv,
                __nv_bfloat16* dqkv, int B, int S, int nq, int nkv, float scale, cudaStream_t st) {
  const int smem_kv = (2 * 64 + 4 * 32) * HD * 2 + 4 * 32 * 4;
  const int smem_q = (2 * 64 + 4 * 32) * HD * 2;
  static bool cfg = false;
  if (!cfg) {
    DTB_CUDA(cudaFuncSetAttribute(attn_bwd_dkdv_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_kv));
    DTB_CUDA(cudaFuncSetAttribute(attn_bwd_dq_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_q));
    cfg = true;
  }
  attn_bwd_dkdv_kernel<HD><<<dim3((S + 63) / 64, nkv, B), 128, smem_kv, st>>>(qkv, dO, lse, Dv, dqkv, S, nq, nkv,
                                                                               scale, scale * LOG2E);
  attn_bwd_dq_kernel<HD><<<dim3((S + 63) / 64, nq, B), 128, smem_q, st>>>(qkv, dO, lse, Dv, dqkv, S, nq, nkv, scale,
                                                                           scale * LOG2E);
}

}  // namespace attn
}  // namespace dtb

using namespace dtb;

static void attn_check(const torch::Tensor& qkv, int64_t B, int64_t S, int64_t nq, int64_t nkv, int64_t hd) {
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && qkv.is_contiguous(), "attention: bf16 packed qkv");
  TORCH_CHECK(hd == 16 || hd == 32 || hd == 64 || hd == 128, "attention kernels support head_dim 16, 32, 64 and 128");
  TORCH_CHECK(S >= 1 && B >= 1, "attention: empty batch or sequence");
  TORCH_CHECK(nq % nkv == 0, "nq must be a multiple of nkv");
  TORCH_CHECK(qkv.size(0) == B * S && qkv.size(1) == (nq + 2 * nkv) * hd, "attention: qkv shape");
}

bool attn_fwd_tc(const torch::Tensor& qkv, torch::Tensor& o, torch::Tensor& lse, int64_t B, int64_t S, int64_t nq,
                 int64_t nkv, int64_t hd, double scale);

std::vector<torch::Tensor> attn_fwd(torch::Tensor qkv, int64_t B, int64_t S, int64_t nq, int64_t nkv, int64_t hd,
                                    double scale, bool legacy) {
  attn_check(qkv, B, S, nq, nkv, hd);
  const c10::cuda::CUDAGuard g(qkv.device());
  auto o = torch::empty({B * S, nq * hd}, qkv.options());
  auto lse = torch::empty({B, nq, S}, qkv.options().dtype(at::kFloat));
  // tcgen05/TMEM kernel (attention_tc.cu) unless the sequence is not a multiple of 128
  if (!legacy && attn_fwd_tc(qkv, o, lse, B, S, nq, nkv, hd, scale)) return {o, lse};
  auto st = at::cuda::getCurrentCUDAStream();
  auto q = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  auto op = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  if (hd == 128) attn::fwd_launch<128>(q, op, lse.data_ptr<float>(), B, S, nq, nkv, (float)scale, st);
  else if (hd == 64) attn::fwd_launch<64>(q, op, lse.data_ptr<float>(), B, S, nq, nkv, (float)scale, st);
  else if (hd == 32) attn::fwd_launch<32>(q, op, lse.data_ptr<float>(), B, S, nq, nkv, (float)scale, st);
  else attn::fwd_launch<16>(q, op, lse.data_ptr<float>(), B, S, nq, nkv, (float)scale, st);
  DTB_LAUNCH_CHECK();
  return {o, lse};
}

bool attn_bwd_tc(const torch::Tensor& dO, const torch::Tensor& qkv, const float* lse, const float* Dv,
                 torch::Tensor& dqkv, int64_t B, int64_t S, int64_t nq, int64_t nkv, int64_t hd, double scale);

torch::Tensor attn_bwd(torch::Tensor dO, torch::Tensor qkv, torch::Tensor o, torch::Tensor lse, int64_t B, int64_t S,
                       int64_t nq, int64_t nkv, int64_t hd, double scale, bool legacy) {
  attn_check(qkv, B, S, nq, nkv, hd);
  TORCH_CHECK(dO.is_contiguous() && dO.sizes() == o.sizes(), "attention bwd: dO shape");
  const c10::cuda::CUDAGuard g(qkv.device());
  auto dqkv = torch::empty_like(qkv);
  auto Dv = torch::empty({B, nq, S}, qkv.options().dtype(at::kFloat));
  auto st = at::cuda::getCurrentCUDAStream();
  auto cast = [](const torch::Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); };
  auto dq = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  if (hd == 128) attn::bwd_pre_launch<128>(cast(o), cast(dO), Dv.data_ptr<float>(), B, S, nq, st);
  else if (hd == 64) attn::bwd_pre_launch<64>(cast(o), cast(dO), Dv.data_ptr<float>(), B, S, nq, st);
  else if (hd == 32) attn::bwd_pre_launch<32>(cast(o), cast(dO), Dv.data_ptr<float>(), B, S, nq, st);
  else attn::bwd_pre_launch<16>(cast(o), cast(dO), Dv.data_ptr<float>(), B, S, nq, st);
  DTB_LAUNCH_CHECK();
  // tcgen05/TMEM kernels (attention_bwd_tc.cu) unless the sequence is not a multiple of 128
  if (!legacy && attn_bwd_tc(dO, qkv, lse.data_ptr<float>(), Dv.data_ptr<float>(), dqkv, B, S, nq, nkv, hd, scale))
    return dqkv;
#define DTB_ATTN_BWD(HDV)                                                                                            \
  attn::bwd_launch<HDV>(cast(qkv), cast(o), cast(dO), lse.data_ptr<float>(), Dv.data_ptr<float>(), dq, B, S, nq, nkv, \
                        (float)scale, st)
  if (hd == 128) DTB_ATTN_BWD(128);
  else if (hd == 64) DTB_ATTN_BWD(64);
  else if (hd == 32) DTB_ATTN_BWD(32);
  else DTB_ATTN_BWD(16);
#undef DTB_ATTN_BWD
  DTB_LAUNCH_CHECK();
  return dqkv;
}
