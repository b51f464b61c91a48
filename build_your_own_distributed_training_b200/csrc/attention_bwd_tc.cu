// Causal GQA flash-attention backward on tcgen05/TMEM (sm_100a), deterministic.
//
// Two kernels, no atomics (every output element is written by one CTA, and
// every sum runs in a fixed order), so the backward is bit-reproducible:
//
// attn_bwd_dkdv_tc: CTA per (128-key tile, kv head, batch).  For every query
//   head of the kv head's group and every 64-query tile at or after the
//   diagonal:
//     S^T  = K Q^T      [128 keys x 64 queries]   (TMEM, double buffered)
//     dP^T = V dO^T     [128 x 64]                (TMEM, double buffered)
//     P^T  = exp2(S^T * scale*log2e - lse*log2e), dS^T = P^T (dP^T - D)
//            (4 warps, thread = key row; both written to shared memory in bf16)
//     dV  += P^T dO     [128 x hd]                (TMEM accumulator)
//     dK  += dS^T Q     [128 x hd]                (TMEM accumulator, * scale at the end)
// attn_bwd_dq_tc: CTA per (128-query tile, head, batch), over 64-key tiles:
//     S = Q K^T, dP = dO V^T, dS = P (dP - D), dQ += dS K.
//
// The Q / dO / K tiles are loaded once by TMA in the 128-byte-swizzled K-major
// layout; the same bytes serve as MN-major operands (a [rows][64] swizzled
// tile is both), so nothing is transposed.  lse and D = rowsum(dO * O) rows
// arrive by bulk copies next to the tiles, three tiles deep; S / dP are issued
// two tiles ahead of the products that consume P / dS, and P / dS sit in two
// shared-memory buffers, so the elementwise warps of tile i only wait for the
// products of tile i-2.  The elementwise part reads its TMEM rows with one
// wait, and computes P with one FFMA and one ex2 per element; the causal mask
// is applied on the tiles that cross the diagonal only.  Warp 0 loads, warp 1
// owns TMEM and issues MMAs, warps 2-9 (two warpgroups, each taking half of a
// tile's columns) do the elementwise part.  Bounded waits only.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include "common.cuh"

namespace dtb {
namespace fab {

constexpr float LOG2E = 1.4426950408889634f;

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// one 64-column bf16 row segment into a [rows][64] 128B-swizzled tile
__device__ __forceinline__ void store_row64(uint8_t* tile, int r, const uint32_t (&pk)[32]) {
#pragma unroll
  for (int cc = 0; cc < 8; ++cc) {
    uint4 v;
    v.x = pk[cc * 4 + 0];
    v.y = pk[cc * 4 + 1];
    v.z = pk[cc * 4 + 2];
    v.w = pk[cc * 4 + 3];
    *reinterpret_cast<uint4*>(tile + r * 128 + ((cc ^ (r & 7)) << 4)) = v;
  }
}

// columns [32*half, 32*half + 32) of row r of a [rows][64] swizzled tile
__device__ __forceinline__ void store_row32(uint8_t* tile, int r, int half, const uint32_t (&pk)[16]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int cc = half * 4 + q;
    uint4 v;
    v.x = pk[q * 4 + 0];
    v.y = pk[q * 4 + 1];
    v.z = pk[q * 4 + 2];
    v.w = pk[q * 4 + 3];
    *reinterpret_cast<uint4*>(tile + r * 128 + ((cc ^ (r & 7)) << 4)) = v;
  }
}

struct BwdArgs {
  const float* lse;   // [B, nq, S] natural log
  const float* Dv;    // [B, nq, S]
  __nv_bfloat16* dqkv;
  int S, nq, nkv;
  float scale, scale_log2;
  int* err;
  long long* trace;   // phase timestamps of one CTA (DTB_ATTN_TRACE=1), else nullptr
  int early_s;        // dK/dV TMEM kernel: issue S^T of the next tile before dK of this one
};

// clock64 timestamp of phase k of iteration j for trace row `role`
__device__ __forceinline__ void trace_mark(const BwdArgs& a, bool on, int role, int j, int k) {
  if (on && j < 64) a.trace[(role * 64 + j) * 8 + k] = clock64();
}

// ============================================================== dK / dV
template <int HD>
struct SmKV {
  static constexpr int KV_TILE = 128 * HD * 2;   // K or V: [hd/64][128 rows][128 B]
  static constexpr int QT = 64 * HD * 2;         // Q or dO tile: [hd/64][64 rows][128 B]
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = K_OFF + KV_TILE;
  static constexpr int NS = 3;                   // Q / dO / lse / D load stages
  static constexpr int Q_OFF = V_OFF + KV_TILE;
  static constexpr int O_OFF = Q_OFF + NS * QT;  // dO
  static constexpr int P_OFF = O_OFF + NS * QT;      // P^T [128][64] bf16, 2 buffers
  static constexpr int DS_OFF = P_OFF + 2 * 16384;   // dS^T, 2 buffers
  static constexpr int LD_OFF = DS_OFF + 2 * 16384;  // NS x (lse[64], D[64]) floats
  static constexpr int BAR_OFF = LD_OFF + NS * 512;
  static constexpr int N_BARS = 16;
  static constexpr int TOTAL = BAR_OFF + N_BARS * 8 + 16 + 1024;
};

template <int HD>
__global__ void __launch_bounds__(320, 1)
    attn_bwd_dkdv_tc_kernel(const __grid_constant__ CUtensorMap tm_kv, const __grid_constant__ CUtensorMap tm_q,
                            const __grid_constant__ CUtensorMap tm_do, const BwdArgs a) {
  using L = SmKV<HD>;
  constexpr int BKV = 128, BQ = 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::BAR_OFF);
  constexpr int NS = L::NS;
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;   // [NS]
  uint64_t* q_empty = bars + 4;  // [NS]
  uint64_t* s_full = bars + 7;   // [2]  S^T and dP^T ready
  uint64_t* s_empty = bars + 9;  // [2]
  uint64_t* p_full = bars + 11;  // [2] P^T / dS^T of tile it written into buffer it & 1
  uint64_t* p_done = bars + 13;  // [2] dV / dK MMAs of tile it (read buffer it & 1) finished
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + L::N_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = a.S / BKV;
  // grid (kv heads x batch, key tiles): tiles near the end have the least work,
  // and blocks start in linear order, so every head's longer tiles start first
  const int kb = nkb - 1 - blockIdx.y;
  const int hk = blockIdx.x % a.nkv, b = blockIdx.x / a.nkv;
  const int grp = a.nq / a.nkv;
  const int kv0 = kb * BKV;
  const int q_first = kv0 / BQ;
  const int nqt = a.S / BQ - q_first;
  const int total = nqt * grp;
  const int row0 = b * a.S;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 256);
      mbar_init(&p_full[i], 256);
      mbar_init(&p_done[i], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  // TMEM: S^T[2] at 0/64, dP^T[2] at 128/192, dV at 256, dK at 256+HD
  const uint32_t t_s[2] = {tmem, tmem + 64}, t_dp[2] = {tmem + 128, tmem + 192};
  const uint32_t t_dv = tmem + 256, t_dk = tmem + 256 + HD;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 2 * L::KV_TILE);
#pragma unroll
      for (int c = 0; c < HD / 64; ++c) {
        tma_load_2d(sm + L::K_OFF + c * 16384, &tm_kv, kv_full, (a.nq + hk) * HD + c * 64, row0 + kv0);
        tma_load_2d(sm + L::V_OFF + c * 16384, &tm_kv, kv_full, (a.nq + a.nkv + hk) * HD + c * 64, row0 + kv0);
      }
      for (int it = 0; it < total; ++it) {
        const int st = it % NS;
        if (*abort_flag || !mbar_wait(&q_empty[st], ((it / NS) & 1) ^ 1, a.err)) {
          *abort_flag = 1;
          break;
        }
        const int hh = hk * grp + it / nqt;
        const int q0 = (q_first + it % nqt) * BQ;
        mbar_arrive_expect_tx(&q_full[st], 2 * L::QT + 512);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c) {
          tma_load_2d(sm + L::Q_OFF + st * L::QT + c * 8192, &tm_q, &q_full[st], hh * HD + c * 64, row0 + q0);
          tma_load_2d(sm + L::O_OFF + st * L::QT + c * 8192, &tm_do, &q_full[st], hh * HD + c * 64, row0 + q0);
        }
        const long li = ((long)b * a.nq + hh) * a.S + q0;
        bulk_load(sm + L::LD_OFF + st * 512, a.lse + li, 256, &q_full[st]);
        bulk_load(sm + L::LD_OFF + st * 512 + 256, a.Dv + li, 256, &q_full[st]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_S = idesc_bf16(128, 64, false, false);   // S^T, dP^T
      constexpr uint32_t ID_G = idesc_bf16(128, HD, false, true);    // dV, dK (B = dO / Q as MN-major)
      const uint32_t k0 = smem_u32(sm + L::K_OFF), v0 = smem_u32(sm + L::V_OFF);
      const uint32_t pt = smem_u32(sm + L::P_OFF), dst = smem_u32(sm + L::DS_OFF);
      bool ok = mbar_wait(kv_full, 0, a.err);
      auto issue_s = [&](int it) -> bool {
        const int st = it % NS, tb = it & 1;
        if (!mbar_wait(&q_full[st], (it / NS) & 1, a.err)) return false;
        if (!mbar_wait(&s_empty[tb], ((it >> 1) & 1) ^ 1, a.err)) return false;
        tc_fence_after();
        const uint32_t q0 = smem_u32(sm + L::Q_OFF + st * L::QT), o0 = smem_u32(sm + L::O_OFF + st * L::QT);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t oa = (kk >> 2) * 16384 + (kk & 3) * 32;  // K / V atoms: 128 rows
          const uint32_t ob = (kk >> 2) * 8192 + (kk & 3) * 32;   // Q / dO atoms: 64 rows
          umma_bf16(t_s[tb], sdesc_sw128(k0 + oa, 16, 1024), sdesc_sw128(q0 + ob, 16, 1024), ID_S, kk != 0);
          umma_bf16(t_dp[tb], sdesc_sw128(v0 + oa, 16, 1024), sdesc_sw128(o0 + ob, 16, 1024), ID_S, kk != 0);
        }
        umma_commit(&s_full[tb]);
        return true;
      };
      // S^T / dP^T run two tiles ahead of the dV / dK products
      if (ok && total > 0) ok = issue_s(0);
      if (ok && total > 1) ok = issue_s(1);
      for (int it = 0; it < total && ok && !*abort_flag; ++it) {
        const int pb = it & 1;
        if (!mbar_wait(&p_full[pb], (it >> 1) & 1, a.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int st = it % NS;
        const uint32_t q0 = smem_u32(sm + L::Q_OFF + st * L::QT), o0 = smem_u32(sm + L::O_OFF + st * L::QT);
        const uint32_t ptb = pt + pb * 16384, dsb = dst + pb * 16384;
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk) {
          const uint32_t pa = kk * 32;        // [128][64] K-major A tile
          const uint32_t gb = kk * 2048;      // 16 query rows of the MN-major B tile
          umma_bf16(t_dv, sdesc_sw128(ptb + pa, 16, 1024), sdesc_sw128(o0 + gb, 8192, 1024), ID_G, (it | kk) != 0);
          umma_bf16(t_dk, sdesc_sw128(dsb + pa, 16, 1024), sdesc_sw128(q0 + gb, 8192, 1024), ID_G, (it | kk) != 0);
        }
        umma_commit(&q_empty[st]);
        umma_commit(&p_done[pb]);
        if (it + 2 < total && !issue_s(it + 2)) {
          ok = false;
          break;
        }
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // warps 2-9: two warpgroups; group g handles columns [32g, 32g+32) of every row
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int c0 = half * 32;
    const int r = quad * 32 + lane;  // key row within the tile
    const int kr = kv0 + r;
    const uint32_t lo = (uint32_t)(quad * 32) << 16;
    bool ok = true;
    for (int it = 0; it < total; ++it) {
      const int tb = it & 1, st = it % NS;
      if (*abort_flag || !mbar_wait(&s_full[tb], (it >> 1) & 1, a.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[32], dr[32];
      tmem_ld32_async(t_s[tb] + lo + c0, sr);
      tmem_ld32_async(t_dp[tb] + lo + c0, dr);
      tmem_wait_ld();
      tmem_regs(sr);
      tmem_regs(dr);
      tc_fence_before();
      mbar_arrive(&s_empty[tb]);
      // lse / D rows of this tile arrived with the tile's bulk copies (already
      // complete: the MMA warp waited for them); waiting here makes the async
      // writes visible to these threads
      if (!mbar_wait(&q_full[st], (it / NS) & 1, a.err)) {
        ok = false;
        break;
      }
      const float* Ls = reinterpret_cast<const float*>(sm + L::LD_OFF + st * 512);
      const float* Ds = Ls + 64;
      const int q0 = (q_first + it % nqt) * BQ;
      // only the two query tiles that overlap the diagonal of this key block are masked
      const bool diag = (it % nqt) < BKV / BQ;
      uint32_t pp[16], pd[16];
#pragma unroll
      for (int c = 0; c < 32; c += 2) {
        float p[2], d[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int qc = c0 + c + e;
          const float xe = fmaf(__uint_as_float(sr[c + e]), a.scale_log2, Ls[qc] * -LOG2E);
          float v = ex2_approx(xe);
          if (diag && q0 + qc < kr) v = 0.f;
          p[e] = v;
          d[e] = v * (__uint_as_float(dr[c + e]) - Ds[qc]);
        }
        pp[c / 2] = pack_bf16x2(p[0], p[1]);
        pd[c / 2] = pack_bf16x2(d[0], d[1]);
      }
      // buffer it & 1 was last read by the dV / dK MMAs of tile it - 2
      if (it > 1) {
        if (!mbar_wait(&p_done[it & 1], ((it - 2) >> 1) & 1, a.err)) {
          ok = false;
          break;
        }
      }
      store_row32(sm + L::P_OFF + (it & 1) * 16384, r, half, pp);
      store_row32(sm + L::DS_OFF + (it & 1) * 16384, r, half, pd);
      fence_proxy_async_smem();
      mbar_arrive(&p_full[it & 1]);
    }
    if (ok && total > 0 && mbar_wait(&p_done[(total - 1) & 1], ((total - 1) >> 1) & 1, a.err)) {
      tc_fence_after();
      const long ld = (long)(a.nq + 2 * a.nkv) * HD;
      __nv_bfloat16* gk = a.dqkv + ((long)row0 + kr) * ld + (a.nq + hk) * HD;
      __nv_bfloat16* gv = a.dqkv + ((long)row0 + kr) * ld + (a.nq + a.nkv + hk) * HD;
#pragma unroll 1
      for (int c = half * (HD / 2); c < (half + 1) * (HD / 2); c += 32) {
        float dk[32], dv[32];
        tmem_ld32(t_dk + lo + c, dk);
        tmem_ld32(t_dv + lo + c, dv);
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 wk, wv;
          wk.x = pack_bf16x2(dk[i] * a.scale, dk[i + 1] * a.scale);
          wk.y = pack_bf16x2(dk[i + 2] * a.scale, dk[i + 3] * a.scale);
          wk.z = pack_bf16x2(dk[i + 4] * a.scale, dk[i + 5] * a.scale);
          wk.w = pack_bf16x2(dk[i + 6] * a.scale, dk[i + 7] * a.scale);
          wv.x = pack_bf16x2(dv[i], dv[i + 1]);
          wv.y = pack_bf16x2(dv[i + 2], dv[i + 3]);
          wv.z = pack_bf16x2(dv[i + 4], dv[i + 5]);
          wv.w = pack_bf16x2(dv[i + 6], dv[i + 7]);
          *reinterpret_cast<uint4*>(gk + c + i) = wk;
          *reinterpret_cast<uint4*>(gv + c + i) = wv;
        }
      }
    } else {
      *abort_flag = 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ============================================================== dK / dV, P in TMEM
// attn_bwd_dkdv_tm_kernel: CTA per (128-key tile, kv head, batch), 128-query
// tiles (every MMA 128 x 128 or 128 x hd wide instead of the 64-query
// kernel's 128 x 64), with P^T and dS^T kept in tensor memory as the A
// operands of the dV / dK products, so they need no shared memory:
//   TMEM  S^T [0,128) | dP^T [128,256) | dV [256, 256+hd) | dK [256+hd, 256+2hd)
//   The elementwise threads (two per key row, 64 queries each) read their
//   S^T / dP^T columns and write P^T / dS^T as bf16 pairs over the first 32
//   of those same columns, so nothing another thread still has to read is
//   overwritten.  MMA order per query tile: S^T, dP^T, then (once P^T is
//   written) dV += P^T dO, then (once dS^T is written) dK += dS^T Q; the next
//   tile's S^T / dP^T are issued after these, and the tensor pipe runs its
//   operations in issue order, so they overwrite P^T / dS^T only after use.
//   The exponentials of tile i overlap its dP^T product, the dS^T products its
//   dV product.  Q / dO / lse / D: 2-deep ring.  Warp 0 loads, warp 1 owns
//   TMEM and issues MMAs, warps 2-9 the elementwise part.  Bounded waits.
__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t (&v)[32]) {
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

template <int HD>
struct SmKVT {
  static constexpr int KV_TILE = 128 * HD * 2;   // K or V: [hd/64][128 rows][128 B]
  static constexpr int QT = 128 * HD * 2;        // Q or dO tile: [hd/64][128 rows][128 B]
  static constexpr int NS = 2;
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = K_OFF + KV_TILE;
  static constexpr int Q_OFF = V_OFF + KV_TILE;
  static constexpr int O_OFF = Q_OFF + NS * QT;
  static constexpr int LD_OFF = O_OFF + NS * QT;     // NS x (lse[128], D[128]) floats
  static constexpr int BAR_OFF = LD_OFF + NS * 1024;
  static constexpr int N_BARS = 16;
  static constexpr int TOTAL = BAR_OFF + N_BARS * 8 + 16 + 1024;
  static_assert(TOTAL <= 232448, "shared memory per CTA");
};

template <int HD>
__global__ void __launch_bounds__(320, 1)
    attn_bwd_dkdv_tm_kernel(const __grid_constant__ CUtensorMap tm_kv, const __grid_constant__ CUtensorMap tm_q,
                            const __grid_constant__ CUtensorMap tm_do, const BwdArgs a) {
  using L = SmKVT<HD>;
  constexpr int BKV = 128, BQ = 128, NS = L::NS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::BAR_OFF);
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;   // [NS]
  uint64_t* q_empty = bars + 3;  // [NS]
  uint64_t* s_full = bars + 5;   // S^T of the current tile
  uint64_t* dp_full = bars + 6;  // dP^T of the current tile
  uint64_t* pt_full = bars + 7;  // P^T written (256 arrivals)
  uint64_t* ds_full = bars + 8;  // dS^T written (256 arrivals)
  uint64_t* g_done = bars + 9;   // dV / dK products of the tile finished
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + L::N_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = a.S / BKV;
  // grid (kv heads x batch, key tiles): tiles near the end have the least work,
  // and blocks start in linear order, so every head's longer tiles start first
  const int kb = nkb - 1 - blockIdx.y;
  const int hk = blockIdx.x % a.nkv, b = blockIdx.x / a.nkv;
  const int grp = a.nq / a.nkv;
  const int kv0 = kb * BKV;
  const int nqt = a.S / BQ - kb;        // query tiles from the diagonal one
  const int total = nqt * grp;
  const int row0 = b * a.S;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(dp_full, 1);
    mbar_init(pt_full, 256);
    mbar_init(ds_full, 256);
    mbar_init(g_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint32_t t_s = tmem, t_dp = tmem + 128, t_dv = tmem + 256, t_dk = tmem + 256 + HD;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 2 * L::KV_TILE);
#pragma unroll
      for (int c = 0; c < HD / 64; ++c) {
        tma_load_2d(sm + L::K_OFF + c * 16384, &tm_kv, kv_full, (a.nq + hk) * HD + c * 64, row0 + kv0);
        tma_load_2d(sm + L::V_OFF + c * 16384, &tm_kv, kv_full, (a.nq + a.nkv + hk) * HD + c * 64, row0 + kv0);
      }
      for (int it = 0; it < total; ++it) {
        const int st = it % NS;
        if (*abort_flag || !mbar_wait(&q_empty[st], ((it / NS) & 1) ^ 1, a.err)) {
          *abort_flag = 1;
          break;
        }
        const int hh = hk * grp + it / nqt;
        const int q0 = (kb + it % nqt) * BQ;
        mbar_arrive_expect_tx(&q_full[st], 2 * L::QT + 1024);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c) {
          tma_load_2d(sm + L::Q_OFF + st * L::QT + c * 16384, &tm_q, &q_full[st], hh * HD + c * 64, row0 + q0);
          tma_load_2d(sm + L::O_OFF + st * L::QT + c * 16384, &tm_do, &q_full[st], hh * HD + c * 64, row0 + q0);
        }
        const long li = ((long)b * a.nq + hh) * a.S + q0;
        bulk_load(sm + L::LD_OFF + st * 1024, a.lse + li, 512, &q_full[st]);
        bulk_load(sm + L::LD_OFF + st * 1024 + 512, a.Dv + li, 512, &q_full[st]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_S = idesc_bf16(BKV, BQ, false, false);   // S^T, dP^T: [keys x queries]
      constexpr uint32_t ID_G = idesc_bf16(BKV, HD, false, true);    // dV, dK: A (TMEM) x B (dO / Q, MN-major)
      const uint32_t k0 = smem_u32(sm + L::K_OFF), v0 = smem_u32(sm + L::V_OFF);
      bool ok = mbar_wait(kv_full, 0, a.err);
      // S^T of query tile `t` once its Q / dO stage has landed
      auto issue_s = [&](int t) -> bool {
        const int ss = t % NS;
        if (!mbar_wait(&q_full[ss], (t / NS) & 1, a.err)) return false;
        tc_fence_after();
        const uint32_t qs = smem_u32(sm + L::Q_OFF + ss * L::QT);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_bf16(t_s, sdesc_sw128(k0 + off, 16, 1024), sdesc_sw128(qs + off, 16, 1024), ID_S, kk != 0);
        }
        umma_commit(s_full);
        return true;
      };
      // early_s: per tile  dP^T(i) | P^T(i) written | dV(i)  S^T(i+1) | dS^T(i) written | dK(i),
      // so the exponentials of tile i+1 run while the tensor pipe does dV(i), dK(i) and dP^T(i+1)
      // (S^T(i+1) overwrites P^T(i) only after dV(i) has read it: the pipe runs in issue order;
      // dP^T(i+1) overwrites dS^T(i) only after dK(i)).  Otherwise S^T(i+1) waits for dK(i).
      const bool early = a.early_s != 0;
      if (early && total > 0 && ok) ok = issue_s(0);
      for (int it = 0; it < total && ok && !*abort_flag; ++it) {
        const int st = it % NS;
        if (!early && !issue_s(it)) {
          ok = false;
          break;
        }
        const uint32_t q0 = smem_u32(sm + L::Q_OFF + st * L::QT), o0 = smem_u32(sm + L::O_OFF + st * L::QT);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_bf16(t_dp, sdesc_sw128(v0 + off, 16, 1024), sdesc_sw128(o0 + off, 16, 1024), ID_S, kk != 0);
        }
        umma_commit(dp_full);
        // dV += P^T dO: A = P^T from TMEM (queries 16kk.. at column 64*(kk/4) + 8*(kk%4)),
        // B = the dO tile read MN-major (16 query rows per step)
        if (!mbar_wait(pt_full, it & 1, a.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk) {
          const uint32_t ta = t_s + 64 * (kk >> 2) + 8 * (kk & 3);
          umma_bf16_ta(t_dv, ta, sdesc_sw128(o0 + kk * 2048, 16384, 1024), ID_G, (it | kk) != 0);
        }
        if (early && it + 1 < total && !issue_s(it + 1)) {
          ok = false;
          break;
        }
        if (!mbar_wait(ds_full, it & 1, a.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk) {
          const uint32_t ta = t_dp + 64 * (kk >> 2) + 8 * (kk & 3);
          umma_bf16_ta(t_dk, ta, sdesc_sw128(q0 + kk * 2048, 16384, 1024), ID_G, (it | kk) != 0);
        }
        umma_commit(&q_empty[st]);
        umma_commit(g_done);
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // warps 2-9: thread = key row r; half h = queries [64h, 64h + 64) of every tile
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int c0 = half * 64;
    const int r = quad * 32 + lane;
    const int kr = kv0 + r;
    const uint32_t lo = (uint32_t)(quad * 32) << 16;
    bool ok = true;
    for (int it = 0; it < total; ++it) {
      const int st = it % NS;
      const int q0 = (kb + it % nqt) * BQ;
      const bool diag = (it % nqt) == 0;  // the first query tile of each head sits on the diagonal
      if (*abort_flag || !mbar_wait(s_full, it & 1, a.err) || !mbar_wait(&q_full[st], (it / NS) & 1, a.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float* Ls = reinterpret_cast<const float*>(sm + L::LD_OFF + st * 1024) + c0;
      const float* Ds = Ls + 128;
      uint32_t sr[2][32];
      tmem_ld32_async(t_s + lo + c0, sr[0]);
      tmem_ld32_async(t_s + lo + c0 + 32, sr[1]);
      tmem_wait_ld();
      tmem_regs(sr[0]);
      tmem_regs(sr[1]);
      float p[64];
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const float xe = fmaf(__uint_as_float(sr[c >> 5][c & 31]), a.scale_log2, Ls[c] * -LOG2E);
        float v = (c & 6) == 6 ? exp2_fma(xe) : ex2_approx(xe);
        if (diag && q0 + c0 + c < kr) v = 0.f;
        p[c] = v;
      }
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) pk[c] = pack_bf16x2(p[2 * c], p[2 * c + 1]);
      tmem_st32u(t_s + lo + c0, pk);  // P^T over this thread's own S^T columns
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      mbar_arrive(pt_full);
      if (!mbar_wait(dp_full, it & 1, a.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t dr[2][32];
      tmem_ld32_async(t_dp + lo + c0, dr[0]);
      tmem_ld32_async(t_dp + lo + c0 + 32, dr[1]);
      tmem_wait_ld();
      tmem_regs(dr[0]);
      tmem_regs(dr[1]);
#pragma unroll
      for (int c = 0; c < 32; ++c)
        pk[c] = pack_bf16x2(p[2 * c] * (__uint_as_float(dr[(2 * c) >> 5][(2 * c) & 31]) - Ds[2 * c]),
                            p[2 * c + 1] * (__uint_as_float(dr[(2 * c + 1) >> 5][(2 * c + 1) & 31]) - Ds[2 * c + 1]));
      tmem_st32u(t_dp + lo + c0, pk);  // dS^T over this thread's own dP^T columns
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      mbar_arrive(ds_full);
    }
    if (ok && total > 0 && mbar_wait(g_done, (total - 1) & 1, a.err)) {
      tc_fence_after();
      const long ld = (long)(a.nq + 2 * a.nkv) * HD;
      __nv_bfloat16* gk = a.dqkv + ((long)row0 + kr) * ld + (a.nq + hk) * HD;
      __nv_bfloat16* gv = a.dqkv + ((long)row0 + kr) * ld + (a.nq + a.nkv + hk) * HD;
#pragma unroll 1
      for (int c = half * (HD / 2); c < (half + 1) * (HD / 2); c += 32) {
        float dk[32], dv[32];
        tmem_ld32(t_dk + lo + c, dk);
        tmem_ld32(t_dv + lo + c, dv);
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 wk, wv;
          wk.x = pack_bf16x2(dk[i] * a.scale, dk[i + 1] * a.scale);
          wk.y = pack_bf16x2(dk[i + 2] * a.scale, dk[i + 3] * a.scale);
          wk.z = pack_bf16x2(dk[i + 4] * a.scale, dk[i + 5] * a.scale);
          wk.w = pack_bf16x2(dk[i + 6] * a.scale, dk[i + 7] * a.scale);
          wv.x = pack_bf16x2(dv[i], dv[i + 1]);
          wv.y = pack_bf16x2(dv[i + 2], dv[i + 3]);
          wv.z = pack_bf16x2(dv[i + 4], dv[i + 5]);
          wv.w = pack_bf16x2(dv[i + 6], dv[i + 7]);
          *reinterpret_cast<uint4*>(gk + c + i) = wk;
          *reinterpret_cast<uint4*>(gv + c + i) = wv;
        }
      }
    } else {
      *abort_flag = 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ============================================================== dQ
template <int HD, int STAGES = 4>
struct SmQ {
  static constexpr int QT = 128 * HD * 2;        // Q or dO: [hd/64][128][128 B]
  static constexpr int KT = 64 * HD * 2;         // K or V tile: [hd/64][64][128 B]
  static constexpr int Q_OFF = 0;
  static constexpr int O_OFF = Q_OFF + QT;
  static constexpr int NS = STAGES;              // K / V load stages
  static constexpr int K_OFF = O_OFF + QT;
  static constexpr int V_OFF = K_OFF + NS * KT;
  static constexpr int DS_OFF = V_OFF + NS * KT;  // dS [128][64], 2 buffers
  static constexpr int BAR_OFF = DS_OFF + 2 * 16384;
  static constexpr int N_BARS = 2 * NS + 10;
  static constexpr int TOTAL = BAR_OFF + N_BARS * 8 + 16 + 1024;
};

template <int HD, int STAGES>
__global__ void __launch_bounds__(320, 1)
    attn_bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tm_q128, const __grid_constant__ CUtensorMap tm_do128,
                          const __grid_constant__ CUtensorMap tm_kv64, const BwdArgs a) {
  using L = SmQ<HD, STAGES>;
  constexpr int BQ = 128, BKV = 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::BAR_OFF);
  constexpr int NS = L::NS;
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;            // [NS]
  uint64_t* kv_empty = bars + 1 + NS;      // [NS]
  uint64_t* s_full = bars + 1 + 2 * NS;    // [2]
  uint64_t* s_empty = bars + 3 + 2 * NS;   // [2]
  uint64_t* p_full = bars + 5 + 2 * NS;    // [2] dS of key tile j written into buffer j & 1
  uint64_t* p_done = bars + 7 + 2 * NS;    // [2] dQ MMAs of key tile j (read buffer j & 1) finished
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + L::N_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool tr = a.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0;
  const int nqb = a.S / BQ;
  const int qb = nqb - 1 - blockIdx.y;  // grid (heads x batch, query tiles): longest rows first
  const int h = blockIdx.x % a.nq, b = blockIdx.x / a.nq;
  const int hk = h / (a.nq / a.nkv);
  const int q0 = qb * BQ;
  const int nkt = (q0 + BQ) / BKV;
  const int row0 = b * a.S;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 256);
      mbar_init(&p_full[i], 256);
      mbar_init(&p_done[i], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint32_t t_s[2] = {tmem, tmem + 64}, t_dp[2] = {tmem + 128, tmem + 192};
  const uint32_t t_dq = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, 2 * L::QT);
#pragma unroll
      for (int c = 0; c < HD / 64; ++c) {
        tma_load_2d(sm + L::Q_OFF + c * 16384, &tm_q128, q_full, h * HD + c * 64, row0 + q0);
        tma_load_2d(sm + L::O_OFF + c * 16384, &tm_do128, q_full, h * HD + c * 64, row0 + q0);
      }
      for (int j = 0; j < nkt; ++j) {
        const int st = j % NS;
        trace_mark(a, tr, 0, j, 0);
        if (*abort_flag || !mbar_wait(&kv_empty[st], ((j / NS) & 1) ^ 1, a.err)) {
          *abort_flag = 1;
          break;
        }
        trace_mark(a, tr, 0, j, 1);
        mbar_arrive_expect_tx(&kv_full[st], 2 * L::KT);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c) {
          tma_load_2d(sm + L::K_OFF + st * L::KT + c * 8192, &tm_kv64, &kv_full[st], (a.nq + hk) * HD + c * 64,
                      row0 + j * BKV);
          tma_load_2d(sm + L::V_OFF + st * L::KT + c * 8192, &tm_kv64, &kv_full[st],
                      (a.nq + a.nkv + hk) * HD + c * 64, row0 + j * BKV);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_S = idesc_bf16(128, 64, false, false);
      constexpr uint32_t ID_Q = idesc_bf16(128, HD, false, true);
      const uint32_t qa = smem_u32(sm + L::Q_OFF), oa = smem_u32(sm + L::O_OFF), dsa = smem_u32(sm + L::DS_OFF);
      bool ok = mbar_wait(q_full, 0, a.err);
      auto issue_s = [&](int j) -> bool {
        const int st = j % NS, tb = j & 1;
        trace_mark(a, tr, 1, j, 0);
        if (!mbar_wait(&kv_full[st], (j / NS) & 1, a.err)) return false;
        trace_mark(a, tr, 1, j, 1);
        if (!mbar_wait(&s_empty[tb], ((j >> 1) & 1) ^ 1, a.err)) return false;
        trace_mark(a, tr, 1, j, 2);
        tc_fence_after();
        const uint32_t k0 = smem_u32(sm + L::K_OFF + st * L::KT), v0 = smem_u32(sm + L::V_OFF + st * L::KT);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t o128 = (kk >> 2) * 16384 + (kk & 3) * 32;
          const uint32_t o64 = (kk >> 2) * 8192 + (kk & 3) * 32;
          umma_bf16(t_s[tb], sdesc_sw128(qa + o128, 16, 1024), sdesc_sw128(k0 + o64, 16, 1024), ID_S, kk != 0);
          umma_bf16(t_dp[tb], sdesc_sw128(oa + o128, 16, 1024), sdesc_sw128(v0 + o64, 16, 1024), ID_S, kk != 0);
        }
        umma_commit(&s_full[tb]);
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok && nkt > 1) ok = issue_s(1);
      for (int j = 0; j < nkt && ok && !*abort_flag; ++j) {
        const int pb = j & 1;
        trace_mark(a, tr, 2, j, 0);
        if (!mbar_wait(&p_full[pb], (j >> 1) & 1, a.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int st = j % NS;
        const uint32_t k0 = smem_u32(sm + L::K_OFF + st * L::KT);
        const uint32_t dsb = dsa + pb * 16384;
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk)
          umma_bf16(t_dq, sdesc_sw128(dsb + kk * 32, 16, 1024), sdesc_sw128(k0 + kk * 2048, 8192, 1024), ID_Q,
                    (j | kk) != 0);
        umma_commit(&kv_empty[st]);
        umma_commit(&p_done[pb]);
        trace_mark(a, tr, 2, j, 1);
        if (j + 2 < nkt && !issue_s(j + 2)) {
          ok = false;
          break;
        }
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // warpgroup: columns [32*half, 32*half + 32)
    const int c0 = half * 32;
    const int r = quad * 32 + lane;
    const int qr = q0 + r;
    const uint32_t lo = (uint32_t)(quad * 32) << 16;
    const long li = ((long)b * a.nq + h) * a.S + qr;
    const float L2 = a.lse[li] * LOG2E, Dr = a.Dv[li];
    bool ok = true;
    for (int j = 0; j < nkt; ++j) {
      const int tb = j & 1;
      const bool trw = tr && warp == 2 && lane == 0;
      trace_mark(a, trw, 3, j, 0);
      if (*abort_flag || !mbar_wait(&s_full[tb], (j >> 1) & 1, a.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[32], dr[32];
      tmem_ld32_async(t_s[tb] + lo + c0, sr);
      tmem_ld32_async(t_dp[tb] + lo + c0, dr);
      trace_mark(a, trw, 3, j, 1);
      tmem_wait_ld();
      tmem_regs(sr);
      tmem_regs(dr);
      trace_mark(a, trw, 3, j, 2);
      tc_fence_before();
      mbar_arrive(&s_empty[tb]);
      // key tiles that reach past the first query row of this tile hold masked columns
      const bool diag = j * BKV + BKV - 1 > q0;
      uint32_t pd[16];
#pragma unroll
      for (int c = 0; c < 32; c += 2) {
        float d[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int kc = j * BKV + c0 + c + e;
          const float xe = fmaf(__uint_as_float(sr[c + e]), a.scale_log2, -L2);
          float p = ex2_approx(xe);
          if (diag && kc > qr) p = 0.f;
          d[e] = p * (__uint_as_float(dr[c + e]) - Dr);
        }
        pd[c / 2] = pack_bf16x2(d[0], d[1]);
      }
      trace_mark(a, trw, 3, j, 3);
      // buffer j & 1 was last read by the dQ MMAs of key tile j - 2
      if (j > 1) {
        if (!mbar_wait(&p_done[j & 1], ((j - 2) >> 1) & 1, a.err)) {
          ok = false;
          break;
        }
      }
      trace_mark(a, trw, 3, j, 4);
      store_row32(sm + L::DS_OFF + (j & 1) * 16384, r, half, pd);
      fence_proxy_async_smem();
      mbar_arrive(&p_full[j & 1]);
      trace_mark(a, trw, 3, j, 5);
    }
    if (ok && mbar_wait(&p_done[(nkt - 1) & 1], ((nkt - 1) >> 1) & 1, a.err)) {
      tc_fence_after();
      const long ld = (long)(a.nq + 2 * a.nkv) * HD;
      __nv_bfloat16* gq = a.dqkv + ((long)row0 + qr) * ld + h * HD;
#pragma unroll 1
      for (int c = half * (HD / 2); c < (half + 1) * (HD / 2); c += 32) {
        float dq[32];
        tmem_ld32(t_dq + lo + c, dq);
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 w;
          w.x = pack_bf16x2(dq[i] * a.scale, dq[i + 1] * a.scale);
          w.y = pack_bf16x2(dq[i + 2] * a.scale, dq[i + 3] * a.scale);
          w.z = pack_bf16x2(dq[i + 4] * a.scale, dq[i + 5] * a.scale);
          w.w = pack_bf16x2(dq[i + 6] * a.scale, dq[i + 7] * a.scale);
          *reinterpret_cast<uint4*>(gq + c + i) = w;
        }
      }
    } else {
      *abort_flag = 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ============================================================== dQ, 128-key tiles
// Same product as attn_bwd_dq_tc_kernel with 128-key tiles: S, dP and dQ are
// M=128 x N=128 MMAs, so each tcgen05.mma carries twice the work of the
// 64-key version and the MMA count per key drops by 40% (that kernel is bound
// by the cost of issuing its small N=64 instructions).  TMEM holds one S and
// one dP (128 columns each) plus dQ; S_{j+1} is issued as soon as the
// elementwise warps have read S_j, so it overlaps their math and dQ_j.
template <int HD>
struct SmQ128 {
  static constexpr int QT = 128 * HD * 2;        // Q or dO: [hd/64][128][128 B]
  static constexpr int KT = 128 * HD * 2;        // K or V: [hd/64][128 keys][128 B]
  // separate rings: a K stage is held until dQ_j finishes, a V stage only until
  // dP_j does, so K gets the depth
  static constexpr int NSK = 3;
  static constexpr int NSV = HD == 128 ? 1 : 2;
  static constexpr int Q_OFF = 0;
  static constexpr int O_OFF = Q_OFF + QT;
  static constexpr int K_OFF = O_OFF + QT;
  static constexpr int V_OFF = K_OFF + NSK * KT;
  static constexpr int DS_OFF = V_OFF + NSV * KT;  // dS [128 q][128 keys] bf16: 2 atoms
  static constexpr int BAR_OFF = DS_OFF + 32768;
  static constexpr int N_BARS = 2 * (NSK + NSV) + 6;
  static constexpr int TOTAL = BAR_OFF + N_BARS * 8 + 16 + 1024;
};

template <int HD>
__global__ void __launch_bounds__(320, 1)
    attn_bwd_dq128_tc_kernel(const __grid_constant__ CUtensorMap tm_q128, const __grid_constant__ CUtensorMap tm_do128,
                             const __grid_constant__ CUtensorMap tm_kv128, const BwdArgs a) {
  using L = SmQ128<HD>;
  constexpr int BQ = 128, BKV = 128, NSK = L::NSK, NSV = L::NSV;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;                   // [NSK]
  uint64_t* k_empty = k_full + NSK;              // [NSK]
  uint64_t* v_full = k_empty + NSK;              // [NSV]
  uint64_t* v_empty = v_full + NSV;              // [NSV]
  uint64_t* s_full = v_empty + NSV;              // S_j and dP_j in TMEM
  uint64_t* s_empty = s_full + 1;                // the elementwise warps have read S_j and dP_j
  uint64_t* p_full = s_full + 2;                 // dS_j in shared memory
  uint64_t* p_done = s_full + 3;                 // the dQ MMAs of key tile j (read dS) finished
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + L::N_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool tr = a.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0;
  const int nqb = a.S / BQ;
  const int qb = nqb - 1 - blockIdx.y;  // grid (heads x batch, query tiles): longest rows first
  const int h = blockIdx.x % a.nq, b = blockIdx.x / a.nq;
  const int hk = h / (a.nq / a.nkv);
  const int q0 = qb * BQ;
  const int nkt = qb + 1;                 // causal: key tiles 0..qb
  const int row0 = b * a.S;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < NSK; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < NSV; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_empty, 256);
    mbar_init(p_full, 256);
    mbar_init(p_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint32_t t_s = tmem, t_dp = tmem + 128, t_dq = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, 2 * L::QT);
#pragma unroll
      for (int c = 0; c < HD / 64; ++c) {
        tma_load_2d(sm + L::Q_OFF + c * 16384, &tm_q128, q_full, h * HD + c * 64, row0 + q0);
        tma_load_2d(sm + L::O_OFF + c * 16384, &tm_do128, q_full, h * HD + c * 64, row0 + q0);
      }
      for (int j = 0; j < nkt; ++j) {
        const int sk = j % NSK, sv = j % NSV;
        trace_mark(a, tr, 0, j, 0);
        if (*abort_flag || !mbar_wait(&k_empty[sk], ((j / NSK) & 1) ^ 1, a.err)) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&k_full[sk], L::KT);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c)
          tma_load_2d(sm + L::K_OFF + sk * L::KT + c * 16384, &tm_kv128, &k_full[sk], (a.nq + hk) * HD + c * 64,
                      row0 + j * BKV);
        trace_mark(a, tr, 0, j, 1);
        if (*abort_flag || !mbar_wait(&v_empty[sv], ((j / NSV) & 1) ^ 1, a.err)) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&v_full[sv], L::KT);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c)
          tma_load_2d(sm + L::V_OFF + sv * L::KT + c * 16384, &tm_kv128, &v_full[sv],
                      (a.nq + a.nkv + hk) * HD + c * 64, row0 + j * BKV);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_S = idesc_bf16(128, BKV, false, false);  // S = Q K^T, dP = dO V^T
      constexpr uint32_t ID_Q = idesc_bf16(128, HD, false, true);    // dQ += dS K (K tile MN-major)
      const uint32_t qa = smem_u32(sm + L::Q_OFF), oa = smem_u32(sm + L::O_OFF), dsa = smem_u32(sm + L::DS_OFF);
      bool ok = mbar_wait(q_full, 0, a.err);
      auto issue_s = [&](int j) -> bool {
        const int sk = j % NSK, sv = j % NSV;
        trace_mark(a, tr, 1, j, 0);
        if (!mbar_wait(&k_full[sk], (j / NSK) & 1, a.err)) return false;
        if (!mbar_wait(&v_full[sv], (j / NSV) & 1, a.err)) return false;
        trace_mark(a, tr, 1, j, 1);
        // TMEM S / dP are free once the elementwise warps read S_{j-1}, dP_{j-1}
        if (j > 0 && !mbar_wait(s_empty, (j - 1) & 1, a.err)) return false;
        trace_mark(a, tr, 1, j, 2);
        tc_fence_after();
        const uint32_t k0 = smem_u32(sm + L::K_OFF + sk * L::KT), v0 = smem_u32(sm + L::V_OFF + sv * L::KT);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t o = (kk >> 2) * 16384 + (kk & 3) * 32;   // 128-row atoms on both sides
          umma_bf16(t_s, sdesc_sw128(qa + o, 16, 1024), sdesc_sw128(k0 + o, 16, 1024), ID_S, kk != 0);
          umma_bf16(t_dp, sdesc_sw128(oa + o, 16, 1024), sdesc_sw128(v0 + o, 16, 1024), ID_S, kk != 0);
        }
        umma_commit(s_full);
        umma_commit(&v_empty[sv]);  // V_j is only read by dP_j
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < nkt && ok && !*abort_flag; ++j) {
        if (j + 1 < nkt && !issue_s(j + 1)) {
          ok = false;
          break;
        }
        trace_mark(a, tr, 2, j, 0);
        if (!mbar_wait(p_full, j & 1, a.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int sk = j % NSK;
        const uint32_t k0 = smem_u32(sm + L::K_OFF + sk * L::KT);
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk)
          umma_bf16(t_dq, sdesc_sw128(dsa + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                    sdesc_sw128(k0 + kk * 2048, 16384, 1024), ID_Q, (j | kk) != 0);
        umma_commit(&k_empty[sk]);
        umma_commit(p_done);
        trace_mark(a, tr, 2, j, 1);
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // warpgroup: key columns [64*half, 64*half + 64)
    const int c0 = half * 64;
    const int r = quad * 32 + lane;
    const int qr = q0 + r;
    const uint32_t lo = (uint32_t)(quad * 32) << 16;
    const long li = ((long)b * a.nq + h) * a.S + qr;
    const float L2 = a.lse[li] * LOG2E, Dr = a.Dv[li];
    bool ok = true;
    for (int j = 0; j < nkt; ++j) {
      const bool trw = tr && warp == 2 && lane == 0;
      trace_mark(a, trw, 3, j, 0);
      if (*abort_flag || !mbar_wait(s_full, j & 1, a.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      trace_mark(a, trw, 3, j, 1);
      // S first; the dP loads then overlap the exponentials
      uint32_t sr[2][32], dr[2][32];
#pragma unroll
      for (int i = 0; i < 2; ++i) tmem_ld32_async(t_s + lo + c0 + 32 * i, sr[i]);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 2; ++i) tmem_regs(sr[i]);
#pragma unroll
      for (int i = 0; i < 2; ++i) tmem_ld32_async(t_dp + lo + c0 + 32 * i, dr[i]);
      const bool diag = j == nkt - 1;  // the last key tile is the diagonal one
      float p[64];
#pragma unroll
      for (int cc = 0; cc < 64; ++cc) {
        {
          const float xe = fmaf(__uint_as_float(sr[cc >> 5][cc & 31]), a.scale_log2, -L2);
          p[cc] = ex2_approx(xe);
        }
        if (diag && j * BKV + c0 + cc > qr) p[cc] = 0.f;
      }
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 2; ++i) tmem_regs(dr[i]);
      trace_mark(a, trw, 3, j, 2);
      tc_fence_before();
      mbar_arrive(s_empty);
      uint32_t pd[32];
#pragma unroll
      for (int c = 0; c < 64; c += 2)
        pd[c / 2] = pack_bf16x2(p[c] * (__uint_as_float(dr[c >> 5][c & 31]) - Dr),
                                p[c + 1] * (__uint_as_float(dr[(c + 1) >> 5][(c + 1) & 31]) - Dr));
      trace_mark(a, trw, 3, j, 3);
      // the dS buffer was last read by the dQ MMAs of key tile j - 1
      if (j > 0 && !mbar_wait(p_done, (j - 1) & 1, a.err)) {
        ok = false;
        break;
      }
      trace_mark(a, trw, 3, j, 4);
      store_row64(sm + L::DS_OFF + half * 16384, r, pd);
      fence_proxy_async_smem();
      mbar_arrive(p_full);
      trace_mark(a, trw, 3, j, 5);
    }
    if (ok && mbar_wait(p_done, (nkt - 1) & 1, a.err)) {
      tc_fence_after();
      const long ld = (long)(a.nq + 2 * a.nkv) * HD;
      __nv_bfloat16* gq = a.dqkv + ((long)row0 + qr) * ld + h * HD;
#pragma unroll 1
      for (int c = half * (HD / 2); c < (half + 1) * (HD / 2); c += 32) {
        float dq[32];
        tmem_ld32(t_dq + lo + c, dq);
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 w;
          w.x = pack_bf16x2(dq[i] * a.scale, dq[i + 1] * a.scale);
          w.y = pack_bf16x2(dq[i + 2] * a.scale, dq[i + 3] * a.scale);
          w.z = pack_bf16x2(dq[i + 4] * a.scale, dq[i + 5] * a.scale);
          w.w = pack_bf16x2(dq[i + 6] * a.scale, dq[i + 7] * a.scale);
          *reinterpret_cast<uint4*>(gq + c + i) = w;
        }
      }
    } else {
      *abort_flag = 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

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

static CUtensorMap map2d(const void* base, long rows, long cols, int box_rows) {
  static thread_local bool bound = false;
  if (!bound) {
    DTB_CUDA(cudaFree(nullptr));  // bind the primary context on this (autograd) thread
    bound = true;
  }
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  DTB_CHECK(r == CUDA_SUCCESS, "attention backward tensor map encode failed (%d)", (int)r);
  return m;
}

template <int HD>
void bwd_tc_launch(const torch::Tensor& qkv, const torch::Tensor& dO, const float* lse, const float* Dv,
                   torch::Tensor& dqkv, int B, int S, int nq, int nkv, float scale) {
  const long rows = (long)B * S, cols = (long)(nq + 2 * nkv) * HD, ocols = (long)nq * HD;
  const CUtensorMap kv128 = map2d(qkv.data_ptr(), rows, cols, 128);
  const CUtensorMap q64 = map2d(qkv.data_ptr(), rows, cols, 64);
  const CUtensorMap do64 = map2d(dO.data_ptr(), rows, ocols, 64);
  const CUtensorMap do128 = map2d(dO.data_ptr(), rows, ocols, 128);
  static bool cfg = false;
  if (!cfg) {
    DTB_CUDA(cudaFuncSetAttribute(attn_bwd_dkdv_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  SmKV<HD>::TOTAL));
    DTB_CUDA(cudaFuncSetAttribute(attn_bwd_dq_tc_kernel<HD, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  SmQ<HD, 3>::TOTAL));
    DTB_CUDA(cudaFuncSetAttribute(attn_bwd_dq_tc_kernel<HD, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  SmQ<HD, 4>::TOTAL));
    DTB_CUDA(cudaFuncSetAttribute(attn_bwd_dq128_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  SmQ128<HD>::TOTAL));
    cfg = true;
  }
  // dQ key tile: 128 unless DTB_ATTN_DQ_BKV=64
  static const bool dq128 = [] {
    const char* e = getenv("DTB_ATTN_DQ_BKV");
    return !(e != nullptr && e[0] == '6');
  }();
  // K/V ring depth of the dQ kernel: 4 unless DTB_ATTN_DQ_STAGES=3
  static const int dq_stages = [] {
    const char* e = getenv("DTB_ATTN_DQ_STAGES");
    return (e != nullptr && e[0] == '3') ? 3 : 4;
  }();
  static const bool trace_on = [] {
    const char* e = getenv("DTB_ATTN_TRACE");
    return e != nullptr && e[0] == '1';
  }();
  torch::Tensor trace;
  if (trace_on) trace = torch::zeros({4 * 64 * 8}, qkv.options().dtype(at::kLong));
  // dK/dV TMEM kernel issue order (see attn_bwd_dkdv_tm_kernel): DTB_ATTN_DKDV_EARLY_S=1
  static const int early_s = [] {
    const char* e = getenv("DTB_ATTN_DKDV_EARLY_S");
    return (e != nullptr && e[0] == '1') ? 1 : 0;
  }();
  BwdArgs args{lse, Dv, reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), S, nq, nkv, scale, scale * LOG2E,
               dtb_error_word(), trace_on ? reinterpret_cast<long long*>(trace.data_ptr<int64_t>()) : nullptr,
               early_s};
  auto st = at::cuda::getCurrentCUDAStream();
  // dK/dV: 128-query tiles with P^T / dS^T in TMEM unless DTB_ATTN_DKDV_TM=0
  static const bool dkdv_tm = [] {
    const char* e = getenv("DTB_ATTN_DKDV_TM");
    return !(e != nullptr && e[0] == '0');
  }();
  if (dkdv_tm) {
    static bool cfg_tm = false;
    if (!cfg_tm) {
      DTB_CUDA(cudaFuncSetAttribute(attn_bwd_dkdv_tm_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    SmKVT<HD>::TOTAL));
      cfg_tm = true;
    }
    attn_bwd_dkdv_tm_kernel<HD><<<dim3(nkv * B, S / 128, 1), 320, SmKVT<HD>::TOTAL, st>>>(kv128, kv128, do128, args);
  } else {
    attn_bwd_dkdv_tc_kernel<HD><<<dim3(nkv * B, S / 128, 1), 320, SmKV<HD>::TOTAL, st>>>(kv128, q64, do64, args);
  }
  DTB_LAUNCH_CHECK();
  if (dq128)
    attn_bwd_dq128_tc_kernel<HD><<<dim3(nq * B, S / 128, 1), 320, SmQ128<HD>::TOTAL, st>>>(kv128, do128, kv128, args);
  else if (dq_stages == 3)
    attn_bwd_dq_tc_kernel<HD, 3><<<dim3(nq * B, S / 128, 1), 320, SmQ<HD, 3>::TOTAL, st>>>(kv128, do128, q64, args);
  else
    attn_bwd_dq_tc_kernel<HD, 4><<<dim3(nq * B, S / 128, 1), 320, SmQ<HD, 4>::TOTAL, st>>>(kv128, do128, q64, args);
  DTB_LAUNCH_CHECK();
  if (trace_on) {
    // diagnostic: per-iteration phase times (SM cycles) of the dQ kernel's first CTA
    auto h = trace.cpu();
    const int64_t* t = h.data_ptr<int64_t>();
    const int64_t t0 = t[(1 * 64 + 0) * 8 + 0];
    fprintf(stderr, "[dtb] dQ trace (cycles from the first S issue): producer(empty,issue) "
                    "mma(kvwait,kvdone,sempty | pwait,pdone) elementwise(start,sfull,ldissued,lddone,computed,stored)\n");
    for (int j = 0; j < 64; ++j) {
      auto v = [&](int role, int k) { const int64_t x = t[(role * 64 + j) * 8 + k]; return x ? x - t0 : -1; };
      if (!t[(3 * 64 + j) * 8 + 0]) break;
      fprintf(stderr, "[dtb] j=%2d P %7lld %7lld | S %7lld %7lld %7lld | G %7lld %7lld | E %7lld %7lld %7lld %7lld %7lld %7lld\n", j,
              (long long)v(0, 0), (long long)v(0, 1), (long long)v(1, 0), (long long)v(1, 1), (long long)v(1, 2),
              (long long)v(2, 0), (long long)v(2, 1), (long long)v(3, 0), (long long)v(3, 1), (long long)v(3, 2),
              (long long)v(3, 3), (long long)v(3, 4), (long long)v(3, 5));
    }
  }
}

}  // namespace fab
}  // namespace dtb

// dK/dV and dQ on tcgen05 (D = rowsum(dO*O) already in Dv).  Returns false
// when the shape is not covered (then the caller uses the mma.sync kernels).
bool attn_bwd_tc(const torch::Tensor& dO, const torch::Tensor& qkv, const float* lse, const float* Dv,
                 torch::Tensor& dqkv, int64_t B, int64_t S, int64_t nq, int64_t nkv, int64_t hd, double scale) {
  if (S % 128 != 0 || (hd != 64 && hd != 128)) return false;
  if (hd == 128)
    dtb::fab::bwd_tc_launch<128>(qkv, dO, lse, Dv, dqkv, (int)B, (int)S, (int)nq, (int)nkv, (float)scale);
  else
    dtb::fab::bwd_tc_launch<64>(qkv, dO, lse, Dv, dqkv, (int)B, (int)S, (int)nq, (int)nkv, (float)scale);
  return true;
}
