// Causal GQA flash-attention forward on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA), sm_100a.
//
// One CTA per (128-row query tile, head, batch); 10 warps:
//   warp 0     TMA producer: the Q tile once, then K and V tiles (128 keys)
//              into 2-deep rings, straight from the packed qkv projection;
//   warp 1     owns TMEM (512 columns: two 128-column S buffers + the O
//              accumulator) and one thread issues the MMAs:
//                S_j = Q K_j^T   (M=128, N=128, K=hd; both operands K-major)
//                O  += P_j V_j   (M=128, N=hd,  K=128; V is MN-major)
//              S_{j+1} is computed while the softmax warps work on S_j;
//   warps 2-9  softmax, two threads per query row: warps w and w+4 read the
//              same TMEM lanes (32*(w%4)..+31 = query rows), warp w columns
//              [0, 64) of S and warp w+4 columns [64, 128) (and the matching
//              halves of O).  Each thread reads its 64 scores with two
//              tcgen05.ld and one wait, applies the causal mask (diagonal tile
//              only), takes its half-row maximum and swaps it with its partner
//              through shared memory (a 64-thread named barrier per row
//              quarter), then runs the online softmax in exp2 form with the
//              scale folded into one FFMA.  One exponential in four is
//              evaluated on the FMA pipes (exp2_fma, common.cuh) instead of
//              the special-function unit (measured: 617 TFLOP/s at b1 s4096
//              h32 hd128; moving half of them, or the bf16 rounding, to the
//              FMA/integer pipes was slower, 549).  P_j goes in bf16 to one of two shared-memory
//              buffers in the 128-byte-swizzled K-major layout the MMA reads
//              (each thread writes one 64-column atom of its row); with two P
//              buffers the softmax of tile j only waits for the PV product of
//              tile j-2, so it runs concurrently with PV_{j-1} and S_{j+1}.
//              At the end the partners add their partial row sums, normalise
//              their halves of O and write them with the log-sum-exp.
//
// O is rescaled only when a row's running maximum grows by more than 8 (in
// log2 units): until then P = exp2(s - m_stale) <= 2^8, which fp32 and bf16
// hold exactly as well, and the final 1/l uses the same stale maximum, so
// the result is the same softmax.  A rescale waits for PV_{j-1} first.
//
// Every mbarrier wait is bounded (common.cuh); no TMA multicast.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include "common.cuh"

namespace dtb {
namespace fa {

constexpr float LOG2E = 1.4426950408889634f;
constexpr int BM = 128, BN = 128;
constexpr float RESCALE_THRESHOLD = 8.f;
constexpr int SOFTMAX_THREADS = 256;   // warps 2-9
constexpr int NTHREADS = 64 + SOFTMAX_THREADS;



__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

template <int HD>
struct Smem {
  static constexpr int Q_BYTES = BM * HD * 2;           // [hd/64 atoms][128 rows][128 B]
  static constexpr int K_BYTES = BN * HD * 2;
  static constexpr int V_BYTES = BN * HD * 2;           // [2 kv chunks][hd/64][64 rows][128 B]
  static constexpr int P_BYTES = BM * BN * 2;           // [2 atoms][128 rows][128 B]
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + Q_BYTES;         // 2 stages
  static constexpr int V_OFF = K_OFF + 2 * K_BYTES;     // 2 stages
  static constexpr int P_OFF = V_OFF + 2 * V_BYTES;   // 2 buffers
  static constexpr int X_OFF = P_OFF + 2 * P_BYTES;     // [2 halves][128 rows] fp32 partner exchange
  static constexpr int BAR_OFF = X_OFF + 2 * BM * 4;
  static constexpr int N_BARS = 22;
  static constexpr int TOTAL = BAR_OFF + N_BARS * 8 + 16 + 1024;
  static_assert(TOTAL <= 232448, "shared memory per CTA");
};

struct FwdArgs {
  __nv_bfloat16* out;
  float* lse;
  int S, nq, nkv;
  float scale_log2;
  int* err;
};

template <int HD>
__global__ void __launch_bounds__(NTHREADS, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_qk, const __grid_constant__ CUtensorMap tm_v,
                       const FwdArgs a) {
  using L = Smem<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;     // [2]
  uint64_t* k_empty = bars + 3;    // [2]
  uint64_t* s_full = bars + 5;     // [2]
  uint64_t* s_empty = bars + 7;    // [2]
  uint64_t* p_full = bars + 9;     // [2]: P_j written into buffer j & 1
  uint64_t* o_done = bars + 11;    // [2]: PV_j (read P buffer j & 1) finished
  uint64_t* v_full = bars + 13;    // [2]
  uint64_t* v_empty = bars + 15;   // [2]
  uint64_t* x_bar = bars + 17;     // [4]: the two softmax threads of each row quarter (64 arrivals)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + L::N_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = a.S / BM;
  // grid (heads x batch, query tiles): blocks start in linear order, so every
  // head's longest rows start before any head's shorter ones (longest first
  // over the whole grid, which shortens the last wave of this causal workload)
  const int qb = nqb - 1 - blockIdx.y;
  const int h = blockIdx.x % a.nq, b = blockIdx.x / a.nq;
  const int hk = h / (a.nq / a.nkv);
  const int nkb = qb + 1;               // kv tiles 0..qb (causal, BN == BM)
  const int row0 = b * a.S;             // first packed row of this sequence

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], SOFTMAX_THREADS);
      mbar_init(&p_full[i], SOFTMAX_THREADS);
      mbar_init(&o_done[i], 1);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&x_bar[i], 64);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_qk);
    tma_prefetch_desc(&tm_v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint32_t t_s[2] = {tmem, tmem + 128};
  const uint32_t t_o = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      // Q tile: hd/64 boxes of [128 rows x 64]
      mbar_arrive_expect_tx(q_full, L::Q_BYTES);
#pragma unroll
      for (int c = 0; c < HD / 64; ++c)
        tma_load_2d(sm + L::Q_OFF + c * 16384, &tm_qk, q_full, h * HD + c * 64, row0 + qb * BM);
      // K and V rings are separate: K_{j} only waits for S_{j-2} to finish,
      // not for the PV product that still reads V_{j-2}
      for (int j = 0; j < nkb; ++j) {
        const int st = j & 1;
        const uint32_t par = ((j >> 1) & 1) ^ 1;
        if (*abort_flag || !mbar_wait(&k_empty[st], par, a.err)) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&k_full[st], L::K_BYTES);
        uint8_t* sk = sm + L::K_OFF + st * L::K_BYTES;
        uint8_t* sv = sm + L::V_OFF + st * L::V_BYTES;
#pragma unroll
        for (int c = 0; c < HD / 64; ++c)
          tma_load_2d(sk + c * 16384, &tm_qk, &k_full[st], (a.nq + hk) * HD + c * 64, row0 + j * BN);
        if (*abort_flag || !mbar_wait(&v_empty[st], par, a.err)) {
          *abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&v_full[st], L::V_BYTES);
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
          for (int c = 0; c < HD / 64; ++c)
            tma_load_2d(sv + i * (HD / 64) * 8192 + c * 8192, &tm_v, &v_full[st], (a.nq + a.nkv + hk) * HD + c * 64,
                        row0 + j * BN + i * 64);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_S = idesc_bf16(BM, BN, false, false);
      constexpr uint32_t ID_O = idesc_bf16(BM, HD, false, true);
      const uint32_t q0 = smem_u32(sm + L::Q_OFF);
      const uint32_t p0 = smem_u32(sm + L::P_OFF);
      bool ok = mbar_wait(q_full, 0, a.err);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(&k_full[st], (j >> 1) & 1, a.err)) return false;
        if (!mbar_wait(&s_empty[st], ((j >> 1) & 1) ^ 1, a.err)) return false;
        tc_fence_after();
        const uint32_t k0 = smem_u32(sm + L::K_OFF + st * L::K_BYTES);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_bf16(t_s[st], sdesc_sw128(q0 + off, 16, 1024), sdesc_sw128(k0 + off, 16, 1024), ID_S, kk != 0);
        }
        umma_commit(&s_full[st]);
        umma_commit(&k_empty[st]);
        return true;
      };
      // S runs two tiles ahead of PV
      if (ok) ok = issue_s(0);
      if (ok && nkb > 1) ok = issue_s(1);
      for (int j = 0; j < nkb && ok && !*abort_flag; ++j) {
        // P_j written (and O rescaled if needed) by the softmax warps
        const int pb = j & 1;
        if (!mbar_wait(&p_full[pb], (j >> 1) & 1, a.err)) {
          ok = false;
          break;
        }
        const int st = j & 1;
        if (!mbar_wait(&v_full[st], (j >> 1) & 1, a.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t v0 = smem_u32(sm + L::V_OFF + st * L::V_BYTES);
        const uint32_t pj = p0 + pb * L::P_BYTES;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint32_t pa = pj + (kk >> 2) * 16384 + (kk & 3) * 32;
          const uint32_t vb = v0 + (kk >> 2) * (HD / 64) * 8192 + (kk & 3) * 2048;
          umma_bf16(t_o, sdesc_sw128(pa, 16, 1024), sdesc_sw128(vb, 8192, 1024), ID_O, (j | kk) != 0);
        }
        umma_commit(&v_empty[st]);
        umma_commit(&o_done[pb]);
        if (j + 2 < nkb && !issue_s(j + 2)) {
          ok = false;
          break;
        }
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ------------------------------------------------------------ softmax warps
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;        // 0: columns [0, 64), 1: [64, 128)
    const int r = quad * 32 + lane;          // row within the tile == TMEM lane
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const int c0 = half * 64;                // first S column of this thread
    float* xch = reinterpret_cast<float*>(sm + L::X_OFF);
    float m_used = -INFINITY, l = 0.f;       // running max (log2 units) and this half's sum
    bool ok = true;
    // rendezvous of the two threads of a row (bounded: a partner that left on an
    // error makes this time out instead of hanging)
    uint32_t xphase = 0;
    auto xsync = [&]() -> bool {
      mbar_arrive(&x_bar[quad]);
      const bool r2 = mbar_wait(&x_bar[quad], xphase, a.err);
      xphase ^= 1;
      return r2;
    };
    for (int j = 0; j < nkb; ++j) {
      const int st = j & 1;
      if (*abort_flag || !mbar_wait(&s_full[st], (j >> 1) & 1, a.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[2][32];
#pragma unroll
      for (int c = 0; c < 2; ++c) tmem_ld32_async(t_s[st] + lane_off + c0 + c * 32, sr[c]);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 2; ++c) tmem_regs(sr[c]);
      tc_fence_before();
      mbar_arrive(&s_empty[st]);  // S buffer free for S_{j+2}
      float sv[64];
#pragma unroll
      for (int c = 0; c < 64; ++c) sv[c] = __uint_as_float(sr[c >> 5][c & 31]);
      if (j == qb) {
        // diagonal tile: key column c is visible to query row r iff c <= r
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (c0 + c > r) sv[c] = -INFINITY;
      }
      float mx4[4] = {sv[0], sv[1], sv[2], sv[3]};
#pragma unroll
      for (int c = 4; c < 64; c += 4) {
#pragma unroll
        for (int i = 0; i < 4; ++i) mx4[i] = fmaxf(mx4[i], sv[c + i]);
      }
      float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      // swap half-row maxima with the partner (same rows, other columns)
      xch[half * BM + r] = mx;
      if (!xsync()) {
        ok = false;
        *abort_flag = 1;
        break;
      }
      mx = fmaxf(mx, xch[(half ^ 1) * BM + r]) * a.scale_log2;
      if (!xsync()) {  // both read before the next write
        ok = false;
        *abort_flag = 1;
        break;
      }
      float alpha = 1.f;
      bool rescale = false;
      if (mx > m_used + RESCALE_THRESHOLD) {
        alpha = (m_used == -INFINITY) ? 0.f : exp2f(m_used - mx);
        rescale = (m_used != -INFINITY);
        m_used = mx;
      }
      // p = 2^(s * scale*log2e - m): one FFMA and one exponential per element,
      // every fourth pair of columns on the FMA pipes
      const float neg_m = -m_used;
      float rs4[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        const float x0 = fmaf(sv[c], a.scale_log2, neg_m), x1 = fmaf(sv[c + 1], a.scale_log2, neg_m);
        float p0, p1;
        if ((c & 6) == 6) {
          p0 = exp2_fma(x0);
          p1 = exp2_fma(x1);
        } else {
          p0 = ex2_approx(x0);
          p1 = ex2_approx(x1);
        }
        rs4[(c >> 1) & 3] += p0 + p1;
        pk[c / 2] = pack_bf16x2(p0, p1);
      }
      l = l * alpha + ((rs4[0] + rs4[1]) + (rs4[2] + rs4[3]));
      if (__any_sync(0xffffffffu, rescale)) {
        // O holds PV_0..PV_{j-1}: wait for the last of them, then scale this half
        if (j > 0) {
          if (!mbar_wait(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1, a.err)) ok = false;
          tc_fence_after();
        }
        if (ok) {
          const float f = rescale ? alpha : 1.f;
#pragma unroll 1
          for (int c = half * (HD / 2); c < (half + 1) * (HD / 2); c += 32) {
            float o[32];
            tmem_ld32(t_o + lane_off + c, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= f;
            tmem_st32(t_o + lane_off + c, o);
          }
          tmem_st_wait();
        }
      }
      // P buffer j & 1 was last read by PV_{j-2}
      if (ok && j > 1 && !mbar_wait(&o_done[j & 1], ((j - 2) >> 1) & 1, a.err)) ok = false;
      if (!ok) {
        *abort_flag = 1;
        break;
      }
      // this half of P row r -> its 64-column atom, 16-byte chunks XOR-swizzled by (r % 8)
      uint8_t* P = sm + L::P_OFF + (j & 1) * L::P_BYTES + half * 16384 + r * 128;
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        uint4 v;
        v.x = pk[cc * 4 + 0];
        v.y = pk[cc * 4 + 1];
        v.z = pk[cc * 4 + 2];
        v.w = pk[cc * 4 + 3];
        *reinterpret_cast<uint4*>(P + ((cc ^ (r & 7)) << 4)) = v;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[j & 1]);
    }
    if (ok && mbar_wait(&o_done[(nkb - 1) & 1], ((nkb - 1) >> 1) & 1, a.err)) {
      tc_fence_after();
      // row sum = half 0 + half 1, the same order in both partners
      xch[half * BM + r] = l;
      if (!xsync()) *abort_flag = 1;
      const float lt = xch[r] + xch[BM + r];
      const float inv = 1.f / lt;
      const long orow = (long)row0 + qb * BM + r;
      __nv_bfloat16* op = a.out + orow * (long)a.nq * HD + h * HD;
#pragma unroll 1
      for (int c = half * (HD / 2); c < (half + 1) * (HD / 2); c += 32) {
        float o[32];
        tmem_ld32(t_o + lane_off + c, o);
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 w;
          w.x = pack_bf16x2(o[i] * inv, o[i + 1] * inv);
          w.y = pack_bf16x2(o[i + 2] * inv, o[i + 3] * inv);
          w.z = pack_bf16x2(o[i + 4] * inv, o[i + 5] * inv);
          w.w = pack_bf16x2(o[i + 6] * inv, o[i + 7] * inv);
          *reinterpret_cast<uint4*>(op + c + i) = w;
        }
      }
      if (half == 0) a.lse[((long)b * a.nq + h) * a.S + qb * BM + r] = (m_used + log2f(lt)) / LOG2E;
    } else {
      *abort_flag = 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ============================================================== two query tiles per CTA
// attn_fwd_pp_kernel: one CTA per (pair of adjacent 128-row query tiles, head,
// batch), so the two tiles share every K/V load and, more importantly, each
// tile's softmax runs while the tensor cores work on the other tile:
//   warp 0     TMA: Q_A, Q_B once; K_j into a 2-deep ring, V_j into one stage
//   warp 1     TMEM (S_A, S_B: 128 columns each; O_A, O_B: hd each) and MMAs
//              in the order S_A(0) S_B(0) | PV_A(j) S_A(j+1) PV_B(j) S_B(j+1) ...
//   warps 2-5  softmax of tile A (thread = query row, 128 scores), warps 6-9 of
//              tile B.  P_X goes to one bf16 shared buffer per tile; the
//              softmax of tile X at step j writes it once PV_X(j-1) has read it.
// Tile A = 2*pair, tile B = 2*pair + 1: B has one more key tile (its diagonal).
// Registers: a 10-warp block is allocated registers as 12 warps (warpgroup
// granularity), so the cap is 168 per thread, not 65536 / 320; a larger cap
// compiles but fails to launch.
// Same online softmax as attn_fwd_tc_kernel (exp2 form, stale-max rescale).
template <int HD>
struct SmemPP {
  static constexpr int Q_BYTES = BM * HD * 2;
  static constexpr int K_BYTES = BN * HD * 2;
  static constexpr int V_BYTES = BN * HD * 2;
  static constexpr int P_BYTES = BM * BN * 2;
  static constexpr int Q_OFF = 0;                         // Q_A, Q_B
  static constexpr int K_OFF = Q_OFF + 2 * Q_BYTES;       // 2 stages
  static constexpr int V_OFF = K_OFF + 2 * K_BYTES;       // 1 stage
  static constexpr int P_OFF = V_OFF + V_BYTES;           // P_A, P_B
  static constexpr int BAR_OFF = P_OFF + 2 * P_BYTES;
  static constexpr int N_BARS = 16;
  static constexpr int TOTAL = BAR_OFF + N_BARS * 8 + 16 + 1024;
  static_assert(TOTAL <= 232448, "shared memory per CTA");
};

template <int HD>
__global__ void __launch_bounds__(320, 1)
    attn_fwd_pp_kernel(const __grid_constant__ CUtensorMap tm_qk, const __grid_constant__ CUtensorMap tm_v,
                       const FwdArgs a) {
  using L = SmemPP<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;     // [2]
  uint64_t* k_empty = bars + 3;    // [2]
  uint64_t* v_full = bars + 5;
  uint64_t* v_empty = bars + 6;
  uint64_t* s_full = bars + 7;     // [2 tiles]
  uint64_t* p_full = bars + 9;     // [2 tiles]
  uint64_t* pv_done = bars + 11;   // [2 tiles]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + L::N_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int npairs = a.S / (2 * BM);
  const int pr = npairs - 1 - blockIdx.y;  // longest rows first over the whole grid
  const int h = blockIdx.x % a.nq, b = blockIdx.x / a.nq;
  const int hk = h / (a.nq / a.nkv);
  const int qb0 = 2 * pr;                  // tile A; tile B = qb0 + 1
  const int nkb_a = qb0 + 1, nkb_b = qb0 + 2;
  const int row0 = b * a.S;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(v_full, 1);
    mbar_init(v_empty, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_qk);
    tma_prefetch_desc(&tm_v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint32_t t_s[2] = {tmem, tmem + 128};
  const uint32_t t_o[2] = {tmem + 256, tmem + 256 + HD};

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, 2 * L::Q_BYTES);
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int c = 0; c < HD / 64; ++c)
          tma_load_2d(sm + L::Q_OFF + t * L::Q_BYTES + c * 16384, &tm_qk, q_full, h * HD + c * 64,
                      row0 + (qb0 + t) * BM);
      auto load_k = [&](int j) -> bool {
        const int st = j & 1;
        if (*abort_flag || !mbar_wait(&k_empty[st], ((j >> 1) & 1) ^ 1, a.err)) return false;
        mbar_arrive_expect_tx(&k_full[st], L::K_BYTES);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c)
          tma_load_2d(sm + L::K_OFF + st * L::K_BYTES + c * 16384, &tm_qk, &k_full[st], (a.nq + hk) * HD + c * 64,
                      row0 + j * BN);
        return true;
      };
      bool ok = load_k(0);
      for (int j = 0; j < nkb_b && ok; ++j) {
        if (*abort_flag || !mbar_wait(v_empty, (j & 1) ^ 1, a.err)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(v_full, L::V_BYTES);
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
          for (int c = 0; c < HD / 64; ++c)
            tma_load_2d(sm + L::V_OFF + i * (HD / 64) * 8192 + c * 8192, &tm_v, v_full,
                        (a.nq + a.nkv + hk) * HD + c * 64, row0 + j * BN + i * 64);
        if (j + 1 < nkb_b) ok = load_k(j + 1);
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_S = idesc_bf16(BM, BN, false, false);
      constexpr uint32_t ID_O = idesc_bf16(BM, HD, false, true);
      const uint32_t q0 = smem_u32(sm + L::Q_OFF);
      const uint32_t p0 = smem_u32(sm + L::P_OFF);
      const uint32_t v0 = smem_u32(sm + L::V_OFF);
      bool ok = mbar_wait(q_full, 0, a.err);
      auto issue_s = [&](int t, int j) -> bool {  // S_t(j) = Q_t K_j^T
        const int st = j & 1;
        if (!mbar_wait(&k_full[st], (j >> 1) & 1, a.err)) return false;
        tc_fence_after();
        const uint32_t k0 = smem_u32(sm + L::K_OFF + st * L::K_BYTES);
        const uint32_t qt = q0 + t * L::Q_BYTES;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_bf16(t_s[t], sdesc_sw128(qt + off, 16, 1024), sdesc_sw128(k0 + off, 16, 1024), ID_S, kk != 0);
        }
        umma_commit(&s_full[t]);
        // K_j is done once tile B (the later user, or the only one past tile A's end) has it
        if (t == 1 || j >= nkb_a) umma_commit(&k_empty[st]);
        return true;
      };
      auto issue_pv = [&](int t, int j) -> bool {  // O_t += P_t V_j
        if (!mbar_wait(&p_full[t], j & 1, a.err)) return false;
        tc_fence_after();
        const uint32_t pt = p0 + t * L::P_BYTES;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint32_t pa = pt + (kk >> 2) * 16384 + (kk & 3) * 32;
          const uint32_t vb = v0 + (kk >> 2) * (HD / 64) * 8192 + (kk & 3) * 2048;
          umma_bf16(t_o[t], sdesc_sw128(pa, 16, 1024), sdesc_sw128(vb, 8192, 1024), ID_O, (j | kk) != 0);
        }
        umma_commit(&pv_done[t]);
        return true;
      };
      if (ok) ok = issue_s(0, 0);
      if (ok) ok = issue_s(1, 0);
      for (int j = 0; j < nkb_b && ok && !*abort_flag; ++j) {
        if (!mbar_wait(v_full, j & 1, a.err)) {
          ok = false;
          break;
        }
        if (j < nkb_a) {
          if (!issue_pv(0, j)) {
            ok = false;
            break;
          }
          if (j + 1 < nkb_a && !issue_s(0, j + 1)) {
            ok = false;
            break;
          }
        }
        if (!issue_pv(1, j)) {
          ok = false;
          break;
        }
        umma_commit(v_empty);  // V_j read by both tiles' products
        if (j + 1 < nkb_b && !issue_s(1, j + 1)) {
          ok = false;
          break;
        }
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ------------------------------------------------------------ softmax warps
    const int t = (warp - 2) >> 2;           // 0: tile A, 1: tile B
    const int quad = warp & 3;
    const int r = quad * 32 + lane;          // row within the tile == TMEM lane
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const int qb = qb0 + t;
    const int nkb = t == 0 ? nkb_a : nkb_b;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkb; ++j) {
      if (*abort_flag || !mbar_wait(&s_full[t], j & 1, a.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32_async(t_s[t] + lane_off + c * 32, sr[c]);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_regs(sr[c]);
      float sv[BN];
#pragma unroll
      for (int c = 0; c < BN; ++c) sv[c] = __uint_as_float(sr[c >> 5][c & 31]);
      if (j == qb) {
#pragma unroll
        for (int c = 0; c < BN; ++c)
          if (c > r) sv[c] = -INFINITY;
      }
      float mx4[4] = {sv[0], sv[1], sv[2], sv[3]};
#pragma unroll
      for (int c = 4; c < BN; c += 4) {
#pragma unroll
        for (int i = 0; i < 4; ++i) mx4[i] = fmaxf(mx4[i], sv[c + i]);
      }
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * a.scale_log2;
      float alpha = 1.f;
      bool rescale = false;
      if (mx > m_used + RESCALE_THRESHOLD) {
        alpha = (m_used == -INFINITY) ? 0.f : exp2f(m_used - mx);
        rescale = (m_used != -INFINITY);
        m_used = mx;
      }
      const float neg_m = -m_used;
      float rs4[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pk[BN / 2];
#pragma unroll
      for (int c = 0; c < BN; c += 2) {
        const float x0 = fmaf(sv[c], a.scale_log2, neg_m), x1 = fmaf(sv[c + 1], a.scale_log2, neg_m);
        float p0, p1;
        if ((c & 6) == 6) {
          p0 = exp2_fma(x0);
          p1 = exp2_fma(x1);
        } else {
          p0 = ex2_approx(x0);
          p1 = ex2_approx(x1);
        }
        rs4[(c >> 1) & 3] += p0 + p1;
        pk[c / 2] = pack_bf16x2(p0, p1);
      }
      l = l * alpha + ((rs4[0] + rs4[1]) + (rs4[2] + rs4[3]));
      // PV_t(j-1) must be done before O is rescaled and before P_t is rewritten
      if (j > 0) {
        if (!mbar_wait(&pv_done[t], (j - 1) & 1, a.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      if (__any_sync(0xffffffffu, rescale)) {
        const float f = rescale ? alpha : 1.f;
#pragma unroll 1
        for (int c = 0; c < HD; c += 32) {
          float o[32];
          tmem_ld32(t_o[t] + lane_off + c, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= f;
          tmem_st32(t_o[t] + lane_off + c, o);
        }
        tmem_st_wait();
      }
      uint8_t* P = sm + L::P_OFF + t * L::P_BYTES;
#pragma unroll
      for (int ch = 0; ch < BN / 8; ++ch) {
        const int atom = ch >> 3, cc = ch & 7;
        uint4 v;
        v.x = pk[ch * 4 + 0];
        v.y = pk[ch * 4 + 1];
        v.z = pk[ch * 4 + 2];
        v.w = pk[ch * 4 + 3];
        *reinterpret_cast<uint4*>(P + atom * 16384 + r * 128 + ((cc ^ (r & 7)) << 4)) = v;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[t]);
    }
    if (ok && mbar_wait(&pv_done[t], (nkb - 1) & 1, a.err)) {
      tc_fence_after();
      const float inv = 1.f / l;
      const long orow = (long)row0 + qb * BM + r;
      __nv_bfloat16* op = a.out + orow * (long)a.nq * HD + h * HD;
#pragma unroll 1
      for (int c = 0; c < HD; c += 32) {
        float o[32];
        tmem_ld32(t_o[t] + lane_off + c, o);
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 w;
          w.x = pack_bf16x2(o[i] * inv, o[i + 1] * inv);
          w.y = pack_bf16x2(o[i + 2] * inv, o[i + 3] * inv);
          w.z = pack_bf16x2(o[i + 4] * inv, o[i + 5] * inv);
          w.w = pack_bf16x2(o[i + 6] * inv, o[i + 7] * inv);
          *reinterpret_cast<uint4*>(op + c + i) = w;
        }
      }
      a.lse[((long)b * a.nq + h) * a.S + qb * BM + r] = (m_used + log2f(l)) / LOG2E;
    } else {
      *abort_flag = 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// ============================================================== two query tiles, P in TMEM
// attn_fwd_ws_kernel: one CTA per (pair of adjacent 128-row query tiles, head,
// batch), like attn_fwd_pp_kernel, with P kept in tensor memory:
//   warp 0     TMA: Q_A, Q_B once; K_j and V_j into separate 2-deep rings
//   warp 1     TMEM S_A [0,128) | S_B [128,256) | O_A [256, 256+hd) | O_B [256+hd, 256+2hd)
//              and the MMAs, in the order S_A(0) S_B(0) | PV_A(j) S_A(j+1) PV_B(j)
//              S_B(j+1) | ...; PV reads P from TMEM as its A operand, so there is
//              no shared-memory P buffer and V gets a second stage
//   warps 2-5  softmax of tile A, warps 6-9 of tile B (thread = query row): two
//              passes over the row's 128 scores, 32 columns at a time (row maximum,
//              then exp2, row sum and P), so no thread holds the whole row; P goes
//              back as bf16 pairs (score k in column k/2) into the first 64 columns
//              of the tile's own S region, over scores the thread has already read
// Ordering: S_X(j+1) overwrites P_X(j) only after PV_X(j) has read it (the tensor
// pipe runs in issue order), and s_full_X(j) completes only after PV_X(j-1) (a
// commit tracks every earlier MMA of the thread), so the softmax may rescale O_X
// as soon as S_X(j) is there.  Same online softmax as attn_fwd_tc_kernel.
template <int HD>
struct SmemWS {
  static constexpr int Q_BYTES = BM * HD * 2;
  static constexpr int K_BYTES = BN * HD * 2;
  static constexpr int V_BYTES = BN * HD * 2;
  static constexpr int Q_OFF = 0;                         // Q_A, Q_B
  static constexpr int K_OFF = Q_OFF + 2 * Q_BYTES;       // 2 stages
  static constexpr int V_OFF = K_OFF + 2 * K_BYTES;       // 2 stages
  static constexpr int BAR_OFF = V_OFF + 2 * V_BYTES;
  static constexpr int N_BARS = 16;
  static constexpr int TOTAL = BAR_OFF + N_BARS * 8 + 16 + 1024;
  static_assert(TOTAL <= 232448, "shared memory per CTA");
};

__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

template <int HD>
__global__ void __launch_bounds__(320, 1)
    attn_fwd_ws_kernel(const __grid_constant__ CUtensorMap tm_qk, const __grid_constant__ CUtensorMap tm_v,
                       const FwdArgs a) {
  using L = SmemWS<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;     // [2 stages]
  uint64_t* k_empty = bars + 3;    // [2 stages]
  uint64_t* v_full = bars + 5;     // [2 stages]
  uint64_t* v_empty = bars + 7;    // [2 stages]
  uint64_t* s_full = bars + 9;     // [2 tiles]
  uint64_t* p_full = bars + 11;    // [2 tiles]
  uint64_t* pv_done = bars + 13;   // [2 tiles]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + L::N_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int npairs = a.S / (2 * BM);
  const int pr = npairs - 1 - blockIdx.y;  // longest rows first over the whole grid
  const int h = blockIdx.x % a.nq, b = blockIdx.x / a.nq;
  const int hk = h / (a.nq / a.nkv);
  const int qb0 = 2 * pr;                  // tile A; tile B = qb0 + 1
  const int nkb_a = qb0 + 1, nkb_b = qb0 + 2;
  const int row0 = b * a.S;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&pv_done[i], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_qk);
    tma_prefetch_desc(&tm_v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint32_t t_s[2] = {tmem, tmem + 128};
  const uint32_t t_o[2] = {tmem + 256, tmem + 256 + HD};

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, 2 * L::Q_BYTES);
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int c = 0; c < HD / 64; ++c)
          tma_load_2d(sm + L::Q_OFF + t * L::Q_BYTES + c * 16384, &tm_qk, q_full, h * HD + c * 64,
                      row0 + (qb0 + t) * BM);
      bool ok = true;
      for (int j = 0; j < nkb_b && ok; ++j) {
        const int st = j & 1;
        const uint32_t par = ((j >> 1) & 1) ^ 1;
        if (*abort_flag || !mbar_wait(&k_empty[st], par, a.err)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&k_full[st], L::K_BYTES);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c)
          tma_load_2d(sm + L::K_OFF + st * L::K_BYTES + c * 16384, &tm_qk, &k_full[st], (a.nq + hk) * HD + c * 64,
                      row0 + j * BN);
        if (*abort_flag || !mbar_wait(&v_empty[st], par, a.err)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&v_full[st], L::V_BYTES);
        uint8_t* sv = sm + L::V_OFF + st * L::V_BYTES;
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
          for (int c = 0; c < HD / 64; ++c)
            tma_load_2d(sv + i * (HD / 64) * 8192 + c * 8192, &tm_v, &v_full[st], (a.nq + a.nkv + hk) * HD + c * 64,
                        row0 + j * BN + i * 64);
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_S = idesc_bf16(BM, BN, false, false);
      constexpr uint32_t ID_O = idesc_bf16(BM, HD, false, true);
      const uint32_t q0 = smem_u32(sm + L::Q_OFF);
      bool ok = mbar_wait(q_full, 0, a.err);
      auto issue_s = [&](int t, int j) -> bool {  // S_t(j) = Q_t K_j^T
        const int st = j & 1;
        if (!mbar_wait(&k_full[st], (j >> 1) & 1, a.err)) return false;
        tc_fence_after();
        const uint32_t k0 = smem_u32(sm + L::K_OFF + st * L::K_BYTES);
        const uint32_t qt = q0 + t * L::Q_BYTES;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_bf16(t_s[t], sdesc_sw128(qt + off, 16, 1024), sdesc_sw128(k0 + off, 16, 1024), ID_S, kk != 0);
        }
        umma_commit(&s_full[t]);
        // K_j is done once tile B (its later user, or its only one past tile A's last key tile) has it
        if (t == 1 || j >= nkb_a) umma_commit(&k_empty[st]);
        return true;
      };
      auto issue_pv = [&](int t, int j) -> bool {  // O_t += P_t V_j, P_t from TMEM
        if (!mbar_wait(&p_full[t], j & 1, a.err)) return false;
        tc_fence_after();
        const uint32_t v0 = smem_u32(sm + L::V_OFF + (j & 1) * L::V_BYTES);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint32_t vb = v0 + (kk >> 2) * (HD / 64) * 8192 + (kk & 3) * 2048;
          umma_bf16_ta(t_o[t], t_s[t] + 8 * kk, sdesc_sw128(vb, 8192, 1024), ID_O, (j | kk) != 0);
        }
        umma_commit(&pv_done[t]);
        return true;
      };
      if (ok) ok = issue_s(0, 0);
      if (ok) ok = issue_s(1, 0);
      for (int j = 0; j < nkb_b && ok && !*abort_flag; ++j) {
        if (!mbar_wait(&v_full[j & 1], (j >> 1) & 1, a.err)) {
          ok = false;
          break;
        }
        if (j < nkb_a) {
          if (!issue_pv(0, j)) {
            ok = false;
            break;
          }
          if (j + 1 < nkb_a && !issue_s(0, j + 1)) {
            ok = false;
            break;
          }
        }
        if (!issue_pv(1, j)) {
          ok = false;
          break;
        }
        umma_commit(&v_empty[j & 1]);  // V_j read by both tiles' products
        if (j + 1 < nkb_b && !issue_s(1, j + 1)) {
          ok = false;
          break;
        }
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ------------------------------------------------------------ softmax warps
    const int t = (warp - 2) >> 2;           // 0: tile A, 1: tile B
    const int quad = warp & 3;
    const int r = quad * 32 + lane;          // row within the tile == TMEM lane
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t ts = t_s[t] + lane_off;
    const int qb = qb0 + t;
    const int nkb = t == 0 ? nkb_a : nkb_b;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkb; ++j) {
      if (*abort_flag || !mbar_wait(&s_full[t], j & 1, a.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool diag = j == qb;             // causal mask: column c > row r on the diagonal tile
      // pass 1: row maximum
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t ra[32], rb[32];
        tmem_ld32_async(ts + 64 * half, ra);
        tmem_ld32_async(ts + 64 * half + 32, rb);
        tmem_wait_ld();
        tmem_regs(ra);
        tmem_regs(rb);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int ca = 64 * half + i, cb = ca + 32;
          const float va = (diag && ca > r) ? -INFINITY : __uint_as_float(ra[i]);
          const float vb = (diag && cb > r) ? -INFINITY : __uint_as_float(rb[i]);
          mx4[i & 3] = fmaxf(mx4[i & 3], fmaxf(va, vb));
        }
      }
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * a.scale_log2;
      float alpha = 1.f;
      bool rescale = false;
      if (mx > m_used + RESCALE_THRESHOLD) {
        alpha = (m_used == -INFINITY) ? 0.f : exp2f(m_used - mx);
        rescale = (m_used != -INFINITY);
        m_used = mx;
      }
      // O_t is not being written: PV_t(j-1) finished before S_t(j) (s_full)
      if (__any_sync(0xffffffffu, rescale)) {
        const float f = rescale ? alpha : 1.f;
#pragma unroll 1
        for (int c = 0; c < HD; c += 32) {
          float o[32];
          tmem_ld32(t_o[t] + lane_off + c, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= f;
          tmem_st32(t_o[t] + lane_off + c, o);
        }
        tmem_st_wait();
      }
      // pass 2: P = exp2(s * scale_log2 - m) in bf16 over columns [16 cc, 16 cc + 16)
      const float neg_m = -m_used;
      float rs4[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t rc[2][32];
      tmem_ld32_async(ts, rc[0]);
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        tmem_wait_ld();
        tmem_regs(rc[cc & 1]);
        if (cc < 3) tmem_ld32_async(ts + 32 * (cc + 1), rc[(cc + 1) & 1]);
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const int c = 32 * cc + i;
          float p0 = 0.f, p1 = 0.f;
          const float x0 = fmaf(__uint_as_float(rc[cc & 1][i]), a.scale_log2, neg_m);
          const float x1 = fmaf(__uint_as_float(rc[cc & 1][i + 1]), a.scale_log2, neg_m);
          if ((c & 6) == 6) {
            p0 = exp2_fma(x0);
            p1 = exp2_fma(x1);
          } else {
            p0 = ex2_approx(x0);
            p1 = ex2_approx(x1);
          }
          if (diag && c > r) p0 = 0.f;
          if (diag && c + 1 > r) p1 = 0.f;
          rs4[(i >> 1) & 3] += p0 + p1;
          pk[i >> 1] = pack_bf16x2(p0, p1);
        }
        tmem_st16u(ts + 16 * cc, pk);
      }
      tmem_st_wait();
      l = l * alpha + ((rs4[0] + rs4[1]) + (rs4[2] + rs4[3]));
      tc_fence_before();
      mbar_arrive(&p_full[t]);
    }
    if (ok && mbar_wait(&pv_done[t], (nkb - 1) & 1, a.err)) {
      tc_fence_after();
      const float inv = 1.f / l;
      const long orow = (long)row0 + qb * BM + r;
      __nv_bfloat16* op = a.out + orow * (long)a.nq * HD + h * HD;
#pragma unroll 1
      for (int c = 0; c < HD; c += 32) {
        float o[32];
        tmem_ld32(t_o[t] + lane_off + c, o);
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 w;
          w.x = pack_bf16x2(o[i] * inv, o[i + 1] * inv);
          w.y = pack_bf16x2(o[i + 2] * inv, o[i + 3] * inv);
          w.z = pack_bf16x2(o[i + 4] * inv, o[i + 5] * inv);
          w.w = pack_bf16x2(o[i + 6] * inv, o[i + 7] * inv);
          *reinterpret_cast<uint4*>(op + c + i) = w;
        }
      }
      a.lse[((long)b * a.nq + h) * a.S + qb * BM + r] = (m_used + log2f(l)) / LOG2E;
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

static CUtensorMap qkv_map(const void* base, long rows, long cols, int box_rows) {
  static thread_local bool bound = false;
  if (!bound) {
    DTB_CUDA(cudaFree(nullptr));  // the encode is a driver call: bind the primary context on this thread
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
  DTB_CHECK(r == CUDA_SUCCESS, "attention tensor map encode failed (%d)", (int)r);
  return m;
}

// Two query tiles per CTA only when DTB_ATTN_FWD_PP=1: measured at b1 s4096 h32
// hd128 it ran at 523 TFLOP/s against 604 for one tile per CTA (its softmax
// threads spill at the 168-register cap, and the single P buffer and V stage
// per tile serialize more than the second tile overlaps).
static bool pp_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("DTB_ATTN_FWD_PP");
    v = (e != nullptr && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

// Two query tiles per CTA with P in tensor memory (attn_fwd_ws_kernel) only when
// DTB_ATTN_FWD_WS=1: built, not yet timed on a B200.
static bool ws_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("DTB_ATTN_FWD_WS");
    v = (e != nullptr && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

template <int HD>
void fwd_tc_launch(const torch::Tensor& qkv, torch::Tensor& o, torch::Tensor& lse, int B, int S, int nq, int nkv,
                   float scale) {
  using L = Smem<HD>;
  const long rows = (long)B * S, cols = (long)(nq + 2 * nkv) * HD;
  const CUtensorMap tqk = qkv_map(qkv.data_ptr(), rows, cols, 128);
  const CUtensorMap tv = qkv_map(qkv.data_ptr(), rows, cols, 64);
  if (S % (2 * BM) == 0 && ws_enabled()) {
    using LW = SmemWS<HD>;
    static bool cfg_ws = false;
    if (!cfg_ws) {
      DTB_CUDA(cudaFuncSetAttribute(attn_fwd_ws_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, LW::TOTAL));
      cfg_ws = true;
    }
    FwdArgs args{reinterpret_cast<__nv_bfloat16*>(o.data_ptr()), lse.data_ptr<float>(), S, nq, nkv, scale * LOG2E,
                 dtb_error_word()};
    attn_fwd_ws_kernel<HD><<<dim3(nq * B, S / (2 * BM), 1), 320, LW::TOTAL, at::cuda::getCurrentCUDAStream()>>>(tqk, tv,
                                                                                                            args);
    DTB_LAUNCH_CHECK();
    return;
  }
  if (S % (2 * BM) == 0 && pp_enabled()) {
    using LP = SmemPP<HD>;
    static bool cfg_pp = false;
    if (!cfg_pp) {
      DTB_CUDA(cudaFuncSetAttribute(attn_fwd_pp_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, LP::TOTAL));
      cfg_pp = true;
    }
    FwdArgs args{reinterpret_cast<__nv_bfloat16*>(o.data_ptr()), lse.data_ptr<float>(), S, nq, nkv, scale * LOG2E,
                 dtb_error_word()};
    attn_fwd_pp_kernel<HD><<<dim3(nq * B, S / (2 * BM), 1), 320, LP::TOTAL, at::cuda::getCurrentCUDAStream()>>>(tqk, tv,
                                                                                                            args);
    DTB_LAUNCH_CHECK();
    return;
  }
  static bool cfg = false;
  if (!cfg) {
    DTB_CUDA(cudaFuncSetAttribute(attn_fwd_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL));
    cfg = true;
  }
  FwdArgs args{reinterpret_cast<__nv_bfloat16*>(o.data_ptr()), lse.data_ptr<float>(), S, nq, nkv, scale * LOG2E,
               dtb_error_word()};
  attn_fwd_tc_kernel<HD><<<dim3(nq * B, S / BM, 1), NTHREADS, L::TOTAL, at::cuda::getCurrentCUDAStream()>>>(tqk, tv,
                                                                                                        args);
  DTB_LAUNCH_CHECK();
}

}  // namespace fa
}  // namespace dtb

// Used by attn_fwd when head_dim is 64/128 and seq_len % 128 == 0.
bool attn_fwd_tc(const torch::Tensor& qkv, torch::Tensor& o, torch::Tensor& lse, int64_t B, int64_t S, int64_t nq,
                 int64_t nkv, int64_t hd, double scale) {
  if (S % 128 != 0 || (hd != 64 && hd != 128)) return false;
  const c10::cuda::CUDAGuard g(qkv.device());
  if (hd == 128) dtb::fa::fwd_tc_launch<128>(qkv, o, lse, (int)B, (int)S, (int)nq, (int)nkv, (float)scale);
  else dtb::fa::fwd_tc_launch<64>(qkv, o, lse, (int)B, (int)S, (int)nq, (int)nkv, (float)scale);
  return true;
}
