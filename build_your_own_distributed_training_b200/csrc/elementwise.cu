// Memory-bound kernels of the training step (sm_100a): RMSNorm forward and
// backward, RoPE (inverse rotation for the backward), SwiGLU backward, token
// embedding forward/backward, fused cross-entropy (loss + logit gradient in
// one pass), AdamW on flat fp32 shards, and sum of squares.
//
// All reductions run in a fixed order (per-block partials reduced by one
// block), so every kernel here is bit-reproducible run to run.  Math uses
// fp32 throughout with bf16 storage; exponentials go through expf / exp2f.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"

namespace dtb {

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  if (w == 0) {
    t = l < NT / 32 ? red[l] : 0.f;
    t = warp_sum(t);
    if (l == 0) red[0] = t;
  }
  __syncthreads();
  return red[0];
}

template <int NT>
__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    float t = l < NT / 32 ? red[l] : -INFINITY;
    t = warp_max(t);
    if (l == 0) red[0] = t;
  }
  __syncthreads();
  return red[0];
}

// ---------------------------------------------------------------- RMSNorm
// One CTA per row; rows of D bf16 read as 16-byte vectors.
template <typename WT, int NT>
__global__ void __launch_bounds__(NT) rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const WT* __restrict__ w,
                                                        __nv_bfloat16* __restrict__ y, float* __restrict__ rstd,
                                                        int D, float eps) {
  __shared__ float red[32];
  const long row = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * D);
  const int nv = D / 8;
  float ss = 0.f;
  for (int i = threadIdx.x; i < nv; i += NT) {
    uint4 q = xr[i];
    const uint32_t* u = &q.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 f = unpack_bf16x2(u[k]);
      ss += f.x * f.x + f.y * f.y;
    }
  }
  const float r = rsqrtf(block_sum<NT>(ss, red) / (float)D + eps);
  if (threadIdx.x == 0) rstd[row] = r;
  uint4* yr = reinterpret_cast<uint4*>(y + row * D);
  for (int i = threadIdx.x; i < nv; i += NT) {
    uint4 q = xr[i];
    uint32_t* u = &q.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 f = unpack_bf16x2(u[k]);
      const int c = i * 8 + 2 * k;
      u[k] = pack_bf16x2(f.x * r * to_f(w[c]), f.y * r * to_f(w[c + 1]));
    }
    yr[i] = q;
  }
}

// 8 consecutive weights as fp32
__device__ __forceinline__ void load_w8(const float* w, int c, float (&o)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(w + c), b = *reinterpret_cast<const float4*>(w + c + 4);
  o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}
__device__ __forceinline__ void load_w8(const __nv_bfloat16* w, int c, float (&o)[8]) {
  const uint4 q = *reinterpret_cast<const uint4*>(w + c);
  const uint32_t* u = &q.x;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 f = unpack_bf16x2(u[k]);
    o[2 * k] = f.x;
    o[2 * k + 1] = f.y;
  }
}

// Forward with the row in registers: two warps per row (4 rows per CTA);
// thread t of a row holds its 16-byte vectors t, t+64, ..., so the row is read
// once; the sum of squares is two warp reductions and one CTA barrier.
// D = 512 * VPL.
template <typename WT, int VPL>
__global__ void __launch_bounds__(256) rmsnorm_fwd_rows_kernel(const __nv_bfloat16* __restrict__ x,
                                                               const WT* __restrict__ w,
                                                               __nv_bfloat16* __restrict__ y,
                                                               float* __restrict__ rstd, int M, float eps) {
  constexpr int D = 512 * VPL;
  __shared__ float wsum[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rl = warp >> 1;                      // row within the CTA
  const int t = (warp & 1) * 32 + lane;          // thread within the row
  const long row = (long)blockIdx.x * 4 + rl;
  const bool valid = row < M;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * D);
  uint4 q[VPL];
  float ss = 0.f;
  if (valid) {
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      q[i] = xr[t + 64 * i];
      const uint32_t* u = &q[i].x;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = unpack_bf16x2(u[k]);
        ss += f.x * f.x + f.y * f.y;
      }
    }
  }
  ss = warp_sum(ss);
  if (lane == 0) wsum[warp] = ss;
  __syncthreads();
  if (!valid) return;
  const float r = rsqrtf((wsum[2 * rl] + wsum[2 * rl + 1]) / (float)D + eps);
  if (t == 0) rstd[row] = r;
  uint4* yr = reinterpret_cast<uint4*>(y + row * D);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    float wv[8];
    load_w8(w, (t + 64 * i) * 8, wv);
    uint32_t* u = &q[i].x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = unpack_bf16x2(u[k]);
      u[k] = pack_bf16x2(f.x * r * wv[2 * k], f.y * r * wv[2 * k + 1]);
    }
    yr[t + 64 * i] = q[i];
  }
}

// Backward with registers: thread t owns columns 8(t + 256j) .. +8 (j < VPT,
// D = 2048 * VPT); the weights and the dw partial sums stay in registers for
// all the CTA's rows and each row of x and dy is read once.  Same arithmetic
// and row order as rmsnorm_bwd_kernel, so the dw partials are identical.
template <typename WT, int VPT>
__global__ void __launch_bounds__(256) rmsnorm_bwd_rows_kernel(const __nv_bfloat16* __restrict__ dy,
                                                               const __nv_bfloat16* __restrict__ x,
                                                               const WT* __restrict__ w,
                                                               const float* __restrict__ rstd,
                                                               __nv_bfloat16* __restrict__ dx, float* __restrict__ part,
                                                               int M, int rows_per_cta) {
  constexpr int D = 2048 * VPT;
  __shared__ float red[32];
  const int t = threadIdx.x;
  float wv[VPT][8], dw[VPT][8];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    load_w8(w, (t + 256 * j) * 8, wv[j]);
#pragma unroll
    for (int k = 0; k < 8; ++k) dw[j][k] = 0.f;
  }
  const int r0 = blockIdx.x * rows_per_cta;
  const int r1 = min(M, r0 + rows_per_cta);
  // row r's loads are issued while row r-1 is reduced (two rows in flight)
  uint4 nx[VPT], ng[VPT];
  float nrs = 0.f;
  if (r0 < r1) {
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      nx[j] = reinterpret_cast<const uint4*>(x + (long)r0 * D)[t + 256 * j];
      ng[j] = reinterpret_cast<const uint4*>(dy + (long)r0 * D)[t + 256 * j];
    }
    nrs = rstd[r0];
  }
  for (int row = r0; row < r1; ++row) {
    uint4 qx[VPT], qg[VPT];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      qx[j] = nx[j];
      qg[j] = ng[j];
    }
    const float rs = nrs;
    if (row + 1 < r1) {
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        nx[j] = reinterpret_cast<const uint4*>(x + (long)(row + 1) * D)[t + 256 * j];
        ng[j] = reinterpret_cast<const uint4*>(dy + (long)(row + 1) * D)[t + 256 * j];
      }
      nrs = rstd[row + 1];
    }
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const uint32_t *ux = &qx[j].x, *ug = &qg[j].x;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 fx = unpack_bf16x2(ux[k]), fg = unpack_bf16x2(ug[k]);
        dot += fg.x * wv[j][2 * k] * fx.x * rs + fg.y * wv[j][2 * k + 1] * fx.y * rs;
      }
    }
    const float mean = block_sum<256>(dot, red) / (float)D;
    uint4* dr = reinterpret_cast<uint4*>(dx + (long)row * D);
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const uint32_t *ux = &qx[j].x, *ug = &qg[j].x;
      uint4 qo;
      uint32_t* uo = &qo.x;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 fx = unpack_bf16x2(ux[k]), fg = unpack_bf16x2(ug[k]);
        const float xh0 = fx.x * rs, xh1 = fx.y * rs;
        uo[k] = pack_bf16x2(rs * (fg.x * wv[j][2 * k] - xh0 * mean), rs * (fg.y * wv[j][2 * k + 1] - xh1 * mean));
        dw[j][2 * k] += fg.x * xh0;
        dw[j][2 * k + 1] += fg.y * xh1;
      }
      dr[t + 256 * j] = qo;
    }
  }
#pragma unroll
  for (int j = 0; j < VPT; ++j)
#pragma unroll
    for (int k = 0; k < 8; ++k) part[(long)blockIdx.x * D + (t + 256 * j) * 8 + k] = dw[j][k];
}

// dx = rstd * (g*w - xhat * mean(g*w*xhat)); per-CTA partial of sum(g*xhat)
// over its rows written to part[blockIdx.x, :].
template <typename WT, int NT>
__global__ void __launch_bounds__(NT) rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                                        const __nv_bfloat16* __restrict__ x, const WT* __restrict__ w,
                                                        const float* __restrict__ rstd, __nv_bfloat16* __restrict__ dx,
                                                        float* __restrict__ part, int M, int D, int rows_per_cta) {
  __shared__ float red[32];
  extern __shared__ float dw_s[];  // [D]
  for (int c = threadIdx.x; c < D; c += NT) dw_s[c] = 0.f;
  __syncthreads();
  const int nv = D / 8;
  const int r0 = blockIdx.x * rows_per_cta;
  const int r1 = min(M, r0 + rows_per_cta);
  for (int row = r0; row < r1; ++row) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + (long)row * D);
    const uint4* gr = reinterpret_cast<const uint4*>(dy + (long)row * D);
    const float rs = rstd[row];
    float dot = 0.f;
    for (int i = threadIdx.x; i < nv; i += NT) {
      uint4 qx = xr[i], qg = gr[i];
      const uint32_t *ux = &qx.x, *ug = &qg.x;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float2 fx = unpack_bf16x2(ux[k]), fg = unpack_bf16x2(ug[k]);
        const int c = i * 8 + 2 * k;
        dot += fg.x * to_f(w[c]) * fx.x * rs + fg.y * to_f(w[c + 1]) * fx.y * rs;
      }
    }
    const float mean = block_sum<NT>(dot, red) / (float)D;
    uint4* dr = reinterpret_cast<uint4*>(dx + (long)row * D);
    for (int i = threadIdx.x; i < nv; i += NT) {
      uint4 qx = xr[i], qg = gr[i], qo;
      const uint32_t *ux = &qx.x, *ug = &qg.x;
      uint32_t* uo = &qo.x;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float2 fx = unpack_bf16x2(ux[k]), fg = unpack_bf16x2(ug[k]);
        const int c = i * 8 + 2 * k;
        const float xh0 = fx.x * rs, xh1 = fx.y * rs;
        uo[k] = pack_bf16x2(rs * (fg.x * to_f(w[c]) - xh0 * mean), rs * (fg.y * to_f(w[c + 1]) - xh1 * mean));
        dw_s[c] += fg.x * xh0;
        dw_s[c + 1] += fg.y * xh1;
      }
      dr[i] = qo;
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += NT) part[(long)blockIdx.x * D + c] = dw_s[c];
}

// acc[c] += sum_b part[b, c] in a fixed order: block = 8 warps x 32 columns;
// warp w sums parts w, w+8, w+16, ... (one coalesced 128-byte row segment per
// load), then the 8 warp sums are added in warp order.
__global__ void __launch_bounds__(256) reduce_partials_kernel(const float* __restrict__ part, float* __restrict__ acc,
                                                              int nparts, int D) {
  __shared__ float red[8][32];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int c = blockIdx.x * 32 + l;
  float s = 0.f;
  if (c < D)
    for (int b = w; b < nparts; b += 8) s += part[(long)b * D + c];
  red[w][l] = s;
  __syncthreads();
  if (w == 0 && c < D) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += red[i][l];
    acc[c] += t;
  }
}

// ---------------------------------------------------------------- RoPE
// In place on x[M, ld]: for every head h < rope_cols/hd, rotate the pair
// (j, j+hd/2) by angle table (cos, sign*sin)[pos].
__global__ void rope_kernel(__nv_bfloat16* __restrict__ x, long ld, const float* __restrict__ cos_t,
                            const float* __restrict__ sin_t, int M, int rope_cols, int hd, int seqlen, float sign) {
  const int half = hd >> 1;
  const long total = (long)M * (rope_cols / 2);
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long row = i / (rope_cols / 2);
    const int p = (int)(i % (rope_cols / 2));
    const int head = p / half, j = p % half;
    const int pos = (int)(row % seqlen);
    __nv_bfloat16* b = x + row * ld + head * hd;
    const float x1 = __bfloat162float(b[j]), x2 = __bfloat162float(b[j + half]);
    const float c = cos_t[(long)pos * hd + j], s = sign * sin_t[(long)pos * hd + j];
    b[j] = __float2bfloat16_rn(x1 * c - x2 * s);
    b[j + half] = __float2bfloat16_rn(x2 * c + x1 * s);
  }
}

// Same rotation, eight consecutive pairs per thread with 16-byte accesses
// (half-head a multiple of 8 and rows 16-byte aligned; the host checks).
__global__ void rope_vec8_kernel(__nv_bfloat16* __restrict__ x, long ld, const float* __restrict__ cos_t,
                                 const float* __restrict__ sin_t, int M, int rope_cols, int hd, int seqlen,
                                 float sign) {
  const int half = hd >> 1;
  const int groups = rope_cols / 16;  // 8-pair groups per row
  const long total = (long)M * groups;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long row = i / groups;
    const int p = (int)(i % groups) * 8;
    const int head = p / half, j = p % half;
    const int pos = (int)(row % seqlen);
    __nv_bfloat16* b = x + row * ld + head * hd;
    uint4 q1 = *reinterpret_cast<const uint4*>(b + j), q2 = *reinterpret_cast<const uint4*>(b + j + half);
    float c[8], sn[8];
    load_w8(cos_t + (long)pos * hd, j, c);
    load_w8(sin_t + (long)pos * hd, j, sn);
    uint32_t *u1 = &q1.x, *u2 = &q2.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 a = unpack_bf16x2(u1[k]), bb = unpack_bf16x2(u2[k]);
      const float s0 = sign * sn[2 * k], s1 = sign * sn[2 * k + 1];
      u1[k] = pack_bf16x2(a.x * c[2 * k] - bb.x * s0, a.y * c[2 * k + 1] - bb.y * s1);
      u2[k] = pack_bf16x2(bb.x * c[2 * k] + a.x * s0, bb.y * c[2 * k + 1] + a.y * s1);
    }
    *reinterpret_cast<uint4*>(b + j) = q1;
    *reinterpret_cast<uint4*>(b + j + half) = q2;
  }
}

// ---------------------------------------------------------------- SwiGLU bwd
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ da, const __nv_bfloat16* __restrict__ gu,
                                  __nv_bfloat16* __restrict__ dgu, int M, int F) {
  const long total = (long)M * F / 2;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long row = (2 * i) / F;
    const int c = (int)((2 * i) % F);
    const float2 a = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(da + row * F + c));
    const float2 g = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(gu + row * 2L * F + c));
    const float2 u = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(gu + row * 2L * F + F + c));
    float dg[2], du[2];
    const float gg[2] = {g.x, g.y}, uu[2] = {u.x, u.y}, aa[2] = {a.x, a.y};
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float sg = 1.f / (1.f + expf(-gg[k]));
      const float silu = gg[k] * sg;
      dg[k] = aa[k] * uu[k] * sg * (1.f + gg[k] * (1.f - sg));
      du[k] = aa[k] * silu;
    }
    *reinterpret_cast<uint32_t*>(dgu + row * 2L * F + c) = pack_bf16x2(dg[0], dg[1]);
    *reinterpret_cast<uint32_t*>(dgu + row * 2L * F + F + c) = pack_bf16x2(du[0], du[1]);
  }
}

// Same arithmetic, eight elements per thread with 16-byte accesses (F % 8 == 0).
__global__ void swiglu_bwd_vec8_kernel(const __nv_bfloat16* __restrict__ da, const __nv_bfloat16* __restrict__ gu,
                                       __nv_bfloat16* __restrict__ dgu, int M, int F) {
  const int groups = F / 8;
  const long total = (long)M * groups;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long row = i / groups;
    const int c = (int)(i % groups) * 8;
    const uint4 qa = *reinterpret_cast<const uint4*>(da + row * F + c);
    const uint4 qg = *reinterpret_cast<const uint4*>(gu + row * 2L * F + c);
    const uint4 qu = *reinterpret_cast<const uint4*>(gu + row * 2L * F + F + c);
    const uint32_t *ua = &qa.x, *ug = &qg.x, *uu = &qu.x;
    uint4 og, ou;
    uint32_t *pg = &og.x, *pu = &ou.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 a = unpack_bf16x2(ua[k]), g = unpack_bf16x2(ug[k]), u = unpack_bf16x2(uu[k]);
      const float gg[2] = {g.x, g.y}, uv[2] = {u.x, u.y}, aa[2] = {a.x, a.y};
      float dg[2], du[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float sg = 1.f / (1.f + expf(-gg[e]));
        const float silu = gg[e] * sg;
        dg[e] = aa[e] * uv[e] * sg * (1.f + gg[e] * (1.f - sg));
        du[e] = aa[e] * silu;
      }
      pg[k] = pack_bf16x2(dg[0], dg[1]);
      pu[k] = pack_bf16x2(du[0], du[1]);
    }
    *reinterpret_cast<uint4*>(dgu + row * 2L * F + c) = og;
    *reinterpret_cast<uint4*>(dgu + row * 2L * F + F + c) = ou;
  }
}

// ---------------------------------------------------------------- embedding
template <typename WT, typename OT>
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ tok, const WT* __restrict__ w, OT* __restrict__ out,
                                     int D, int V, int* err) {
  const long row = blockIdx.x;
  long t = tok[row];
  if (t < 0 || t >= V) {
    if (threadIdx.x == 0) atomicExch(err, ERR_BAD_ARG);
    t = 0;
  }
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    const float v = to_f(w[t * D + c]);
    if constexpr (sizeof(OT) == 4) out[row * D + c] = v;
    else out[row * D + c] = __float2bfloat16_rn(v);
  }
}

// sorted ids + their original positions: CTA i handles segment starting at i.
__global__ void embedding_bwd_kernel(const int64_t* __restrict__ sorted_tok, const int64_t* __restrict__ order,
                                     const __nv_bfloat16* __restrict__ dout, float* __restrict__ acc, int M, int D,
                                     int V) {
  const int i = blockIdx.x;
  const int64_t t = sorted_tok[i];
  if (i > 0 && sorted_tok[i - 1] == t) return;
  if (t < 0 || t >= V) return;
  int end = i + 1;
  while (end < M && sorted_tok[end] == t) ++end;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float s = 0.f;
    for (int j = i; j < end; ++j) s += __bfloat162float(dout[order[j] * (long)D + c]);
    acc[t * (long)D + c] += s;
  }
}

// Stable sort of the token ids for the embedding backward, in one CTA: key =
// (id << shift) | position, so keys are unique and any correct sort is stable;
// bitonic network over a power-of-two padded shared-memory array (pads are
// 0xFFFFFFFF and sort last).  Ids outside [0, V) get the key of bucket V,
// which embedding_bwd_kernel skips.  Writes the sorted ids and their positions.
__global__ void __launch_bounds__(1024) sort_tokens_kernel(const int64_t* __restrict__ tok, int M, int V, int shift,
                                                           int npow2, int64_t* __restrict__ sorted_tok,
                                                           int64_t* __restrict__ order) {
  extern __shared__ uint32_t keys[];
  for (int i = threadIdx.x; i < npow2; i += blockDim.x) {
    uint32_t k = 0xFFFFFFFFu;
    if (i < M) {
      const int64_t t = tok[i];
      const uint32_t b = (t < 0 || t >= V) ? (uint32_t)V : (uint32_t)t;
      k = (b << shift) | (uint32_t)i;
    }
    keys[i] = k;
  }
  __syncthreads();
  for (int k = 2; k <= npow2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < npow2; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint32_t a = keys[i], b = keys[ixj];
          const bool ascending = (i & k) == 0;
          if ((a > b) == ascending) {
            keys[i] = b;
            keys[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  const uint32_t mask = (1u << shift) - 1u;
  for (int i = threadIdx.x; i < M; i += blockDim.x) {
    const uint32_t k = keys[i];
    const uint32_t b = k >> shift;
    sorted_tok[i] = (b == (uint32_t)V) ? (int64_t)-1 : (int64_t)b;
    order[i] = (int64_t)(k & mask);
  }
}

// ---------------------------------------------------------------- cross-entropy
// Per row: lse, loss_row = lse - x[label] (0 if ignored), and
// dlogits = (softmax - onehot) / n_valid  (n_valid from device memory).
template <int NT>
__global__ void __launch_bounds__(NT) ce_row_kernel(const float* __restrict__ logits, const int64_t* __restrict__ labels,
                                                   __nv_bfloat16* __restrict__ dlog, float* __restrict__ row_loss,
                                                   const int* __restrict__ n_valid, int V, long ignore) {
  __shared__ float red[32];
  const long row = blockIdx.x;
  const float* x = logits + row * V;
  const long lab = labels[row];
  float mx = -INFINITY;
  for (int c = threadIdx.x; c < V; c += NT) mx = fmaxf(mx, x[c]);
  mx = block_max<NT>(mx, red);
  float se = 0.f;
  for (int c = threadIdx.x; c < V; c += NT) se += expf(x[c] - mx);
  se = block_sum<NT>(se, red);
  const float lse = mx + logf(se);
  const bool valid = lab != ignore && lab >= 0 && lab < V;
  const int nv = *n_valid;
  const float inv_n = valid && nv > 0 ? 1.f / (float)nv : 0.f;
  __nv_bfloat16* d = dlog + row * V;
  for (int c = threadIdx.x; c < V; c += NT) {
    const float p = expf(x[c] - lse);
    d[c] = __float2bfloat16_rn((p - (c == lab ? 1.f : 0.f)) * inv_n);
  }
  if (threadIdx.x == 0) row_loss[row] = valid ? (lse - x[lab]) : 0.f;
}

__global__ void count_valid_kernel(const int64_t* __restrict__ labels, int M, long ignore, int V, int* out) {
  __shared__ int s;
  if (threadIdx.x == 0) s = 0;
  __syncthreads();
  int c = 0;
  for (int i = threadIdx.x; i < M; i += blockDim.x) c += (labels[i] != ignore && labels[i] >= 0 && labels[i] < V);
  atomicAdd(&s, c);  // integer: order does not matter
  __syncthreads();
  if (threadIdx.x == 0) *out = s;
}

// one CTA: fixed-order sum of row losses / n_valid
template <int NT>
__global__ void __launch_bounds__(NT) ce_finish_kernel(const float* __restrict__ row_loss, const int* __restrict__ n_valid,
                                                      float* __restrict__ loss, int M) {
  __shared__ float red[32];
  float s = 0.f;
  for (int i = threadIdx.x; i < M; i += NT) s += row_loss[i];
  s = block_sum<NT>(s, red);
  if (threadIdx.x == 0) {
    const int n = *n_valid;
    *loss = n > 0 ? s / (float)n : __int_as_float(0x7fc00000);
  }
}

// ---------------------------------------------------------------- AdamW
// Decoupled decay, bias-corrected moments (torch.optim.AdamW semantics).
// clip = [coef, finite] (device): the update is skipped when finite == 0.
__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, __nv_bfloat16* __restrict__ out, const float* __restrict__ clip,
                             long n, float lr, float b1, float b2, float eps, float wd, float bc1, float bc2_sqrt) {
  float coef = 1.f;
  if (clip != nullptr) {
    if (clip[1] == 0.f) return;
    coef = clip[0];
  }
  const float step = lr / bc1;
  const float decay = 1.f - lr * wd;
  auto upd = [&](float pi, float gi, float& mi, float& vi) {
    gi *= coef;
    pi *= decay;
    mi = b1 * mi + (1.f - b1) * gi;
    vi = b2 * vi + (1.f - b2) * gi * gi;
    return pi - step * mi / (sqrtf(vi) / bc2_sqrt + eps);
  };
  // 16-byte vectors when every pointer allows it, scalar tail / fallback
  const bool vec = ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(m) |
                     reinterpret_cast<uintptr_t>(v)) & 15) == 0 && (reinterpret_cast<uintptr_t>(out) & 7) == 0;
  long done = 0;
  if (vec) {
    const long nv = n / 4;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < nv; i += (long)gridDim.x * blockDim.x) {
      float4 pp = reinterpret_cast<const float4*>(p)[i], gg = reinterpret_cast<const float4*>(g)[i];
      float4 mm = reinterpret_cast<const float4*>(m)[i], vv = reinterpret_cast<const float4*>(v)[i];
      pp.x = upd(pp.x, gg.x, mm.x, vv.x);
      pp.y = upd(pp.y, gg.y, mm.y, vv.y);
      pp.z = upd(pp.z, gg.z, mm.z, vv.z);
      pp.w = upd(pp.w, gg.w, mm.w, vv.w);
      reinterpret_cast<float4*>(p)[i] = pp;
      reinterpret_cast<float4*>(m)[i] = mm;
      reinterpret_cast<float4*>(v)[i] = vv;
      uint2 o;
      o.x = pack_bf16x2(pp.x, pp.y);
      o.y = pack_bf16x2(pp.z, pp.w);
      reinterpret_cast<uint2*>(out)[i] = o;
    }
    done = nv * 4;
  }
  for (long i = done + blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    float mi = m[i], vi = v[i];
    const float pi = upd(p[i], g[i], mi, vi);
    m[i] = mi;
    v[i] = vi;
    p[i] = pi;
    out[i] = __float2bfloat16_rn(pi);
  }
}

// ---------------------------------------------------------------- sum of squares
// per-block partial sums of x^2: 16-byte loads, four independent accumulators
// per thread (64 bytes in flight), fixed grid and order -> deterministic
template <int NT>
__global__ void __launch_bounds__(NT) sumsq_part_kernel(const float* __restrict__ x, long n, float* __restrict__ part) {
  __shared__ float red[32];
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  // scalar head up to the first 16-byte boundary, float4 body, scalar tail
  const long head = min(n, (long)(((16 - (reinterpret_cast<uintptr_t>(x) & 15)) & 15) / 4));
  const long nv = (n - head) / 4;
  const float4* xv = reinterpret_cast<const float4*>(x + head);
  const long stride = (long)gridDim.x * NT;
  long i = blockIdx.x * (long)NT + threadIdx.x;
  for (; i + 3 * stride < nv; i += 4 * stride) {
    const float4 a = xv[i], b = xv[i + stride], c = xv[i + 2 * stride], d = xv[i + 3 * stride];
    s0 += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
    s1 += b.x * b.x + b.y * b.y + b.z * b.z + b.w * b.w;
    s2 += c.x * c.x + c.y * c.y + c.z * c.z + c.w * c.w;
    s3 += d.x * d.x + d.y * d.y + d.z * d.z + d.w * d.w;
  }
  for (; i < nv; i += stride) {
    const float4 a = xv[i];
    s0 += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
  }
  if (blockIdx.x == 0) {
    for (long t = threadIdx.x; t < head; t += NT) s1 += x[t] * x[t];
    for (long t = head + nv * 4 + threadIdx.x; t < n; t += NT) s1 += x[t] * x[t];
  }
  float s = block_sum<NT>((s0 + s1) + (s2 + s3), red);
  if (threadIdx.x == 0) part[blockIdx.x] = s;
}

template <int NT>
__global__ void __launch_bounds__(NT) sum_parts_kernel(const float* __restrict__ part, int n, float* __restrict__ out) {
  __shared__ float red[32];
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += NT) s += part[i];
  s = block_sum<NT>(s, red);
  if (threadIdx.x == 0) *out = s;
}

static int grid_for(long n, int nt) {
  long g = (n + nt - 1) / nt;
  return (int)std::max<long>(1, std::min<long>(g, 16L * device_sm_count()));
}

}  // namespace dtb

using namespace dtb;

static cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream(); }

// The register-resident forward for the usual widths (512 ... 8192); false
// when D needs the general kernel.
template <typename WT>
static bool rmsnorm_fwd_rows_t(const __nv_bfloat16* x, const WT* w, __nv_bfloat16* y, float* rstd, int M, int D,
                               float eps) {
  const dim3 grid((M + 3) / 4);
  auto st = cur_stream();
  switch (D) {
    case 512: rmsnorm_fwd_rows_kernel<WT, 1><<<grid, 256, 0, st>>>(x, w, y, rstd, M, eps); return true;
    case 1024: rmsnorm_fwd_rows_kernel<WT, 2><<<grid, 256, 0, st>>>(x, w, y, rstd, M, eps); return true;
    case 2048: rmsnorm_fwd_rows_kernel<WT, 4><<<grid, 256, 0, st>>>(x, w, y, rstd, M, eps); return true;
    case 3072: rmsnorm_fwd_rows_kernel<WT, 6><<<grid, 256, 0, st>>>(x, w, y, rstd, M, eps); return true;
    case 4096: rmsnorm_fwd_rows_kernel<WT, 8><<<grid, 256, 0, st>>>(x, w, y, rstd, M, eps); return true;
    case 5120: rmsnorm_fwd_rows_kernel<WT, 10><<<grid, 256, 0, st>>>(x, w, y, rstd, M, eps); return true;
    case 8192: rmsnorm_fwd_rows_kernel<WT, 16><<<grid, 256, 0, st>>>(x, w, y, rstd, M, eps); return true;
    default: return false;
  }
}

static bool rmsnorm_fwd_rows(const torch::Tensor& x, const torch::Tensor& w, torch::Tensor& y, torch::Tensor& rstd,
                             int M, int D, float eps) {
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  bool done;
  if (w.scalar_type() == at::kFloat)
    done = rmsnorm_fwd_rows_t(xp, w.data_ptr<float>(), yp, rstd.data_ptr<float>(), M, D, eps);
  else
    done = rmsnorm_fwd_rows_t(xp, reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), yp, rstd.data_ptr<float>(), M,
                              D, eps);
  if (done) DTB_LAUNCH_CHECK();
  return done;
}

std::vector<torch::Tensor> rmsnorm_fwd(torch::Tensor x, torch::Tensor w, double eps) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.is_contiguous(), "rmsnorm: bf16 [M,D]");
  const c10::cuda::CUDAGuard g(x.device());
  const int M = (int)x.size(0), D = (int)x.size(1);
  TORCH_CHECK(D % 8 == 0 && w.numel() == D, "rmsnorm: D % 8 == 0 and w[D]");
  auto y = torch::empty_like(x);
  auto rstd = torch::empty({M}, x.options().dtype(at::kFloat));
  if (M == 0) return {y, rstd};
  if (rmsnorm_fwd_rows(x, w, y, rstd, M, D, (float)eps)) return {y, rstd};
  if (w.scalar_type() == at::kFloat)
    rmsnorm_fwd_kernel<float, 256><<<M, 256, 0, cur_stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), w.data_ptr<float>(),
        reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), rstd.data_ptr<float>(), D, (float)eps);
  else
    rmsnorm_fwd_kernel<__nv_bfloat16, 256><<<M, 256, 0, cur_stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), rstd.data_ptr<float>(), D, (float)eps);
  DTB_LAUNCH_CHECK();
  return {y, rstd};
}

// Workspace-explicit form used by both the torch entry point and the
// allocation-free C entry point: part must hold ceil(M/rows_per_cta) * D floats.
void rmsnorm_bwd_launch(const __nv_bfloat16* dy, const __nv_bfloat16* x, const void* w, bool w_f32,
                        const float* rstd, __nv_bfloat16* dx, float* dw_acc, float* part, int M, int D,
                        int rows_per_cta, cudaStream_t st) {
  const int nb = (M + rows_per_cta - 1) / rows_per_cta;
  const size_t sh = (size_t)D * sizeof(float);
  const int vpt = D % 2048 == 0 ? D / 2048 : 0;
  if (vpt >= 1 && vpt <= 4) {
    // register-resident variant: same partials, one read of x and dy
#define DTB_RMS_BWD_ROWS(WT, V)                                                                                   \
  rmsnorm_bwd_rows_kernel<WT, V><<<nb, 256, 0, st>>>(dy, x, (const WT*)w, rstd, dx, part, M, rows_per_cta)
    if (w_f32) {
      if (vpt == 1) DTB_RMS_BWD_ROWS(float, 1); else if (vpt == 2) DTB_RMS_BWD_ROWS(float, 2);
      else if (vpt == 3) DTB_RMS_BWD_ROWS(float, 3); else DTB_RMS_BWD_ROWS(float, 4);
    } else {
      if (vpt == 1) DTB_RMS_BWD_ROWS(__nv_bfloat16, 1); else if (vpt == 2) DTB_RMS_BWD_ROWS(__nv_bfloat16, 2);
      else if (vpt == 3) DTB_RMS_BWD_ROWS(__nv_bfloat16, 3); else DTB_RMS_BWD_ROWS(__nv_bfloat16, 4);
    }
#undef DTB_RMS_BWD_ROWS
    reduce_partials_kernel<<<(D + 31) / 32, 256, 0, st>>>(part, dw_acc, nb, D);
    return;
  }
  if (w_f32)
    rmsnorm_bwd_kernel<float, 256><<<nb, 256, sh, st>>>(dy, x, (const float*)w, rstd, dx, part, M, D, rows_per_cta);
  else
    rmsnorm_bwd_kernel<__nv_bfloat16, 256><<<nb, 256, sh, st>>>(dy, x, (const __nv_bfloat16*)w, rstd, dx, part, M, D,
                                                                 rows_per_cta);
  reduce_partials_kernel<<<(D + 31) / 32, 256, 0, st>>>(part, dw_acc, nb, D);
}

int rmsnorm_bwd_rows_per_cta(int M) {
  // enough CTAs to fill the GPU, few enough partial rows to keep the reduce cheap
  return std::max(1, M / (device_sm_count() * 4));
}

torch::Tensor rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd, torch::Tensor dw_acc) {
  TORCH_CHECK(dy.is_contiguous() && x.is_contiguous() && dy.sizes() == x.sizes(), "rmsnorm_bwd: shapes");
  TORCH_CHECK(dw_acc.scalar_type() == at::kFloat && dw_acc.is_contiguous(), "rmsnorm_bwd: fp32 dw accumulator");
  TORCH_CHECK(((reinterpret_cast<uintptr_t>(dy.data_ptr()) | reinterpret_cast<uintptr_t>(x.data_ptr()) |
                reinterpret_cast<uintptr_t>(w.data_ptr())) & 15) == 0,
              "rmsnorm_bwd: dy, x and w must start on 16-byte boundaries");
  const c10::cuda::CUDAGuard g(x.device());
  const int M = (int)x.size(0), D = (int)x.size(1);
  TORCH_CHECK(D * 4 <= 48 * 1024, "rmsnorm_bwd: D up to 12288");
  auto dx = torch::empty_like(x);
  if (M == 0) return dx;
  const int rpc = rmsnorm_bwd_rows_per_cta(M);
  const int nb = (M + rpc - 1) / rpc;
  auto part = torch::empty({(long)nb * D}, x.options().dtype(at::kFloat));
  rmsnorm_bwd_launch(reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()),
                     reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), w.data_ptr(), w.scalar_type() == at::kFloat,
                     rstd.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), dw_acc.data_ptr<float>(),
                     part.data_ptr<float>(), M, D, rpc, cur_stream());
  DTB_LAUNCH_CHECK();
  return dx;
}

void rope_apply(torch::Tensor x, torch::Tensor cos_t, torch::Tensor sin_t, int64_t rope_cols, int64_t hd,
                int64_t seqlen, double sign) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.stride(1) == 1, "rope: bf16 rows");
  const c10::cuda::CUDAGuard g(x.device());
  const int M = (int)x.size(0);
  const long total = (long)M * rope_cols / 2;
  if (total == 0) return;
  const bool vec = (hd / 2) % 8 == 0 && rope_cols % hd == 0 && x.stride(0) % 8 == 0 &&
                   (reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(cos_t.data_ptr()) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(sin_t.data_ptr()) & 15) == 0;
  if (vec) {
    rope_vec8_kernel<<<grid_for(total / 8, 256), 256, 0, cur_stream()>>>(
        reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), x.stride(0), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(),
        M, (int)rope_cols, (int)hd, (int)seqlen, (float)sign);
    DTB_LAUNCH_CHECK();
    return;
  }
  rope_kernel<<<grid_for(total, 256), 256, 0, cur_stream()>>>(
      reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), x.stride(0), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), M,
      (int)rope_cols, (int)hd, (int)seqlen, (float)sign);
  DTB_LAUNCH_CHECK();
}

void rope_bwd(torch::Tensor d, torch::Tensor c, torch::Tensor s, int64_t rc, int64_t hd, int64_t sl) {
  rope_apply(d, c, s, rc, hd, sl, -1.0);
}
void rope_fwd(torch::Tensor d, torch::Tensor c, torch::Tensor s, int64_t rc, int64_t hd, int64_t sl) {
  rope_apply(d, c, s, rc, hd, sl, 1.0);
}

void swiglu_bwd(torch::Tensor da, torch::Tensor gu, torch::Tensor dgu) {
  const c10::cuda::CUDAGuard g(da.device());
  const int M = (int)da.size(0), F = (int)da.size(1);
  TORCH_CHECK(F % 2 == 0 && gu.size(1) == 2 * F && da.is_contiguous() && gu.is_contiguous(), "swiglu_bwd shapes");
  const long total = (long)M * F / 2;
  if (total == 0) return;
  if (F % 8 == 0 && (reinterpret_cast<uintptr_t>(da.data_ptr()) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(gu.data_ptr()) & 15) == 0 && (reinterpret_cast<uintptr_t>(dgu.data_ptr()) & 15) == 0) {
    swiglu_bwd_vec8_kernel<<<grid_for(total / 4, 256), 256, 0, cur_stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(da.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(dgu.data_ptr()), M, F);
    DTB_LAUNCH_CHECK();
    return;
  }
  swiglu_bwd_kernel<<<grid_for(total, 256), 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(da.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(dgu.data_ptr()), M, F);
  DTB_LAUNCH_CHECK();
}

torch::Tensor embedding_fwd(torch::Tensor tok, torch::Tensor w, c10::ScalarType out_dtype) {
  TORCH_CHECK(tok.scalar_type() == at::kLong && w.dim() == 2 && w.is_contiguous(), "embedding: int64 ids, [V,D]");
  const c10::cuda::CUDAGuard g(w.device());
  const int M = (int)tok.numel(), D = (int)w.size(1), V = (int)w.size(0);
  auto out = torch::empty({M, D}, w.options().dtype(out_dtype));
  if (M == 0) return out;
  int* err = dtb_error_word();
  const int nt = std::min(256, std::max(32, D));
  auto st = cur_stream();
  if (w.scalar_type() == at::kFloat && out_dtype == at::kFloat)
    embedding_fwd_kernel<float, float><<<M, nt, 0, st>>>(tok.data_ptr<int64_t>(), w.data_ptr<float>(), out.data_ptr<float>(), D, V, err);
  else if (w.scalar_type() == at::kFloat)
    embedding_fwd_kernel<float, __nv_bfloat16><<<M, nt, 0, st>>>(tok.data_ptr<int64_t>(), w.data_ptr<float>(),
                                                                 reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), D, V, err);
  else if (out_dtype == at::kFloat)
    embedding_fwd_kernel<__nv_bfloat16, float><<<M, nt, 0, st>>>(
        tok.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), out.data_ptr<float>(), D, V, err);
  else
    embedding_fwd_kernel<__nv_bfloat16, __nv_bfloat16><<<M, nt, 0, st>>>(
        tok.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), D, V, err);
  DTB_LAUNCH_CHECK();
  return out;
}

void embedding_bwd(torch::Tensor tok, torch::Tensor dout, torch::Tensor acc) {
  TORCH_CHECK(dout.scalar_type() == at::kBFloat16 && acc.scalar_type() == at::kFloat && acc.is_contiguous(),
              "embedding_bwd: bf16 grad, fp32 accumulator");
  const c10::cuda::CUDAGuard g(dout.device());
  const int M = (int)tok.numel(), D = (int)acc.size(1), V = (int)acc.size(0);
  if (M == 0) return;
  // own single-CTA sort while the keys fit 32 bits and the array fits shared memory
  // (every training shape here: <= 32768 tokens, vocabulary < 2^17); beyond that
  // the library's stable radix sort
  int shift = 0;
  while ((1L << shift) < M) ++shift;
  int npow2 = 1;
  while (npow2 < M) npow2 <<= 1;
  torch::Tensor st_tok, order;
  if (M <= 32768 && ((long)(V + 1) << shift) <= (1L << 32)) {
    st_tok = torch::empty({M}, tok.options().dtype(at::kLong));
    order = torch::empty({M}, tok.options().dtype(at::kLong));
    const int smem = npow2 * 4;
    static bool cfg = false;
    if (!cfg) {
      DTB_CUDA(cudaFuncSetAttribute(sort_tokens_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 32768 * 4));
      cfg = true;
    }
    auto tk = tok.reshape({-1}).to(at::kLong).contiguous();
    sort_tokens_kernel<<<1, 1024, smem, cur_stream()>>>(tk.data_ptr<int64_t>(), M, V, shift, npow2,
                                                        st_tok.data_ptr<int64_t>(), order.data_ptr<int64_t>());
    DTB_LAUNCH_CHECK();
  } else {
    auto sorted = at::sort(tok.reshape({-1}), /*stable=*/true, 0, false);
    st_tok = std::get<0>(sorted).contiguous();
    order = std::get<1>(sorted).contiguous();
  }
  embedding_bwd_kernel<<<M, std::min(256, std::max(32, D)), 0, cur_stream()>>>(
      st_tok.data_ptr<int64_t>(), order.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
      acc.data_ptr<float>(), M, D, V);
  DTB_LAUNCH_CHECK();
}

std::vector<torch::Tensor> cross_entropy_fwd(torch::Tensor logits, torch::Tensor labels, int64_t ignore) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.is_contiguous(), "ce: fp32 [M,V]");
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.numel() == logits.size(0), "ce: int64 labels [M]");
  const c10::cuda::CUDAGuard g(logits.device());
  const int M = (int)logits.size(0), V = (int)logits.size(1);
  auto dlog = torch::empty({M, V}, logits.options().dtype(at::kBFloat16));
  auto rows = torch::empty({std::max(M, 1)}, logits.options());
  auto nvalid = torch::empty({1}, logits.options().dtype(at::kInt));
  auto loss = torch::empty({}, logits.options());
  auto st = cur_stream();
  count_valid_kernel<<<1, 1024, 0, st>>>(labels.data_ptr<int64_t>(), M, ignore, V, nvalid.data_ptr<int>());
  if (M > 0)
    ce_row_kernel<512><<<M, 512, 0, st>>>(logits.data_ptr<float>(), labels.data_ptr<int64_t>(),
                                         reinterpret_cast<__nv_bfloat16*>(dlog.data_ptr()), rows.data_ptr<float>(),
                                         nvalid.data_ptr<int>(), V, ignore);
  ce_finish_kernel<1024><<<1, 1024, 0, st>>>(rows.data_ptr<float>(), nvalid.data_ptr<int>(), loss.data_ptr<float>(), M);
  DTB_LAUNCH_CHECK();
  return {loss, dlog};
}

void adamw(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, torch::Tensor out,
           c10::optional<torch::Tensor> clip, double lr, double b1, double b2, double eps, double wd, int64_t step) {
  TORCH_CHECK(p.scalar_type() == at::kFloat && g.scalar_type() == at::kFloat && out.scalar_type() == at::kBFloat16,
              "adamw: fp32 master/grad, bf16 out");
  const c10::cuda::CUDAGuard gd(p.device());
  const long n = p.numel();
  if (n == 0) return;
  const float bc1 = 1.f - (float)std::pow(b1, (double)step);
  const float bc2s = (float)std::sqrt(1.0 - std::pow(b2, (double)step));
  adamw_kernel<<<grid_for(n, 256), 256, 0, cur_stream()>>>(
      p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), clip.has_value() ? clip->data_ptr<float>() : nullptr, n,
      (float)lr, (float)b1, (float)b2, (float)eps, (float)wd, bc1, bc2s);
  DTB_LAUNCH_CHECK();
}

// Fixed-order sum of a small fp32 buffer (per-block partials) in one CTA.
torch::Tensor sum_small(torch::Tensor x) {
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.is_contiguous() && x.numel() < (1L << 31), "sum_small: fp32");
  const c10::cuda::CUDAGuard g(x.device());
  auto out = torch::empty({}, x.options());
  sum_parts_kernel<1024><<<1, 1024, 0, cur_stream()>>>(x.data_ptr<float>(), (int)x.numel(), out.data_ptr<float>());
  DTB_LAUNCH_CHECK();
  return out;
}

torch::Tensor sumsq(torch::Tensor x) {
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.is_contiguous(), "sumsq: contiguous fp32");
  const c10::cuda::CUDAGuard g(x.device());
  const long n = x.numel();
  const int nb = device_sm_count() * 8;
  auto part = torch::empty({nb}, x.options());
  auto out = torch::empty({}, x.options());
  auto st = cur_stream();
  sumsq_part_kernel<256><<<nb, 256, 0, st>>>(x.data_ptr<float>(), n, part.data_ptr<float>());
  sum_parts_kernel<1024><<<1, 1024, 0, st>>>(part.data_ptr<float>(), nb, out.data_ptr<float>());
  DTB_LAUNCH_CHECK();
  return out;
}
