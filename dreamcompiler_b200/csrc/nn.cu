// Building blocks of the GPT training step that sit
// between the GEMMs and the attention kernels, as device kernels so the step
// never leaves the GPU. Each one restates the reference op it replaces:
//   layer_norm   runtime/io/builtins.inc:167-197, backward ops/autograd.inc:453-470
//   gelu (tanh)  runtime/io/builtins.inc:548-560, backward ops/autograd.inc:293-303
//   embedding    runtime/nn/training.inc:579-600, backward ops/autograd.inc:330-341
//   log_softmax  runtime/ops/elementwise.inc:1550-1568, backward autograd.inc:212-231
//   nll_loss     runtime/ops/elementwise.inc:1575-1603, backward autograd.inc:232-245
//   adamw_update runtime/io/builtins.inc:578-617
// All are HBM-bound element-wise or row-wise passes: one warp per row for the
// row reductions, 16-byte accesses where the layout allows, deterministic
// reductions except the embedding-table scatter (fp32 atomics, as any
// scatter-add of repeated token ids).
#include <cuda_bf16.h>

#include <cmath>

#include "common.h"
#include "sm100.cuh"

namespace dgx {
namespace {

constexpr float kLnEps = 1e-5f;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------- layer norm
// One warp per row; two passes over the row (mean, then centred variance), as
// the reference does in f64.
__global__ void ln_fwd_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, float* __restrict__ mean,
                              float* __restrict__ rstd, int R, int C) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= R) return;
  const float* xr = x + (size_t)row * C;
  float s = 0.f;
  for (int j = lane; j < C; j += 32) s += xr[j];
  const float mu = warp_sum(s) / C;
  float v = 0.f;
  for (int j = lane; j < C; j += 32) {
    const float d = xr[j] - mu;
    v = fmaf(d, d, v);
  }
  const float rs = rsqrtf(warp_sum(v) / C + kLnEps);
  __nv_bfloat16* yr = y + (size_t)row * C;
  for (int j = lane; j < C; j += 32) yr[j] = __float2bfloat16_rn((xr[j] - mu) * rs);
  if (lane == 0) {
    mean[row] = mu;
    rstd[row] = rs;
  }
}

// Row-in-registers forms for C a multiple of 128 (C <= 128 * LN_MAXV) and
// 16-byte aligned rows: lane l holds float4 groups l, l+32, ... of the row,
// so every access is a 16-byte load or store and the row is read once.
// Same two-pass statistics and formulas as the scalar kernels.
constexpr int LN_MAXV = 8;

__device__ __forceinline__ uint2 pack_bf16x4(float a, float b, float c, float d) {
  return make_uint2(pack_bf16x2(a, b), pack_bf16x2(c, d));
}

__global__ void ln_fwd_vec_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, float* __restrict__ mean,
                                  float* __restrict__ rstd, int R, int C) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= R) return;
  const int nv = C / 128;
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * C);
  float4 xv[LN_MAXV];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < LN_MAXV; ++i)
    if (i < nv) {
      xv[i] = __ldg(xr + lane + 32 * i);
      s += (xv[i].x + xv[i].y) + (xv[i].z + xv[i].w);
    }
  const float mu = warp_sum(s) / C;
  float v = 0.f;
#pragma unroll
  for (int i = 0; i < LN_MAXV; ++i)
    if (i < nv) {
      const float a = xv[i].x - mu, b = xv[i].y - mu, c = xv[i].z - mu, d = xv[i].w - mu;
      v = fmaf(a, a, v);
      v = fmaf(b, b, v);
      v = fmaf(c, c, v);
      v = fmaf(d, d, v);
    }
  const float rs = rsqrtf(warp_sum(v) / C + kLnEps);
  uint2* yr = reinterpret_cast<uint2*>(y + (size_t)row * C);
#pragma unroll
  for (int i = 0; i < LN_MAXV; ++i)
    if (i < nv)
      yr[lane + 32 * i] = pack_bf16x4((xv[i].x - mu) * rs, (xv[i].y - mu) * rs, (xv[i].z - mu) * rs,
                                      (xv[i].w - mu) * rs);
  if (lane == 0) {
    mean[row] = mu;
    rstd[row] = rs;
  }
}

__global__ void ln_bwd_vec_kernel(const float* __restrict__ x, const float* __restrict__ mean,
                                  const float* __restrict__ rstd, const float* __restrict__ dy, float* __restrict__ dx,
                                  __nv_bfloat16* __restrict__ dx16, int R, int C, int accumulate) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= R) return;
  const int nv = C / 128;
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * C);
  const float4* gr = reinterpret_cast<const float4*>(dy + (size_t)row * C);
  const float mu = mean[row], rs = rstd[row];
  float4 yv[LN_MAXV], gv[LN_MAXV];
  float sg = 0.f, sgy = 0.f;
#pragma unroll
  for (int i = 0; i < LN_MAXV; ++i)
    if (i < nv) {
      const float4 xi = __ldg(xr + lane + 32 * i);
      gv[i] = __ldg(gr + lane + 32 * i);
      yv[i] = make_float4((xi.x - mu) * rs, (xi.y - mu) * rs, (xi.z - mu) * rs, (xi.w - mu) * rs);
      sg += (gv[i].x + gv[i].y) + (gv[i].z + gv[i].w);
      sgy = fmaf(gv[i].x, yv[i].x, sgy);
      sgy = fmaf(gv[i].y, yv[i].y, sgy);
      sgy = fmaf(gv[i].z, yv[i].z, sgy);
      sgy = fmaf(gv[i].w, yv[i].w, sgy);
    }
  sg = warp_sum(sg);
  sgy = warp_sum(sgy);
  const float a = rs / C;
  float4* dr = reinterpret_cast<float4*>(dx + (size_t)row * C);
  uint2* d16 = reinterpret_cast<uint2*>(dx16 + (size_t)row * C);
#pragma unroll
  for (int i = 0; i < LN_MAXV; ++i)
    if (i < nv) {
      float4 o = make_float4(a * (C * gv[i].x - sg - yv[i].x * sgy), a * (C * gv[i].y - sg - yv[i].y * sgy),
                             a * (C * gv[i].z - sg - yv[i].z * sgy), a * (C * gv[i].w - sg - yv[i].w * sgy));
      if (accumulate) {
        const float4 p = dr[lane + 32 * i];
        o = make_float4(p.x + o.x, p.y + o.y, p.z + o.z, p.w + o.w);
      }
      dr[lane + 32 * i] = o;
      if (dx16) d16[lane + 32 * i] = pack_bf16x4(o.x, o.y, o.z, o.w);
    }
}

// dx (+)= rstd/C * (C*dy - sum(dy) - y*sum(dy*y)), y recomputed from x;
// dx16 (may be null) receives bf16(dx) as well, the operand of the next GEMMs.
__global__ void ln_bwd_kernel(const float* __restrict__ x, const float* __restrict__ mean,
                              const float* __restrict__ rstd, const float* __restrict__ dy, float* __restrict__ dx,
                              __nv_bfloat16* __restrict__ dx16, int R, int C, int accumulate) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= R) return;
  const float* xr = x + (size_t)row * C;
  const float* gr = dy + (size_t)row * C;
  const float mu = mean[row], rs = rstd[row];
  float sg = 0.f, sgy = 0.f;
  for (int j = lane; j < C; j += 32) {
    const float g = gr[j];
    sg += g;
    sgy = fmaf(g, (xr[j] - mu) * rs, sgy);
  }
  sg = warp_sum(sg);
  sgy = warp_sum(sgy);
  const float a = rs / C;
  float* dr = dx + (size_t)row * C;
  for (int j = lane; j < C; j += 32) {
    const float yv = (xr[j] - mu) * rs;
    const float v = a * (C * gr[j] - sg - yv * sgy);
    const float o = accumulate ? dr[j] + v : v;
    dr[j] = o;
    if (dx16) dx16[(size_t)row * C + j] = __float2bfloat16_rn(o);
  }
}

// ---------------------------------------------------------------- GELU (tanh form)
constexpr float kGeluK = 0.7978845608028654f;  // sqrt(2/pi)
constexpr float kGeluC = 0.044715f;

__device__ __forceinline__ float ld_as_float(const float* p, long long i) { return p[i]; }
__device__ __forceinline__ float ld_as_float(const __nv_bfloat16* p, long long i) { return __bfloat162float(p[i]); }

template <typename TX>
__global__ void gelu_fwd_kernel(const TX* __restrict__ x, __nv_bfloat16* __restrict__ y, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float v = ld_as_float(x, i);
    const float t = tanhf(kGeluK * fmaf(kGeluC * v, v * v, v));
    y[i] = __float2bfloat16_rn(0.5f * v * (1.f + t));
  }
}

// bf16 in, bf16 out, 8 elements per thread (16-byte loads and stores) with
// the hardware tanh (tanh.approx.f32: relative error about 2^-11, far below
// the bf16 output's 2^-8): the MLP activation of the GPT step.
__device__ __forceinline__ float tanh_fast(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

__global__ void gelu_fwd_bf16x8_kernel(const uint4* __restrict__ x, uint4* __restrict__ y, int n8) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += gridDim.x * blockDim.x) {
    const uint4 v = __ldg(x + i);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float a = bf_lo(w[k]), b = bf_hi(w[k]);
      const float ta = tanh_fast(kGeluK * fmaf(kGeluC * a, a * a, a));
      const float tb = tanh_fast(kGeluK * fmaf(kGeluC * b, b * b, b));
      o[k] = pack_bf16x2(0.5f * a * (1.f + ta), 0.5f * b * (1.f + tb));
    }
    y[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__global__ void gelu_bwd_bf16x8_kernel(const uint4* __restrict__ x, const uint4* __restrict__ dy, uint4* __restrict__ dx,
                                       int n8) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += gridDim.x * blockDim.x) {
    const uint4 v = __ldg(x + i), gv = __ldg(dy + i);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w}, gw[4] = {gv.x, gv.y, gv.z, gv.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float r[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float a = h ? bf_hi(w[k]) : bf_lo(w[k]);
        const float th = tanh_fast(kGeluK * fmaf(kGeluC * a, a * a, a));
        const float dinner = kGeluK * fmaf(3.f * kGeluC * a, a, 1.f);
        const float gg = 0.5f * (1.f + th) + 0.5f * a * (1.f - th * th) * dinner;
        r[h] = gg * (h ? bf_hi(gw[k]) : bf_lo(gw[k]));
      }
      o[k] = pack_bf16x2(r[0], r[1]);
    }
    dx[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// dx = (0.5*(1+th) + 0.5*x*(1-th^2)*k*(1+3c x^2)) * dy, written as bf16 (the
// next consumer is a GEMM).
template <typename TX, typename TG>
__global__ void gelu_bwd_kernel(const TX* __restrict__ x, const TG* __restrict__ dy, __nv_bfloat16* __restrict__ dx,
                                long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float v = ld_as_float(x, i);
    const float th = tanhf(kGeluK * fmaf(kGeluC * v, v * v, v));
    const float dinner = kGeluK * fmaf(3.f * kGeluC * v, v, 1.f);
    const float g = 0.5f * (1.f + th) + 0.5f * v * (1.f - th * th) * dinner;
    dx[i] = __float2bfloat16_rn(g * ld_as_float(dy, i));
  }
}

// ---------------------------------------------------------------- embedding
// x[i][:] = W[tok[i]][:] + P[i % S][:]   (token id outside [0, V): zero row,
// as the reference leaves the output row at zero)
__global__ void emb_fwd_kernel(const int* __restrict__ tok, const float* __restrict__ W, const float* __restrict__ P,
                               float* __restrict__ x, int n, int S, int d, int V) {
  const long long total = (long long)n * d;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
    const int i = (int)(e / d), j = (int)(e % d);
    const int t = tok[i];
    float v = (t >= 0 && t < V) ? W[(size_t)t * d + j] : 0.f;
    if (P) v += P[(size_t)(i % S) * d + j];
    x[e] = v;
  }
}

// dW[tok[i]] += dx[i]: fp32 atomics (repeated ids collide).
__global__ void emb_bwd_table_kernel(const int* __restrict__ tok, const float* __restrict__ dx, float* __restrict__ dW,
                                     int n, int d, int V) {
  const long long total = (long long)n * d;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
    const int i = (int)(e / d), j = (int)(e % d);
    const int t = tok[i];
    if (t >= 0 && t < V) atomicAdd(&dW[(size_t)t * d + j], dx[e]);
  }
}

// dP[s][j] += sum_b dx[b*S + s][j]  (fixed order over b: deterministic)
__global__ void emb_bwd_pos_kernel(const float* __restrict__ dx, float* __restrict__ dP, int n, int S, int d) {
  const int total = S * d;
  const int B = n / S;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int b = 0; b < B; ++b) s += dx[(size_t)b * total + e];
    dP[e] += s;
  }
}

// ---------------------------------------------------------------- log_softmax + nll
// One warp per row over the V valid columns of a row of pitch ld:
// nll[r] = lse - x[target], dlogits = (softmax - onehot(target)) / n, and the
// columns past V are written as zero.
template <typename TG>
__global__ void softmax_nll_kernel(const float* __restrict__ logits, int ld, int V, const int* __restrict__ target,
                                   int n, float* __restrict__ nll, TG* __restrict__ dlogits) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= n) return;
  const float* xr = logits + (size_t)row * ld;
  float mx = -INFINITY;
  for (int j = lane; j < V; j += 32) mx = fmaxf(mx, xr[j]);
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float s = 0.f;
  for (int j = lane; j < V; j += 32) s += expf(xr[j] - mx);
  s = warp_sum(s);
  const float lse = mx + logf(s);
  const int t = target[row];
  if (lane == 0) nll[row] = (t >= 0 && t < V) ? lse - xr[t] : 0.f;
  if (dlogits) {
    const float inv_n = 1.f / n, inv_s = 1.f / s;
    TG* gr = dlogits + (size_t)row * ld;
    for (int j = lane; j < ld; j += 32) {
      float g = 0.f;
      if (j < V) g = (expf(xr[j] - mx) * inv_s - (j == t ? 1.f : 0.f)) * inv_n;
      if constexpr (sizeof(TG) == 2)
        gr[j] = __float2bfloat16_rn(g);
      else
        gr[j] = g;
    }
  }
}

// loss = mean(nll) in a fixed order (one CTA).
__global__ void mean_kernel(const float* __restrict__ v, int n, float* __restrict__ out) {
  __shared__ float red[32];
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += v[i];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    s = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    s = warp_sum(s);
    if (threadIdx.x == 0) *out = s / n;
  }
}

// ---------------------------------------------------------------- AdamW
__global__ void adamw_kernel(float* __restrict__ p, float* __restrict__ g, float* __restrict__ m, float* __restrict__ v,
                             long long n, float lr, float b1, float b2, float eps, float wd, float bc1, float bc2,
                             const int* __restrict__ step_dev) {
  if (step_dev) {  // step from device memory (replayable CUDA graphs)
    const float t = (float)*step_dev;
    bc1 = 1.f - powf(b1, t);
    bc2 = 1.f - powf(b2, t);
  }
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float gi = g[i];
    const float mi = fmaf(b1, m[i], (1.f - b1) * gi);
    const float vi = fmaf(b2, v[i], (1.f - b2) * gi * gi);
    m[i] = mi;
    v[i] = vi;
    const float mh = mi / bc1, vh = vi / bc2;
    const float pi = p[i];
    p[i] = pi - lr * (mh / (sqrtf(vh) + eps) + wd * pi);
    g[i] = 0.f;
  }
}

// ---------------------------------------------------------------- column sums (bias gradients)
// Stage 1: CTA (column block of 32, row slice) -> partial sums; stage 2 adds
// the slices in order. Both fixed-order: deterministic.
constexpr int CS_SLICES = 32;
template <typename T>
__global__ void colsum_partial_kernel(const T* __restrict__ dy, float* __restrict__ part, int R, int N) {
  __shared__ float red[8][33];
  const int c = blockIdx.x * 32 + (threadIdx.x & 31);
  const int ty = threadIdx.x >> 5;  // 8 row groups
  const int rows_per = (R + CS_SLICES - 1) / CS_SLICES;
  const int r0 = blockIdx.y * rows_per, r1 = min(R, r0 + rows_per);
  float s = 0.f;
  if (c < N)
    for (int r = r0 + ty; r < r1; r += 8) {
      if constexpr (sizeof(T) == 2)
        s += __bfloat162float(dy[(size_t)r * N + c]);
      else
        s += dy[(size_t)r * N + c];
    }
  red[ty][threadIdx.x & 31] = s;
  __syncthreads();
  if (ty == 0 && c < N) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) t += red[k][threadIdx.x];
    part[(size_t)blockIdx.y * N + c] = t;
  }
}
// Vector form (N a multiple of 16 bytes' worth of columns, aligned rows):
// a thread sums VEC adjacent columns with 16-byte loads; `slices` row slices
// sized so that the grid covers the SMs.
template <typename T>
__global__ void colsum_partial_vec_kernel(const T* __restrict__ dy, float* __restrict__ part, int R, int N,
                                          int slices) {
  constexpr int VEC = 16 / sizeof(T);
  __shared__ float red[8][32 * VEC + 1];
  const int cv = blockIdx.x * 32 + (threadIdx.x & 31);  // column vector index
  const int ty = threadIdx.x >> 5;                       // 8 row groups
  const int rows_per = (R + slices - 1) / slices;
  const int r0 = blockIdx.y * rows_per, r1 = min(R, r0 + rows_per);
  float acc[VEC];
#pragma unroll
  for (int k = 0; k < VEC; ++k) acc[k] = 0.f;
  if (cv * VEC < N)
#pragma unroll 4
    for (int r = r0 + ty; r < r1; r += 8) {
      const uint4 w = __ldg(reinterpret_cast<const uint4*>(dy + (size_t)r * N) + cv);
      if constexpr (sizeof(T) == 2) {
        const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          acc[2 * k] += __uint_as_float(u[k] << 16);
          acc[2 * k + 1] += __uint_as_float(u[k] & 0xFFFF0000u);
        }
      } else {
        acc[0] += __uint_as_float(w.x);
        acc[1] += __uint_as_float(w.y);
        acc[2] += __uint_as_float(w.z);
        acc[3] += __uint_as_float(w.w);
      }
    }
#pragma unroll
  for (int k = 0; k < VEC; ++k) red[ty][(threadIdx.x & 31) * VEC + k] = acc[k];
  __syncthreads();
  for (int j = threadIdx.x; j < 32 * VEC; j += blockDim.x) {
    const int c = blockIdx.x * 32 * VEC + j;
    if (c < N) {
      float t = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) t += red[k][j];
      part[(size_t)blockIdx.y * N + c] = t;
    }
  }
}

// db[c] (+)= sum over slices of part[k][c]. A block of 8 warps owns 32
// columns: warp w sums slices w, w+8, ... (four independent partial sums so
// four loads are in flight), then warp 0 adds the 8 warp sums in order. The
// order is fixed, so the result is the same on every run.
__global__ void colsum_final_kernel(const float* __restrict__ part, float* __restrict__ db, int N, int accumulate,
                                    int slices) {
  __shared__ float red[8][33];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  if (c < N) {
    int k = w;
    for (; k + 24 < slices; k += 32) {
      s0 += part[(size_t)k * N + c];
      s1 += part[(size_t)(k + 8) * N + c];
      s2 += part[(size_t)(k + 16) * N + c];
      s3 += part[(size_t)(k + 24) * N + c];
    }
    for (; k < slices; k += 8) s0 += part[(size_t)k * N + c];
  }
  red[w][lane] = (s0 + s1) + (s2 + s3);
  __syncthreads();
  if (w == 0 && c < N) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) s += red[j][lane];
    db[c] = accumulate ? db[c] + s : s;
  }
}

// ---------------------------------------------------------------- head layout
// rows [B*S][ld] (head h of width D at column col0 + h*D) <-> heads [B*H][S][D].
// One thread moves 8 consecutive elements of a head row (D % 8 == 0; 32-bit
// index arithmetic: B*S*H*D < 2^31 is checked by the callers).
template <typename TS>
__global__ void rows_to_heads_kernel(const TS* __restrict__ src, int ld, int col0, __nv_bfloat16* __restrict__ dst,
                                     int B, int S, int H, int D) {
  const int D8 = D >> 3;
  const int total = B * H * S * D8;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += gridDim.x * blockDim.x) {
    const int dd = (e % D8) << 3;
    int t = e / D8;
    const int s = t % S;
    t /= S;
    const int h = t % H, b = t / H;
    const size_t so = ((size_t)b * S + s) * ld + col0 + h * D + dd;
    uint4 w;
    if constexpr (sizeof(TS) == 2) {
      w = *reinterpret_cast<const uint4*>(src + so);
    } else {
      const float4 a = *reinterpret_cast<const float4*>(src + so);
      const float4 c = *reinterpret_cast<const float4*>(src + so + 4);
      __nv_bfloat162 q[4] = {__floats2bfloat162_rn(a.x, a.y), __floats2bfloat162_rn(a.z, a.w),
                             __floats2bfloat162_rn(c.x, c.y), __floats2bfloat162_rn(c.z, c.w)};
      w = *reinterpret_cast<uint4*>(q);
    }
    *reinterpret_cast<uint4*>(dst + (size_t)e * 8) = w;
  }
}
__global__ void heads_to_rows_kernel(const __nv_bfloat16* __restrict__ src, __nv_bfloat16* __restrict__ dst, int ld,
                                     int col0, int B, int S, int H, int D) {
  const int D8 = D >> 3;
  const int total = B * H * S * D8;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += gridDim.x * blockDim.x) {
    const int dd = (e % D8) << 3;
    int t = e / D8;
    const int s = t % S;
    t /= S;
    const int h = t % H, b = t / H;
    *reinterpret_cast<uint4*>(dst + ((size_t)b * S + s) * ld + col0 + h * D + dd) =
        *reinterpret_cast<const uint4*>(src + (size_t)e * 8);
  }
}

int ew_grid(long long n) {
  const long long b = (n + 255) / 256;
  const long long cap = (long long)num_sms() * 8;
  return (int)(b < cap ? (b > 0 ? b : 1) : cap);
}

}  // namespace
}  // namespace dgx

using namespace dgx;

namespace {
// The row-in-registers layer-norm kernels apply: C a multiple of 128 up to
// 128 * LN_MAXV, every row 16-byte aligned (bf16 rows: 8-byte aligned).
bool ln_vec_ok(int C, const void* a, const void* b = nullptr, const void* c = nullptr, const void* d = nullptr) {
  if (C % 128 || C > 128 * LN_MAXV) return false;
  return ((((uintptr_t)a) | (uintptr_t)b | (uintptr_t)c | (uintptr_t)d) & 15) == 0;
}
}  // namespace

extern "C" {

dgx_status dgx_layernorm_fwd(const float* x, void* y16, float* mean, float* rstd, int R, int C, void* stream) {
  DGX_FAULT_POINT("dgx_layernorm_fwd");
  if (R < 0 || C <= 0) return set_error(DGX_EINVAL, "dgx_layernorm_fwd: R=%d C=%d", R, C);
  if (R == 0) return DGX_OK;
  if (!x || !y16 || !mean || !rstd) return set_error(DGX_EINVAL, "dgx_layernorm_fwd: null pointer");
  if (ln_vec_ok(C, x, y16))
    ln_fwd_vec_kernel<<<(R + 7) / 8, 256, 0, (cudaStream_t)stream>>>(x, (__nv_bfloat16*)y16, mean, rstd, R, C);
  else
    ln_fwd_kernel<<<(R + 7) / 8, 256, 0, (cudaStream_t)stream>>>(x, (__nv_bfloat16*)y16, mean, rstd, R, C);
  return cuda_status(cudaGetLastError(), "dgx_layernorm_fwd");
}

dgx_status dgx_layernorm_bwd(const float* x, const float* mean, const float* rstd, const float* dy, float* dx, int R,
                             int C, int accumulate, void* stream) {
  DGX_FAULT_POINT("dgx_layernorm_bwd");
  if (R < 0 || C <= 0) return set_error(DGX_EINVAL, "dgx_layernorm_bwd: R=%d C=%d", R, C);
  if (R == 0) return DGX_OK;
  if (!x || !mean || !rstd || !dy || !dx) return set_error(DGX_EINVAL, "dgx_layernorm_bwd: null pointer");
  if (ln_vec_ok(C, x, dy, dx))
    ln_bwd_vec_kernel<<<(R + 7) / 8, 256, 0, (cudaStream_t)stream>>>(x, mean, rstd, dy, dx, nullptr, R, C, accumulate);
  else
    ln_bwd_kernel<<<(R + 7) / 8, 256, 0, (cudaStream_t)stream>>>(x, mean, rstd, dy, dx, nullptr, R, C, accumulate);
  return cuda_status(cudaGetLastError(), "dgx_layernorm_bwd");
}

dgx_status dgx_layernorm_bwd_x16(const float* x, const float* mean, const float* rstd, const float* dy, float* dx,
                                 void* dx16, int R, int C, int accumulate, void* stream) {
  DGX_FAULT_POINT("dgx_layernorm_bwd_x16");
  if (R < 0 || C <= 0) return set_error(DGX_EINVAL, "dgx_layernorm_bwd_x16: R=%d C=%d", R, C);
  if (R == 0) return DGX_OK;
  if (!x || !mean || !rstd || !dy || !dx || !dx16) return set_error(DGX_EINVAL, "dgx_layernorm_bwd_x16: null pointer");
  if (ln_vec_ok(C, x, dy, dx, dx16))
    ln_bwd_vec_kernel<<<(R + 7) / 8, 256, 0, (cudaStream_t)stream>>>(x, mean, rstd, dy, dx, (__nv_bfloat16*)dx16, R,
                                                                     C, accumulate);
  else
    ln_bwd_kernel<<<(R + 7) / 8, 256, 0, (cudaStream_t)stream>>>(x, mean, rstd, dy, dx, (__nv_bfloat16*)dx16, R, C,
                                                                 accumulate);
  return cuda_status(cudaGetLastError(), "dgx_layernorm_bwd_x16");
}

dgx_status dgx_gelu_fwd(const void* x, int x_type, void* y16, long long n, void* stream) {
  DGX_FAULT_POINT("dgx_gelu_fwd");
  if (n < 0) return set_error(DGX_EINVAL, "dgx_gelu_fwd: n=%lld", n);
  if (x_type != DGX_F32 && x_type != DGX_BF16) return set_error(DGX_EINVAL, "dgx_gelu_fwd: type %d", x_type);
  if (n == 0) return DGX_OK;
  if (!x || !y16) return set_error(DGX_EINVAL, "dgx_gelu_fwd: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  if (x_type == DGX_BF16 && ((((uintptr_t)x) | (uintptr_t)y16) & 15) == 0 && n < (1LL << 33)) {
    // bf16 -> bf16: 8-wide vector kernel, the last n % 8 elements by the scalar one
    const long long n8 = n / 8;
    if (n8) gelu_fwd_bf16x8_kernel<<<ew_grid(n8), 256, 0, s>>>((const uint4*)x, (uint4*)y16, (int)n8);
    if (n % 8)
      gelu_fwd_kernel<__nv_bfloat16><<<1, 256, 0, s>>>((const __nv_bfloat16*)x + n8 * 8,
                                                     (__nv_bfloat16*)y16 + n8 * 8, n % 8);
  } else if (x_type == DGX_F32) {
    gelu_fwd_kernel<float><<<ew_grid(n), 256, 0, s>>>((const float*)x, (__nv_bfloat16*)y16, n);
  } else {
    gelu_fwd_kernel<__nv_bfloat16><<<ew_grid(n), 256, 0, s>>>((const __nv_bfloat16*)x, (__nv_bfloat16*)y16, n);
  }
  return cuda_status(cudaGetLastError(), "dgx_gelu_fwd");
}

dgx_status dgx_gelu_bwd(const void* x, int x_type, const void* dy, int dy_type, void* dx16, long long n, void* stream) {
  DGX_FAULT_POINT("dgx_gelu_bwd");
  if (n < 0) return set_error(DGX_EINVAL, "dgx_gelu_bwd: n=%lld", n);
  const bool xt = x_type == DGX_F32 || x_type == DGX_BF16, gt = dy_type == DGX_F32 || dy_type == DGX_BF16;
  if (!xt || !gt) return set_error(DGX_EINVAL, "dgx_gelu_bwd: types %d %d", x_type, dy_type);
  if (n == 0) return DGX_OK;
  if (!x || !dy || !dx16) return set_error(DGX_EINVAL, "dgx_gelu_bwd: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  __nv_bfloat16* o = (__nv_bfloat16*)dx16;
  const int g = ew_grid(n);
  if (x_type == DGX_BF16 && dy_type == DGX_BF16 && ((((uintptr_t)x) | (uintptr_t)dy | (uintptr_t)dx16) & 15) == 0 &&
      n < (1LL << 33)) {
    const long long n8 = n / 8;
    if (n8) gelu_bwd_bf16x8_kernel<<<ew_grid(n8), 256, 0, s>>>((const uint4*)x, (const uint4*)dy, (uint4*)dx16, (int)n8);
    if (n % 8)
      gelu_bwd_kernel<__nv_bfloat16, __nv_bfloat16><<<1, 256, 0, s>>>(
          (const __nv_bfloat16*)x + n8 * 8, (const __nv_bfloat16*)dy + n8 * 8, o + n8 * 8, n % 8);
    return cuda_status(cudaGetLastError(), "dgx_gelu_bwd");
  }
  if (x_type == DGX_F32 && dy_type == DGX_F32)
    gelu_bwd_kernel<float, float><<<g, 256, 0, s>>>((const float*)x, (const float*)dy, o, n);
  else if (x_type == DGX_F32)
    gelu_bwd_kernel<float, __nv_bfloat16><<<g, 256, 0, s>>>((const float*)x, (const __nv_bfloat16*)dy, o, n);
  else if (dy_type == DGX_F32)
    gelu_bwd_kernel<__nv_bfloat16, float><<<g, 256, 0, s>>>((const __nv_bfloat16*)x, (const float*)dy, o, n);
  else
    gelu_bwd_kernel<__nv_bfloat16, __nv_bfloat16><<<g, 256, 0, s>>>((const __nv_bfloat16*)x,
                                                                    (const __nv_bfloat16*)dy, o, n);
  return cuda_status(cudaGetLastError(), "dgx_gelu_bwd");
}

dgx_status dgx_embedding_fwd(const int* tok, const float* W, const float* P, float* x, int n, int S, int d, int V,
                             void* stream) {
  DGX_FAULT_POINT("dgx_embedding_fwd");
  if (n < 0 || d <= 0 || V <= 0 || (P && S <= 0)) return set_error(DGX_EINVAL, "dgx_embedding_fwd: sizes");
  if (n == 0) return DGX_OK;
  if (!tok || !W || !x) return set_error(DGX_EINVAL, "dgx_embedding_fwd: null pointer");
  emb_fwd_kernel<<<ew_grid((long long)n * d), 256, 0, (cudaStream_t)stream>>>(tok, W, P, x, n, P ? S : 1, d, V);
  return cuda_status(cudaGetLastError(), "dgx_embedding_fwd");
}

dgx_status dgx_embedding_bwd(const int* tok, const float* dx, float* dW, float* dP, int n, int S, int d, int V,
                             void* stream) {
  DGX_FAULT_POINT("dgx_embedding_bwd");
  if (n < 0 || d <= 0 || V <= 0) return set_error(DGX_EINVAL, "dgx_embedding_bwd: sizes");
  if (dP && (S <= 0 || n % S)) return set_error(DGX_EINVAL, "dgx_embedding_bwd: n=%d not a multiple of S=%d", n, S);
  if (n == 0) return DGX_OK;
  if (!tok || !dx || !dW) return set_error(DGX_EINVAL, "dgx_embedding_bwd: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  emb_bwd_table_kernel<<<ew_grid((long long)n * d), 256, 0, s>>>(tok, dx, dW, n, d, V);
  if (dP) emb_bwd_pos_kernel<<<ew_grid((long long)S * d), 256, 0, s>>>(dx, dP, n, S, d);
  return cuda_status(cudaGetLastError(), "dgx_embedding_bwd");
}

dgx_status dgx_softmax_nll(const float* logits, int ld, int V, const int* target, int n, float* loss, void* dlogits,
                           int dlogits_type, void* stream) {
  DGX_FAULT_POINT("dgx_softmax_nll");
  if (n < 0 || V <= 0 || ld < V) return set_error(DGX_EINVAL, "dgx_softmax_nll: n=%d V=%d ld=%d", n, V, ld);
  if (dlogits && dlogits_type != DGX_F32 && dlogits_type != DGX_BF16)
    return set_error(DGX_EINVAL, "dgx_softmax_nll: dlogits type %d", dlogits_type);
  if (n == 0) return DGX_OK;
  if (!logits || !target || !loss) return set_error(DGX_EINVAL, "dgx_softmax_nll: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  float* nll = (float*)library_scratch((size_t)n * sizeof(float), s);
  if (!nll) return set_error(DGX_ENOMEM, "dgx_softmax_nll: scratch");
  const int grid = (n + 7) / 8;
  if (!dlogits || dlogits_type == DGX_F32)
    softmax_nll_kernel<float><<<grid, 256, 0, s>>>(logits, ld, V, target, n, nll, (float*)dlogits);
  else
    softmax_nll_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(logits, ld, V, target, n, nll, (__nv_bfloat16*)dlogits);
  mean_kernel<<<1, 1024, 0, s>>>(nll, n, loss);
  return cuda_status(cudaGetLastError(), "dgx_softmax_nll");
}

dgx_status dgx_adamw(float* param, float* grad, float* m, float* v, long long n, float lr, float b1, float b2,
                     float eps, float wd, int step, const int* step_dev, void* stream) {
  DGX_FAULT_POINT("dgx_adamw");
  if (n < 0 || (!step_dev && step < 1)) return set_error(DGX_EINVAL, "dgx_adamw: n=%lld step=%d", n, step);
  if (n == 0) return DGX_OK;
  if (!param || !grad || !m || !v) return set_error(DGX_EINVAL, "dgx_adamw: null pointer");
  // Bias corrections in double on the host, as the reference (std::pow).
  const int t = step_dev ? 1 : step;
  const float bc1 = (float)(1.0 - std::pow((double)b1, t)), bc2 = (float)(1.0 - std::pow((double)b2, t));
  adamw_kernel<<<ew_grid(n), 256, 0, (cudaStream_t)stream>>>(param, grad, m, v, n, lr, b1, b2, eps, wd, bc1, bc2,
                                                             step_dev);
  return cuda_status(cudaGetLastError(), "dgx_adamw");
}

dgx_status dgx_colsum(const void* dy, int dy_type, float* db, int R, int N, int accumulate, void* stream) {
  DGX_FAULT_POINT("dgx_colsum");
  if (R < 0 || N <= 0) return set_error(DGX_EINVAL, "dgx_colsum: R=%d N=%d", R, N);
  if (dy_type != DGX_F32 && dy_type != DGX_BF16) return set_error(DGX_EINVAL, "dgx_colsum: type %d", dy_type);
  if (!dy || !db) return set_error(DGX_EINVAL, "dgx_colsum: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  constexpr int kMaxSlices = 128;
  float* part = (float*)library_scratch((size_t)kMaxSlices * N * sizeof(float), s);
  if (!part) return set_error(DGX_ENOMEM, "dgx_colsum: scratch");
  const int esz = dy_type == DGX_F32 ? 4 : 2, vec = 16 / esz;
  int slices = CS_SLICES;
  if (N % vec == 0 && ((uintptr_t)dy & 15) == 0) {
    const int cblocks = (N / vec + 31) / 32;
    slices = (2 * num_sms() + cblocks - 1) / cblocks;
    slices = slices < 1 ? 1 : (slices > kMaxSlices ? kMaxSlices : slices);
    dim3 grid(cblocks, slices);
    if (dy_type == DGX_F32)
      colsum_partial_vec_kernel<float><<<grid, 256, 0, s>>>((const float*)dy, part, R, N, slices);
    else
      colsum_partial_vec_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)dy, part, R, N, slices);
  } else {
    dim3 grid((N + 31) / 32, CS_SLICES);
    if (dy_type == DGX_F32)
      colsum_partial_kernel<float><<<grid, 256, 0, s>>>((const float*)dy, part, R, N);
    else
      colsum_partial_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>((const __nv_bfloat16*)dy, part, R, N);
  }
  colsum_final_kernel<<<(N + 31) / 32, 256, 0, s>>>(part, db, N, accumulate, slices);
  return cuda_status(cudaGetLastError(), "dgx_colsum");
}

dgx_status dgx_rows_to_heads(const void* src, int src_type, int ld, int col0, void* dst, int B, int S, int H, int D,
                             void* stream) {
  DGX_FAULT_POINT("dgx_rows_to_heads");
  if (B < 0 || S < 0 || H <= 0 || D <= 0 || D % 8 || col0 < 0 || col0 % 8 || ld % 8 || col0 + H * D > ld)
    return set_error(DGX_EINVAL, "dgx_rows_to_heads: sizes (D, col0 and ld must be multiples of 8)");
  if (src_type != DGX_F32 && src_type != DGX_BF16) return set_error(DGX_EINVAL, "dgx_rows_to_heads: type");
  const long long n = (long long)B * S * H * D;
  if (n == 0) return DGX_OK;
  if (n >= (1ll << 31)) return set_error(DGX_EINVAL, "dgx_rows_to_heads: %lld elements", n);
  if (!src || !dst || (((uintptr_t)src | (uintptr_t)dst) & 15))
    return set_error(DGX_EINVAL, "dgx_rows_to_heads: null or unaligned pointer");
  cudaStream_t s = (cudaStream_t)stream;
  if (src_type == DGX_F32)
    rows_to_heads_kernel<float><<<ew_grid(n / 8), 256, 0, s>>>((const float*)src, ld, col0, (__nv_bfloat16*)dst, B,
                                                               S, H, D);
  else
    rows_to_heads_kernel<__nv_bfloat16><<<ew_grid(n / 8), 256, 0, s>>>((const __nv_bfloat16*)src, ld, col0,
                                                                       (__nv_bfloat16*)dst, B, S, H, D);
  return cuda_status(cudaGetLastError(), "dgx_rows_to_heads");
}

dgx_status dgx_heads_to_rows(const void* src, void* dst, int ld, int col0, int B, int S, int H, int D, void* stream) {
  DGX_FAULT_POINT("dgx_heads_to_rows");
  if (B < 0 || S < 0 || H <= 0 || D <= 0 || D % 8 || col0 < 0 || col0 % 8 || ld % 8 || col0 + H * D > ld)
    return set_error(DGX_EINVAL, "dgx_heads_to_rows: sizes (D, col0 and ld must be multiples of 8)");
  const long long n = (long long)B * S * H * D;
  if (n == 0) return DGX_OK;
  if (n >= (1ll << 31)) return set_error(DGX_EINVAL, "dgx_heads_to_rows: %lld elements", n);
  if (!src || !dst || (((uintptr_t)src | (uintptr_t)dst) & 15))
    return set_error(DGX_EINVAL, "dgx_heads_to_rows: null or unaligned pointer");
  heads_to_rows_kernel<<<ew_grid(n / 8), 256, 0, (cudaStream_t)stream>>>((const __nv_bfloat16*)src, (__nv_bfloat16*)dst,
                                                                     ld, col0, B, S, H, D);
  return cuda_status(cudaGetLastError(), "dgx_heads_to_rows");
}

}  // extern "C"
