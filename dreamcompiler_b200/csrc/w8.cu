// int8 weight-only dense layer on sm_100a.
//
// Replaces the export-only int8 path of the reference: the quantiser and the
// emitted dense_q of export_c_header_int8 (runtime/nn/training.inc:3668-3752),
// y[j] = b[j] + sum_k scale*w[j,k]*x[k] in fp32, generalised to a per-output-
// channel scale and a batch of rows, and run on the device.
//
// Both modes run on the tensor cores (w8_tc.cu) whenever the weight rows can
// be fetched by TMA (K a multiple of 16):
//   mode 0 (W8A32): fp32 activations split exactly into three int8 planes,
//                   int32 sums combined exactly, y = b + scale*acc rounded once.
//   mode 1 (W8A8) : activations pre-quantised per row (dgx_quantize_rows_i8),
//                   exact int32 dot products, y = b + scale*sx*acc.
// The SIMT kernel below serves the other shapes: each warp owns two output
// channels and reads their weight rows with 16-byte loads, fp32 products and
// sums in mode 0, dp4a in mode 1.

#include "common.h"
#include "w8.h"

namespace dgx {

namespace {
constexpr int CPW = 2;       // output channels per warp
constexpr int WARPS = 8;
constexpr int BT = 8;        // batch rows per block
constexpr int KSTEP = 512;   // K consumed by one warp step (32 lanes x 16)

__device__ __forceinline__ float4 ld4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

template <int MODE>
__global__ void __launch_bounds__(256) w8_kernel(const void* __restrict__ X, const int8_t* __restrict__ W,
                                                 const float* __restrict__ scale, const float* __restrict__ bias,
                                                 const float* __restrict__ sx, float* __restrict__ Y,
                                                 int32_t* __restrict__ acc_out, int B, int N, int K, W8Epi epi) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = (blockIdx.x * WARPS + warp) * CPW;
  const int b0 = blockIdx.y * BT;
  const int nb = min(BT, B - b0);
  if (n0 >= N) return;
  float facc[CPW][BT];
  int iacc[CPW][BT];
#pragma unroll
  for (int c = 0; c < CPW; ++c)
#pragma unroll
    for (int b = 0; b < BT; ++b) {
      facc[c][b] = 0.f;
      iacc[c][b] = 0;
    }
  const bool vec = (K % 16) == 0;
  for (int k0 = 0; k0 < K; k0 += KSTEP) {
    const int k = k0 + lane * 16;
    if (k >= K) continue;
    int4 w[CPW];
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      if (n0 + c < N && vec) {
        w[c] = __ldg(reinterpret_cast<const int4*>(W + (size_t)(n0 + c) * K + k));
      } else {
        int8_t t[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) t[u] = (n0 + c < N && k + u < K) ? W[(size_t)(n0 + c) * K + k + u] : 0;
        w[c] = *reinterpret_cast<int4*>(t);
      }
    }
#pragma unroll
    for (int b = 0; b < BT; ++b) {
      if (b >= nb) break;
      if (MODE == 0) {
        const float* xr = reinterpret_cast<const float*>(X) + (size_t)(b0 + b) * K + k;
        float xv[16];
        if (vec) {
#pragma unroll
          for (int u = 0; u < 16; u += 4) *reinterpret_cast<float4*>(&xv[u]) = ld4(xr + u);
        } else {
#pragma unroll
          for (int u = 0; u < 16; ++u) xv[u] = (k + u < K) ? xr[u] : 0.f;
        }
#pragma unroll
        for (int c = 0; c < CPW; ++c) {
          const int8_t* wb = reinterpret_cast<const int8_t*>(&w[c]);
          float s = facc[c][b];
#pragma unroll
          for (int u = 0; u < 16; ++u) s = fmaf((float)wb[u], xv[u], s);
          facc[c][b] = s;
        }
      } else {
        const int8_t* xr = reinterpret_cast<const int8_t*>(X) + (size_t)(b0 + b) * K + k;
        int4 xv;
        if (vec) {
          xv = __ldg(reinterpret_cast<const int4*>(xr));
        } else {
          int8_t t[16];
#pragma unroll
          for (int u = 0; u < 16; ++u) t[u] = (k + u < K) ? xr[u] : 0;
          xv = *reinterpret_cast<int4*>(t);
        }
#pragma unroll
        for (int c = 0; c < CPW; ++c) {
          int s = iacc[c][b];
          s = __dp4a(w[c].x, xv.x, s);
          s = __dp4a(w[c].y, xv.y, s);
          s = __dp4a(w[c].z, xv.z, s);
          s = __dp4a(w[c].w, xv.w, s);
          iacc[c][b] = s;
        }
      }
    }
  }
#pragma unroll
  for (int c = 0; c < CPW; ++c) {
    const int n = n0 + c;
#pragma unroll
    for (int b = 0; b < BT; ++b) {
      if (MODE == 0) {
        float v = facc[c][b];
#pragma unroll
        for (int off = 16; off; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if (lane == 0 && n < N && b < nb) {
          const float y = (bias ? bias[n] : 0.f) + (scale ? scale[n] : epi.scale_all) * v;
          Y[(size_t)(b0 + b) * N + n] = epi.relu ? fmaxf(y, 0.f) : y;
        }
      } else {
        int v = iacc[c][b];
#pragma unroll
        for (int off = 16; off; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if (lane == 0 && n < N && b < nb) {
          if (acc_out) acc_out[(size_t)(b0 + b) * N + n] = v;
          if (Y) {
            const float y = (bias ? bias[n] : 0.f) + (scale ? scale[n] : epi.scale_all) * sx[b0 + b] * (float)v;
            Y[(size_t)(b0 + b) * N + n] = epi.relu ? fmaxf(y, 0.f) : y;
          }
        }
      }
    }
  }
}

// Per-row symmetric quantisation: sx = max|x|/127, q = clamp(round(x/sx)).
// Generic form: two passes over the row (any K, any alignment).
__global__ void quant_rows_kernel(const float* __restrict__ X, int8_t* __restrict__ Xq, float* __restrict__ sx,
                                  int K) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // the GEMM may start streaming weights
  asm volatile("griddepcontrol.wait;" ::: "memory");  // X may come from the kernel before (launched as its dependent)
  __shared__ float red[32];
  const int b = blockIdx.x;
  const float* x = X + (size_t)b * K;
  float m = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) m = fmaxf(m, fabsf(x[k]));
#pragma unroll
  for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (threadIdx.x == 0) red[0] = m;
  }
  __syncthreads();
  m = red[0];
  const float s = m > 0.f ? m / 127.f : 1.f;
  const float inv = 1.f / s;
  if (threadIdx.x == 0) sx[b] = s;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    float v = roundf(x[k] * inv);
    v = fminf(127.f, fmaxf(-127.f, v));
    Xq[(size_t)b * K + k] = (int8_t)v;
  }
}

// Same quantisation with the row held in registers: one read of the row,
// every load issued before the first use (K <= 1024*NV, K % 4 == 0, X 16-byte
// aligned). 256 threads, one CTA per row.
template <int NV>
__global__ void __launch_bounds__(256) quant_rows_reg_kernel(const float* __restrict__ X, int8_t* __restrict__ Xq,
                                                             float* __restrict__ sx, int K) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ float red[8];
  const int b = blockIdx.x;
  const float* x = X + (size_t)b * K;
  float4 v[NV];
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int k = (threadIdx.x + 256 * j) * 4;
    v[j] = k < K ? __ldg(reinterpret_cast<const float4*>(x + k)) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int j = 0; j < NV; ++j)
    m = fmaxf(m, fmaxf(fmaxf(fabsf(v[j].x), fabsf(v[j].y)), fmaxf(fabsf(v[j].z), fabsf(v[j].w))));
#pragma unroll
  for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  m = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w]);
  const float s = m > 0.f ? m / 127.f : 1.f;
  const float inv = 1.f / s;
  if (threadIdx.x == 0) sx[b] = s;
  auto q = [&](float f) { return (int8_t)fminf(127.f, fmaxf(-127.f, roundf(f * inv))); };
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int k = (threadIdx.x + 256 * j) * 4;
    if (k < K) {
      char4 c;
      c.x = q(v[j].x);
      c.y = q(v[j].y);
      c.z = q(v[j].z);
      c.w = q(v[j].w);
      *reinterpret_cast<char4*>(Xq + (size_t)b * K + k) = c;
    }
  }
}
}  // namespace

cudaError_t w8_simt(const void* X, const int8_t* W, const float* scale, const float* bias, const float* sx,
                    float* Y, int32_t* acc, int B, int N, int K, int mode, cudaStream_t s,
                    const W8Epi& epi = W8Epi()) {
  dim3 grid((N + WARPS * CPW - 1) / (WARPS * CPW), (B + BT - 1) / BT);
  if (mode == 0)
    w8_kernel<0><<<grid, 256, 0, s>>>(X, W, scale, bias, sx, Y, acc, B, N, K, epi);
  else
    w8_kernel<1><<<grid, 256, 0, s>>>(X, W, scale, bias, sx, Y, acc, B, N, K, epi);
  return cudaGetLastError();
}

cudaError_t quantize_rows(const float* X, int8_t* Xq, float* sx, int B, int K, cudaStream_t s) {
  const bool vec = K % 4 == 0 && (((uintptr_t)X | (uintptr_t)Xq) & 15) == 0;
  if (vec && K <= 1024) return launch_dependent(quant_rows_reg_kernel<1>, B, 256, s, X, Xq, sx, K);
  if (vec && K <= 2048) return launch_dependent(quant_rows_reg_kernel<2>, B, 256, s, X, Xq, sx, K);
  if (vec && K <= 4096) return launch_dependent(quant_rows_reg_kernel<4>, B, 256, s, X, Xq, sx, K);
  if (vec && K <= 8192) return launch_dependent(quant_rows_reg_kernel<8>, B, 256, s, X, Xq, sx, K);
  return launch_dependent(quant_rows_kernel, B, 256, s, X, Xq, sx, K);
}

// W8A8 from already quantised activations: tensor cores when TMA can fetch
// the rows, else the SIMT kernel.
cudaError_t w8a8_from_q(const int8_t* xq, const int8_t* W, const float* scale, const float* bias, const float* sx,
                        float* Y, int32_t* acc, int B, int N, int K, bool after_quant, cudaStream_t s) {
  if (K % 16 == 0 && K <= kW8MaxK)
    return w8_tc_gemm(xq, 1, W, scale, bias, sx, Y, acc, B, N, K, after_quant, s);
  return w8_simt(xq, W, scale, bias, sx, Y, acc, B, N, K, 1, s);
}

}  // namespace dgx

using namespace dgx;

extern "C" {

dgx_status dgx_quantize_rows_i8(const float* X, int8_t* Xq, float* sx, int B, int K, void* stream) {
  DGX_FAULT_POINT("dgx_quantize_rows_i8");
  if (B < 0 || K < 0) return set_error(DGX_EINVAL, "dgx_quantize_rows_i8: negative size");
  if (B == 0) return DGX_OK;
  if (!X || !Xq || !sx) return set_error(DGX_EINVAL, "dgx_quantize_rows_i8: null pointer");
  return cuda_status(quantize_rows(X, Xq, sx, B, K, (cudaStream_t)stream), "dgx_quantize_rows_i8");
}

dgx_status dgx_gemm_i8i32(const int8_t* Xq, const int8_t* W, int32_t* acc, int B, int N, int K, void* stream) {
  DGX_FAULT_POINT("dgx_gemm_i8i32");
  if (B < 0 || N < 0 || K < 0) return set_error(DGX_EINVAL, "dgx_gemm_i8i32: negative size");
  if (B == 0 || N == 0) return DGX_OK;
  if (!Xq || !W || !acc) return set_error(DGX_EINVAL, "dgx_gemm_i8i32: null pointer");
  if (((uintptr_t)Xq | (uintptr_t)W) & 15) return set_error(DGX_EINVAL, "dgx_gemm_i8i32: pointers must be 16-byte aligned");
  return cuda_status(w8a8_from_q(Xq, W, nullptr, nullptr, nullptr, nullptr, acc, B, N, K, false, (cudaStream_t)stream),
                     "dgx_gemm_i8i32");
}

}  // extern "C"

namespace dgx {

// The fp32-activation int8 layer of dgx_gemm_w8 and dgx_dense_q.
static dgx_status w8_layer(const char* op, const float* X, const int8_t* W, const float* scale, const float* bias,
                           float* Y, int B, int N, int K, int mode, const W8Epi& epi, cudaStream_t s) {
  if (mode == 0 && (K % 16 != 0 || K > kW8MaxK))
    return cuda_status(w8_simt(X, W, scale, bias, nullptr, Y, nullptr, B, N, K, 0, s, epi), op);
  // Library scratch: the int8 activation planes (3 for W8A32, 1 for W8A8)
  // and one fp32 scale per row.
  const int planes = mode == 0 ? 3 : 1;
  const size_t xq_bytes = ((size_t)planes * B * K + 255) & ~size_t(255);
  uint8_t* ws = (uint8_t*)library_scratch(xq_bytes + (size_t)B * sizeof(float), s);
  if (!ws) return set_error(DGX_ENOMEM, "%s: scratch", op);
  int8_t* xq = reinterpret_cast<int8_t*>(ws);
  float* rs = reinterpret_cast<float*>(ws + xq_bytes);
  if (mode == 0) {
    cudaError_t e = w8_split_planes(X, xq, rs, B, K, s);
    if (e != cudaSuccess) return cuda_status(e, op);
    return cuda_status(w8_tc_gemm(xq, 3, W, scale, bias, rs, Y, nullptr, B, N, K, true, s, epi), op);
  }
  cudaError_t e = quantize_rows(X, xq, rs, B, K, s);
  if (e != cudaSuccess) return cuda_status(e, op);
  return cuda_status(w8a8_from_q(xq, W, scale, bias, rs, Y, nullptr, B, N, K, true, s), op);
}

}  // namespace dgx

extern "C" {

dgx_status dgx_gemm_w8(const float* X, const int8_t* W, const float* scale, const float* bias, float* Y, int B,
                       int N, int K, int mode, void* stream) {
  DGX_FAULT_POINT("dgx_gemm_w8");
  if (B < 0 || N < 0 || K < 0) return set_error(DGX_EINVAL, "dgx_gemm_w8: negative size");
  if (mode != 0 && mode != 1) return set_error(DGX_EINVAL, "dgx_gemm_w8: mode %d", mode);
  if (B == 0 || N == 0) return DGX_OK;
  if (!X || !W || !scale || !Y) return set_error(DGX_EINVAL, "dgx_gemm_w8: null pointer");
  if (((uintptr_t)X | (uintptr_t)W) & 15) return set_error(DGX_EINVAL, "dgx_gemm_w8: X and W must be 16-byte aligned");
  return w8_layer("dgx_gemm_w8", X, W, scale, bias, Y, B, N, K, mode, W8Epi(), (cudaStream_t)stream);
}

dgx_status dgx_dense_q(const float* X, const int8_t* W, float scale, const float* scales, const float* bias,
                       float* Y, int B, int out_dim, int in_dim, int relu, void* stream) {
  DGX_FAULT_POINT("dgx_dense_q");
  if (B < 0 || out_dim < 0 || in_dim < 0) return set_error(DGX_EINVAL, "dgx_dense_q: negative size");
  if (B == 0 || out_dim == 0) return DGX_OK;
  if (!X || !W || !Y) return set_error(DGX_EINVAL, "dgx_dense_q: null pointer");
  if (((uintptr_t)X | (uintptr_t)W) & 15) return set_error(DGX_EINVAL, "dgx_dense_q: X and W must be 16-byte aligned");
  W8Epi epi;
  epi.scale_all = scale;
  epi.relu = relu ? 1 : 0;
  return w8_layer("dgx_dense_q", X, W, scales, bias, Y, B, out_dim, in_dim, 0, epi, (cudaStream_t)stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// dgx_gemm_w8a8_noalloc: the W8A8 layer without any device allocation.
//
// The activations quantised per row (int8) and their row scales need
// somewhere to live between the two kernels. dgx_gemm_w8 takes that space
// from the library's own buffer, which it grows with cudaMalloc on first use.
// Some callers cannot let a library allocate: a deployment that hands the
// whole device memory budget to its own pool at start-up, or a serving loop
// that must not call cudaMalloc once it runs (cudaMalloc can synchronise the
// device and take unbounded time). For them the space is this fixed array in
// the library's own device image, reserved when the library is loaded.
// ---------------------------------------------------------------------------
namespace {
// Largest problem the fixed array serves: B*K quantised activations and B rows.
constexpr size_t kNoAllocMaxActs = (size_t)4 << 20;  // 4,194,304 int8 values (4 MiB)
constexpr int kNoAllocMaxRows = 4096;                // row scales (16 KiB)
}  // namespace

// Every GPU that loads libdgx holds this array (4 MiB + 16 KiB) until the
// process exits. All calls share it and it keeps the last call's contents.
static __device__ __align__(256) unsigned char g_w8a8_noalloc_scratch[kNoAllocMaxActs + kNoAllocMaxRows * sizeof(float)];

namespace {
// In host code the array's name only stands for it; the kernels need its
// device address, looked up on every call with the caller's device current
// (the lookup allocates nothing and stays right after a device reset).
dgx_status noalloc_scratch(unsigned char** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_w8a8_noalloc_scratch);
  if (e != cudaSuccess) return dgx::cuda_status(e, "dgx_gemm_w8a8_noalloc: cudaGetSymbolAddress");
  *out = static_cast<unsigned char*>(p);
  return DGX_OK;
}
}  // namespace

extern "C" dgx_status dgx_gemm_w8a8_noalloc(const float* X, const int8_t* W, const float* scale, const float* bias,
                                            float* Y, int B, int N, int K, void* stream) {
  if (B < 0 || N < 0 || K < 0) return set_error(DGX_EINVAL, "dgx_gemm_w8a8_noalloc: negative size");
  if (B > kNoAllocMaxRows || (size_t)B * (size_t)K > kNoAllocMaxActs)
    return set_error(DGX_EINVAL,
                     "dgx_gemm_w8a8_noalloc: B=%d, K=%d exceeds the fixed scratch (B <= %d and B*K <= %zu); "
                     "use dgx_gemm_w8 for larger batches",
                     B, K, kNoAllocMaxRows, kNoAllocMaxActs);
  if (B == 0 || N == 0) return DGX_OK;
  if (!X || !W || !scale || !Y) return set_error(DGX_EINVAL, "dgx_gemm_w8a8_noalloc: null pointer");
  if (((uintptr_t)X | (uintptr_t)W) & 15)
    return set_error(DGX_EINVAL, "dgx_gemm_w8a8_noalloc: X and W must be 16-byte aligned");
  unsigned char* base = nullptr;
  const dgx_status st = noalloc_scratch(&base);
  if (st != DGX_OK) return st;
  // Nothing here has to start at zero: the quantiser overwrites the B*K
  // activations and B scales that the GEMM then reads.
  int8_t* xq = reinterpret_cast<int8_t*>(base);
  float* sx = reinterpret_cast<float*>(base + kNoAllocMaxActs);
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = quantize_rows(X, xq, sx, B, K, s);
  if (e != cudaSuccess) return cuda_status(e, "dgx_gemm_w8a8_noalloc quantize");
  return cuda_status(w8a8_from_q(xq, W, scale, bias, sx, Y, nullptr, B, N, K, true, s), "dgx_gemm_w8a8_noalloc");
}
