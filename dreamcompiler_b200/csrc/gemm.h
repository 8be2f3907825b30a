// Internal interface of the GEMM kernels (not part of the public C ABI).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "common.h"
#include "sm100.cuh"

namespace dgx {

struct GemmArgs {
  int M, N, K;
  int lda, ldb, ldc;
  int transA, transB;      // A stored [K,M] / B stored [N,K]
  void* C;
  int c_bf16;              // output element type: 0 fp32, 1 bf16
  const float* bias;       // [N] or null
  int relu;
  float beta;              // C = beta*C + op(A).op(B) (+bias)
  uint32_t* err;           // device error word
  int tiles_m, tiles_n, group_m;  // filled by the launcher
  // Extra destinations with C's layout (pitch ldc) that receive the same
  // output, e.g. other GPUs' buffers through NVLink peer mappings (the
  // tensor-parallel all-gather fused into the epilogue). beta must be 0.
  // They take the TMA-store epilogue when C and every extra pointer are
  // 16-byte aligned (ExtraOutMaps), else per-thread stores.
  void* C_extra[7];
  int n_extra;
  // Output path of the epilogue: 0 per-thread stores (any layout, beta, extra
  // destinations); 1 TMA tensor store of staged tiles (beta = 0); 2 TMA
  // reduce-add of staged tiles (fp32 C, beta = 1, no ReLU); 3 raw fp32
  // partial sums of K slice z into a split-K workspace [splits][M][N] (the
  // bias / beta / ReLU epilogue then runs in the reduction kernel).
  int tma_out;
  int splits;  // K slices per output tile (1: no split)
  // Batched GEMM (dream_bmm): `batch` independent products in one launch,
  // operand / output b at A + b*sA, B + b*sB, C + b*sC (elements). 0 or 1:
  // a single product.
  int batch;
  long long sA, sB, sC;
};

// TMA maps of the extra destinations (GemmArgs::C_extra[e], C's geometry).
// With the TMA-store epilogue (tma_out 1) every staged box goes to C and then
// to each extra destination from the same shared-memory buffer: whole
// 128-byte rows per copy, the write size NVLink peer stores want.
struct ExtraOutMaps {
  CUtensorMap m[7];
};

// Whether every extra destination can take TMA stores (16-byte aligned).
inline bool extras_tma_aligned(const GemmArgs& a) {
  for (int e = 0; e < a.n_extra; ++e)
    if (reinterpret_cast<uintptr_t>(a.C_extra[e]) & 15) return false;
  return true;
}

// 2-SM bf16 kernel (gemm2.cu) and the algorithm switch.
bool gemm2_eligible(const GemmArgs& a, const void* A, const void* B);
cudaError_t gemm2_launch(const GemmArgs& args, const void* A, const void* B, cudaStream_t stream);
void gemm_set_algo(int algo);

// Bias of the 8 columns n..n+7 (zero past N): two 16-byte loads when the
// slice is whole and aligned, else guarded scalar loads.
__device__ __forceinline__ void load_bias8(const float* bias, int n, int N, float (&b)[8]) {
  if (n + 8 <= N && (reinterpret_cast<uintptr_t>(bias + n) & 15) == 0) {
    const float4 x = __ldg(reinterpret_cast<const float4*>(bias + n));
    const float4 y = __ldg(reinterpret_cast<const float4*>(bias + n + 4));
    b[0] = x.x; b[1] = x.y; b[2] = x.z; b[3] = x.w;
    b[4] = y.x; b[5] = y.y; b[6] = y.z; b[7] = y.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) b[i] = n + i < N ? bias[n + i] : 0.f;
  }
}
// Bring the bias columns [n0, n0 + width) of a tile into L1 (one 128-byte
// line per lane) while the epilogue still waits for the accumulator, so the
// per-chunk bias loads hit L1 instead of waiting on L2.
__device__ __forceinline__ void prefetch_bias_l1(const float* bias, int n0, int width, int N, int lane) {
  const int n = n0 + lane * 32;
  if (bias && lane * 32 < width && n < N) asm volatile("prefetch.global.L1 [%0];" ::"l"(bias + n));
}

__device__ __forceinline__ float gemm_finish(const GemmArgs& a, int n, float acc, float old) {
  float v = acc;
  if (a.beta != 0.f) v = fmaf(a.beta, old, v);
  if (a.bias) v += a.bias[n];
  if (a.relu) v = fmaxf(v, 0.f);
  return v;
}

__device__ __forceinline__ void gemm_store_one(const GemmArgs& a, int m, int n, float acc, long long boff = 0) {
  const long long off = boff + (long long)m * a.ldc + n;
  if (a.c_bf16) {
    __nv_bfloat16* c = reinterpret_cast<__nv_bfloat16*>(a.C) + off;
    const float old = a.beta != 0.f ? __bfloat162float(*c) : 0.f;
    *c = __float2bfloat16_rn(gemm_finish(a, n, acc, old));
    for (int e = 0; e < a.n_extra; ++e) reinterpret_cast<__nv_bfloat16*>(a.C_extra[e])[off] = *c;
  } else {
    float* c = reinterpret_cast<float*>(a.C) + off;
    const float old = a.beta != 0.f ? *c : 0.f;
    *c = gemm_finish(a, n, acc, old);
    for (int e = 0; e < a.n_extra; ++e) reinterpret_cast<float*>(a.C_extra[e])[off] = *c;
  }
}

// Store 32 consecutive accumulator columns [n0, n0+32) of row m (to C and
// to every extra destination); `boff` = the batch's element offset in C.
__device__ __forceinline__ void gemm_store_row32(const GemmArgs& a, int m, int n0, const float* v,
                                                 long long boff = 0) {
  const int nvalid = a.N - n0;
  const long long off = boff + (long long)m * a.ldc + n0;
  if (!a.c_bf16) {
    float* row = reinterpret_cast<float*>(a.C) + off;
    if (nvalid >= 32 && (reinterpret_cast<uintptr_t>(row) & 15) == 0) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        float4 old = make_float4(0.f, 0.f, 0.f, 0.f);
        if (a.beta != 0.f) old = *reinterpret_cast<const float4*>(row + j);
        float4 o;
        o.x = gemm_finish(a, n0 + j + 0, v[j + 0], old.x);
        o.y = gemm_finish(a, n0 + j + 1, v[j + 1], old.y);
        o.z = gemm_finish(a, n0 + j + 2, v[j + 2], old.z);
        o.w = gemm_finish(a, n0 + j + 3, v[j + 3], old.w);
        *reinterpret_cast<float4*>(row + j) = o;
        for (int e = 0; e < a.n_extra; ++e)
          *reinterpret_cast<float4*>(reinterpret_cast<float*>(a.C_extra[e]) + off + j) = o;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < nvalid) {
          const float old = a.beta != 0.f ? row[j] : 0.f;
          const float o = gemm_finish(a, n0 + j, v[j], old);
          row[j] = o;
          for (int e = 0; e < a.n_extra; ++e) reinterpret_cast<float*>(a.C_extra[e])[off + j] = o;
        }
    }
  } else {
    __nv_bfloat16* row = reinterpret_cast<__nv_bfloat16*>(a.C) + off;
    if (nvalid >= 32 && (reinterpret_cast<uintptr_t>(row) & 15) == 0) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        uint4 oldv = make_uint4(0, 0, 0, 0);
        if (a.beta != 0.f) oldv = *reinterpret_cast<const uint4*>(row + j);
        const __nv_bfloat16* ob = reinterpret_cast<const __nv_bfloat16*>(&oldv);
        uint32_t w[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float x0 = gemm_finish(a, n0 + j + 2 * h, v[j + 2 * h], __bfloat162float(ob[2 * h]));
          const float x1 = gemm_finish(a, n0 + j + 2 * h + 1, v[j + 2 * h + 1], __bfloat162float(ob[2 * h + 1]));
          w[h] = pack_bf16x2(x0, x1);
        }
        const uint4 o = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4*>(row + j) = o;
        for (int e = 0; e < a.n_extra; ++e)
          *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.C_extra[e]) + off + j) = o;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < nvalid) {
          const float old = a.beta != 0.f ? __bfloat162float(row[j]) : 0.f;
          const __nv_bfloat16 o = __float2bfloat16_rn(gemm_finish(a, n0 + j, v[j], old));
          row[j] = o;
          for (int e = 0; e < a.n_extra; ++e) reinterpret_cast<__nv_bfloat16*>(a.C_extra[e])[off + j] = o;
        }
    }
  }
}

int gemm_tc_supported(const GemmArgs& a, int esz, const void* A, const void* B);
// Runs a validated GemmArgs on the best kernel for it (api.cu).
dgx_status gemm_run(const GemmArgs& a, const void* A, const void* B, dgx_dtype ab_type, int f32_mode,
                    void* workspace, size_t workspace_bytes, cudaStream_t s);
cudaError_t gemm_bf16_tc(const GemmArgs& args, const void* A, const void* B, cudaStream_t s);
size_t gemm_f32_scratch_floats(const GemmArgs& a);
cudaError_t gemm_f32_3xtf32(const GemmArgs& args, const float* A, const float* B, float* scratch,
                            cudaStream_t s);
cudaError_t gemm_simt(const GemmArgs& args, const void* A, const void* B, int bf16_in, cudaStream_t s);

}  // namespace dgx
