// Element-wise math of the FlashAttention softmax, balanced across pipes.
//
// On sm_100 the MUFU unit (ex2) retires 16 results per clock per SM, an
// eighth of the FMA pipe's rate, and at head dim 64 the softmax needs one
// exponential per 2*64 MMA FLOPs, so MUFU, not the tensor core, sets the
// speed. Part of the exponentials therefore run on the FMA/ALU pipes as a
// polynomial, and bf16 packing uses integer ops.
#pragma once
#include <stdint.h>

namespace dgx {

// Columns (out of 16) whose exp2 runs as a polynomial instead of on MUFU,
// for the forward and the backward kernel (measured on B200: the forward's
// exponential phase is MUFU-bound, the backward's is not).
#ifndef DGX_EXP_EMU_FWD
#define DGX_EXP_EMU_FWD 0
#endif
#ifndef DGX_EXP_EMU_BWD
#define DGX_EXP_EMU_BWD 0
#endif
// 1: pack bf16 pairs with integer ops (round half away from zero) instead of cvt.
#ifndef DGX_PACK_INT
#define DGX_PACK_INT 0
#endif

__device__ __forceinline__ float ex2_mufu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for softmax arguments (x <= ~8), Cody-Waite style: x = j + f with j the
// nearest integer (added to 1.5*2^23 so it lands in the low mantissa bits) and
// f in [-1/2, 1/2]; 2^f from a degree-3 polynomial whose coefficients were
// fitted for this file by iteratively reweighted least squares (Lawson) on
// Chebyshev nodes, minimising relative error (max 7.5e-5 in fp32, far below
// bf16's 3.9e-3 resolution); j is added to the exponent field with integer
// ops. x is clamped at -126, so fully masked entries give ~1e-38, not 0.
__device__ __forceinline__ float ex2_poly(float x) {
  x = fmaxf(x, -126.0f);
  const float t = x + 12582912.0f;
  const float f = x - (t - 12582912.0f);
  const float p = fmaf(fmaf(fmaf(0.05517166f, f, 0.24261113f), f, 0.69326097f), f, 0.99992806f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// exp2 for column c of a row: compile-time split between MUFU and polynomial
// (EMU of every 16 columns on the polynomial).
template <int C, int EMU>
__device__ __forceinline__ float ex2_col(float x) {
  if constexpr ((C & 15) < EMU)
    return ex2_poly(x);
  else
    return ex2_mufu(x);
}

__device__ __forceinline__ uint32_t pack_bf16x2_fast(float lo, float hi) {
#if DGX_PACK_INT
  const uint32_t a = __float_as_uint(lo) + 0x8000u, b = __float_as_uint(hi) + 0x8000u;
  return __byte_perm(a, b, 0x7632);
#else
  return pack_bf16x2(lo, hi);
#endif
}

}  // namespace dgx
