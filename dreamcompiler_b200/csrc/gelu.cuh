// GELU, tanh form, and its derivative on bf16 values: shared by the
// element-wise kernels (nn.cu) and the GEMM epilogue (gemm.cu), so the fused
// and the separate passes compute the same bits.
//
//   gelu(x)  = 0.5 x (1 + tanh(k (x + c x^3)))          runtime/io/builtins.inc:548-560
//   gelu'(x) = 0.5 (1 + t) + 0.5 x (1 - t^2) k (1 + 3 c x^2)   runtime/ops/autograd.inc:293-303
//
// with k = sqrt(2/pi), c = 0.044715, t = tanh(k (x + c x^3)). The hardware
// tanh (tanh.approx.f32, relative error about 2^-11) is far below the bf16
// output's 2^-8.
#pragma once
#include <stdint.h>

namespace dgx {

constexpr float kGeluK = 0.7978845608028654f;  // sqrt(2/pi)
constexpr float kGeluC = 0.044715f;

__device__ __forceinline__ float tanh_fast(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// The two bf16 halves of a packed pair, as fp32.
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

__device__ __forceinline__ float gelu_fast(float a) {
  const float t = tanh_fast(kGeluK * fmaf(kGeluC * a, a * a, a));
  return 0.5f * a * (1.f + t);
}
__device__ __forceinline__ float gelu_grad_fast(float a) {
  const float th = tanh_fast(kGeluK * fmaf(kGeluC * a, a * a, a));
  const float dinner = kGeluK * fmaf(3.f * kGeluC * a, a, 1.f);
  return 0.5f * (1.f + th) + 0.5f * a * (1.f - th * th) * dinner;
}

}  // namespace dgx
