// Element conversion kernels behind dgx_convert (include/dgx.h).
#include <cuda_bf16.h>

#include "common.h"

namespace dgx {
namespace {

template <typename T>
__device__ __forceinline__ double load(const void* p, size_t i) {
  return (double)reinterpret_cast<const T*>(p)[i];
}
__device__ __forceinline__ double load_bf16(const void* p, size_t i) {
  return (double)__bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

// The reference's rounding on the raw fp32 bits (dream_to_bf16,
// runtime/nn/training.inc:1969-1976): add 0x7FFF plus the lowest kept bit,
// keep the high half. For finite values this is IEEE round-to-nearest-even;
// NaN and infinity go through the same integer steps, so every input gives
// the reference's bits (a NaN whose payload sits only in the dropped half
// becomes infinity, and the all-ones negative NaNs wrap to +0, as there).
__device__ __forceinline__ uint16_t bf16_bits_rne(float x) {
  uint32_t u = __float_as_uint(x);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

__global__ void convert_kernel(const void* src, int st, void* dst, int dt, size_t n, int acc) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    double v;
    switch (st) {
      case DGX_F64: v = load<double>(src, i); break;
      case DGX_F32: v = load<float>(src, i); break;
      case DGX_BF16: v = load_bf16(src, i); break;
      default: v = (double)reinterpret_cast<const int8_t*>(src)[i]; break;
    }
    switch (dt) {
      case DGX_F64: {
        double* d = reinterpret_cast<double*>(dst) + i;
        *d = acc ? *d + v : v;
        break;
      }
      case DGX_F32: {
        float* d = reinterpret_cast<float*>(dst) + i;
        *d = acc ? *d + (float)v : (float)v;
        break;
      }
      default: {
        // f64 -> bf16 goes through f32 first (round to nearest), as the
        // reference rounds an fp32 value (dream_to_bf16 takes a float).
        reinterpret_cast<uint16_t*>(dst)[i] = bf16_bits_rne((float)v);
        break;
      }
    }
  }
}

}  // namespace
}  // namespace dgx

using namespace dgx;

extern "C" dgx_status dgx_convert(const void* src, dgx_dtype src_type, void* dst, dgx_dtype dst_type, size_t n,
                                  int accumulate, void* stream) {  DGX_FAULT_POINT("dgx_convert");

  if (n == 0) return DGX_OK;
  if (!src || !dst) return set_error(DGX_EINVAL, "dgx_convert: null pointer");
  if (src_type < DGX_F32 || src_type > DGX_F64 || dst_type < DGX_F32 || dst_type > DGX_F64 || dst_type == DGX_I8)
    return set_error(DGX_EINVAL, "dgx_convert: types %d -> %d", src_type, dst_type);
  if (accumulate && dst_type == DGX_BF16) return set_error(DGX_EINVAL, "dgx_convert: accumulate into bf16");
  const int blocks = (int)((n + 255) / 256 < (size_t)(8 * num_sms()) ? (n + 255) / 256 : 8 * num_sms());
  convert_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(src, src_type, dst, dst_type, n, accumulate);
  return cuda_status(cudaGetLastError(), "dgx_convert");
}
