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
                                  int accumulate, void* stream) {
  DGX_FAULT_POINT("dgx_convert");
  if (n == 0) return DGX_OK;
  if (!src || !dst) return set_error(DGX_EINVAL, "dgx_convert: null pointer");
  if (src_type < DGX_F32 || src_type > DGX_F64 || dst_type < DGX_F32 || dst_type > DGX_F64 || dst_type == DGX_I8)
    return set_error(DGX_EINVAL, "dgx_convert: types %d -> %d", src_type, dst_type);
  if (accumulate && dst_type == DGX_BF16) return set_error(DGX_EINVAL, "dgx_convert: accumulate into bf16");
  const int blocks = (int)((n + 255) / 256 < (size_t)(8 * num_sms()) ? (n + 255) / 256 : 8 * num_sms());
  convert_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(src, src_type, dst, dst_type, n, accumulate);
  return cuda_status(cudaGetLastError(), "dgx_convert");
}

// ---------------------------------------------------------------------------
// Content fingerprint of a device buffer, the same value a host computes
// over the same bytes (dgx_fingerprint in include/dgx.h). Word i (8 bytes,
// little endian; a tail of fewer than 8 bytes zero-padded into one last word)
// contributes splitmix64(w_i + (i + 1) * 0x9E3779B97F4A7C15) and the
// contributions are summed mod 2^64. splitmix64 is Vigna's published 64-bit
// finalizer; the sum makes the result independent of reduction order.
namespace dgx {
namespace {

__device__ __forceinline__ unsigned long long fp_mix(unsigned long long z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void fingerprint_kernel(const unsigned char* p, size_t bytes, unsigned long long* out) {
  const size_t words = bytes / 8, tail = bytes % 8;
  unsigned long long acc = 0;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < words; i += (size_t)gridDim.x * blockDim.x) {
    unsigned long long w;
    memcpy(&w, p + i * 8, 8);
    acc += fp_mix(w + (i + 1) * 0x9E3779B97F4A7C15ull);
  }
  if (tail && blockIdx.x == 0 && threadIdx.x == 0) {
    unsigned long long w = 0;
    for (size_t b = 0; b < tail; ++b) w |= (unsigned long long)p[words * 8 + b] << (8 * b);
    acc += fp_mix(w + (words + 1) * 0x9E3779B97F4A7C15ull);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0 && acc) atomicAdd(out, acc);
}

}  // namespace
}  // namespace dgx

extern "C" dgx_status dgx_fingerprint(const void* data, size_t bytes, unsigned long long* out, void* stream) {
  DGX_FAULT_POINT("dgx_fingerprint");
  if (!out || (bytes && !data)) return set_error(DGX_EINVAL, "dgx_fingerprint: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(out, 0, sizeof(unsigned long long), s);
  if (e != cudaSuccess) return cuda_status(e, "dgx_fingerprint");
  if (bytes == 0) return DGX_OK;
  const size_t words = bytes / 8 + 1;
  const int blocks = (int)((words + 255) / 256 < (size_t)(4 * num_sms()) ? (words + 255) / 256 : 4 * num_sms());
  fingerprint_kernel<<<blocks, 256, 0, s>>>(static_cast<const unsigned char*>(data), bytes, out);
  return cuda_status(cudaGetLastError(), "dgx_fingerprint");
}
