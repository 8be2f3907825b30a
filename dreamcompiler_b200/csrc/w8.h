// Internal interface between the int8 dense-layer translation units.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace dgx {

// Output options for the exported-network form (dgx_dense_q): one scale for
// every channel when the per-channel `scale` pointer is null, and ReLU.
struct W8Epi {
  float scale_all = 0.f;
  int relu = 0;
};

// Largest K for which the exact int32 accumulators of the tensor-core path
// cannot overflow: |w*q| <= 128*127 per product.
constexpr int kW8MaxK = 131072;

// Y[b,n] (and/or acc_out[b,n]) from int8 activation planes Xp[planes][B][K]
// and int8 weights W[N][K] on the tensor cores (tcgen05 kind::i8).
//   planes == 1: acc = sum_k Xp[0][b][k]*W[n][k] (exact int32);
//                acc_out <- acc, Y <- bias + scale[n]*rowscale[b]*acc.
//   planes == 3: the three int8 planes of an exact fixed-point split of fp32
//                activations (x = rowscale[b]*(q0 + q1/2^7 + q2/2^14 + r));
//                Y <- bias + scale[n]*rowscale[b]*(A0 + A1/2^7 + A2/2^14).
// K % 16 == 0, Xp and W 16-byte aligned. `after_producer` launches the
// kernel as a programmatic dependent of the kernel just issued on `s`: the
// weight stream starts before that kernel (which writes Xp and rowscale)
// has finished.
cudaError_t w8_tc_gemm(const int8_t* Xp, int planes, const int8_t* W, const float* scale, const float* bias,
                       const float* rowscale, float* Y, int32_t* acc_out, int B, int N, int K,
                       bool after_producer, cudaStream_t s, const W8Epi& epi = W8Epi());

// Launch `kern` as a programmatic dependent of the kernel issued before it on
// `s`: it may start while that kernel finishes, and must griddepcontrol.wait
// before it reads anything that kernel writes (the activation pre-passes do,
// so a layer's quantisation overlaps the tail of the layer before it).
template <typename... KArgs, typename... Args>
cudaError_t launch_dependent(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Split fp32 rows into the three int8 planes above (Xp[3][B][K]) and the
// power-of-two row scales. K % 16 == 0.
cudaError_t w8_split_planes(const float* X, int8_t* Xp, float* rowscale, int B, int K, cudaStream_t s);

}  // namespace dgx
