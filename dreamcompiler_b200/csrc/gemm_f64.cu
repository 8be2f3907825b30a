// Double-precision GEMM behind dgx_gemm_f64 (include/dgx.h).
//
// The reference computes `@` on its default (float64) tensors in f64
// (dream_gemm_d, runtime/ops/elementwise.inc:516-638) and its "matmul" /
// "linear" backward in f64 loops (runtime/ops/autograd.inc:91-125,
// :156-211). This kernel keeps that precision on the device: every product
// and sum is an f64 fused multiply-add (DFMA), no tensor-core splitting.
//
// Tiling: a 256-thread block owns a (16R x 16R) tile of C, each thread an
// R x R register block in four (R/2 x R/2) quadrants, so that a warp's
// fragment loads from shared memory are contiguous 16-byte vectors. K runs in
// steps of 8 through two shared-memory buffers: the next step's operands are
// fetched from global memory into registers while the current step's DFMAs
// run, then stored (transposed as the operand layout needs) into the other
// buffer. R = 8 (128 x 128 tiles) when those fill the SMs, else R = 4.
#include "common.h"

namespace dgx {
namespace {

constexpr int BK = 8;

template <int R>
struct F64Tile {
  static constexpr int BM = 16 * R;              // rows (and columns) of C per block
  static constexpr int LOADS = BM * BK / 256;     // elements of each operand a thread fetches per K step
};

struct F64Args {
  const double* A;
  const double* B;
  double* C;
  const double* bias;
  int M, N, K, lda, ldb, ldc, transA, transB, relu;
  double beta;
};

// Element (row r, column c) of op(X) for a tile fetch, zero outside.
__device__ __forceinline__ double ld_op(const double* X, int ld, int trans, int rows, int cols, int r, int c) {
  if (r >= rows || c >= cols) return 0.0;
  return trans ? __ldg(X + (size_t)c * ld + r) : __ldg(X + (size_t)r * ld + c);
}

template <int R>
__global__ void __launch_bounds__(256) gemm_f64_kernel(F64Args a) {
  constexpr int BM = F64Tile<R>::BM, L = F64Tile<R>::LOADS, H = R / 2;
  __shared__ __align__(16) double As[2][BK][BM];
  __shared__ __align__(16) double Bs[2][BK][BM];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BM;

  // Fetch pattern: along the operand's contiguous dimension, so a warp's
  // global loads are coalesced. A: op(A) is M x K; contiguous in k unless
  // transposed. B: op(B) is K x N; contiguous in n unless transposed.
  double ra[L], rb[L];
  auto fetch = [&](int k0) {
#pragma unroll
    for (int i = 0; i < L; ++i) {
      const int e = tid + 256 * i;
      int r, c;
      if (a.transA) { r = e % BM; c = e / BM; } else { r = e / BK; c = e % BK; }  // (m, k)
      ra[i] = ld_op(a.A, a.lda, a.transA, a.M, a.K, m0 + r, k0 + c);
      int kr, n;
      if (a.transB) { n = e / BK; kr = e % BK; } else { kr = e / BM; n = e % BM; }  // (k, n)
      rb[i] = a.transB ? ((n0 + n < a.N && k0 + kr < a.K) ? __ldg(a.B + (size_t)(n0 + n) * a.ldb + k0 + kr) : 0.0)
                       : ((k0 + kr < a.K && n0 + n < a.N) ? __ldg(a.B + (size_t)(k0 + kr) * a.ldb + n0 + n) : 0.0);
    }
  };
  auto stash = [&](int buf) {
#pragma unroll
    for (int i = 0; i < L; ++i) {
      const int e = tid + 256 * i;
      if (a.transA) As[buf][e / BM][e % BM] = ra[i];
      else As[buf][e % BK][e / BK] = ra[i];
      if (a.transB) Bs[buf][e % BK][e / BK] = rb[i];
      else Bs[buf][e / BM][e % BM] = rb[i];
    }
  };

  double acc[R][R];
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int j = 0; j < R; ++j) acc[i][j] = 0.0;

  const int nk = (a.K + BK - 1) / BK;
  fetch(0);
  stash(0);
  __syncthreads();
  for (int kt = 0; kt < nk; ++kt) {
    const int cur = kt & 1;
    if (kt + 1 < nk) fetch((kt + 1) * BK);
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      double fa[R], fb[R];
#pragma unroll
      for (int q = 0; q < 2; ++q)
#pragma unroll
        for (int i = 0; i < H; i += 2) {
          const double2 va = *reinterpret_cast<const double2*>(&As[cur][k][q * (BM / 2) + ty * H + i]);
          const double2 vb = *reinterpret_cast<const double2*>(&Bs[cur][k][q * (BM / 2) + tx * H + i]);
          fa[q * H + i] = va.x;
          fa[q * H + i + 1] = va.y;
          fb[q * H + i] = vb.x;
          fb[q * H + i + 1] = vb.y;
        }
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int j = 0; j < R; ++j) acc[i][j] = fma(fa[i], fb[j], acc[i][j]);
    }
    if (kt + 1 < nk) {
      stash(cur ^ 1);
      __syncthreads();
    }
  }

  // Epilogue: C = beta*C + acc (+ bias) (ReLU), f64 throughout.
#pragma unroll
  for (int i = 0; i < R; ++i) {
    const int m = m0 + (i / H) * (BM / 2) + ty * H + (i % H);
    if (m >= a.M) continue;
#pragma unroll
    for (int j = 0; j < R; ++j) {
      const int n = n0 + (j / H) * (BM / 2) + tx * H + (j % H);
      if (n >= a.N) continue;
      double* c = a.C + (size_t)m * a.ldc + n;
      double v = acc[i][j];
      if (a.beta != 0.0) v = fma(a.beta, *c, v);
      if (a.bias) v += a.bias[n];
      if (a.relu && v < 0.0) v = 0.0;
      *c = v;
    }
  }
}

}  // namespace
}  // namespace dgx

using namespace dgx;

extern "C" dgx_status dgx_gemm_f64(const double* A, const double* B, double* C, int M, int N, int K, int lda,
                                   int ldb, int ldc, int transA, int transB, const double* bias, int epilogue,
                                   double beta, void* stream) {
  DGX_FAULT_POINT("dgx_gemm_f64");
  if (M < 0 || N < 0 || K < 0) return set_error(DGX_EINVAL, "dgx_gemm_f64: negative size %dx%dx%d", M, N, K);
  if (M == 0 || N == 0) return DGX_OK;
  if (!C || (K > 0 && (!A || !B))) return set_error(DGX_EINVAL, "dgx_gemm_f64: null operand");
  if (epilogue < DGX_EPI_NONE || epilogue > DGX_EPI_RELU) return set_error(DGX_EINVAL, "dgx_gemm_f64: epilogue");
  if ((epilogue == DGX_EPI_BIAS || epilogue == DGX_EPI_BIAS_RELU) && !bias)
    return set_error(DGX_EINVAL, "dgx_gemm_f64: bias epilogue without bias");
  const int min_lda = transA ? M : K, min_ldb = transB ? K : N;
  if (lda < min_lda || ldb < min_ldb || ldc < N)
    return set_error(DGX_EINVAL, "dgx_gemm_f64: leading dimension too small (lda %d ldb %d ldc %d)", lda, ldb,
                     ldc);
  F64Args a{};
  a.A = A;
  a.B = B;
  a.C = C;
  a.bias = (epilogue == DGX_EPI_BIAS || epilogue == DGX_EPI_BIAS_RELU) ? bias : nullptr;
  a.M = M;
  a.N = N;
  a.K = K;
  a.lda = lda;
  a.ldb = ldb;
  a.ldc = ldc;
  a.transA = transA ? 1 : 0;
  a.transB = transB ? 1 : 0;
  a.relu = (epilogue == DGX_EPI_BIAS_RELU || epilogue == DGX_EPI_RELU);
  a.beta = beta;
  cudaStream_t s = (cudaStream_t)stream;
  const long long big_tiles = (long long)((M + 127) / 128) * ((N + 127) / 128);
  TimerScope timer(s);
  if (big_tiles >= num_sms()) {
    const dim3 grid((N + 127) / 128, (M + 127) / 128);
    gemm_f64_kernel<8><<<grid, 256, 0, s>>>(a);
  } else {
    const dim3 grid((N + 63) / 64, (M + 63) / 64);
    gemm_f64_kernel<4><<<grid, 256, 0, s>>>(a);
  }
  return cuda_status(cudaGetLastError(), "dgx_gemm_f64");
}
