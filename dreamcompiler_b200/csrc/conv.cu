// 2-D convolution through the tensor-core GEMM.
//
// Replaces dream_conv2d / dream_conv2d_padded (runtime/nn/conv.inc:12-187:
// per sample, im2col then kernel[Cout][Cin*KH*KW] . col[Cin*KH*KW][OH*OW],
// plus bias) and the "conv2d" backward (runtime/ops/autograd.inc:507-535:
// dK += dY . col^T, dX += col2im(K^T . dY)).
//
// Device form: one GEMM for the whole batch instead of one per sample. The
// im2col matrix is built positions-major, colT[N*OH*OW][Cin*KH*KW] (K
// contiguous, the tensor cores' K-major operand), so
//   forward   YT[N*OHW][Cout]   = colT . K^T        (+ bias per column)
//   backward  dK[Cout][CKK]    += dYT^T . colT      (K = N*OHW: split-K)
//             dcolT[N*OHW][CKK] = dYT . K
// and the NCHW tensors are moved in and out of the positions-major layout
// by a tiled transpose (which also adds the bias). col2im is a gather: each
// input element sums its KH*KW window taps in a fixed order, no atomics.
// Operands are fp32 (3xTF32 GEMMs) or bf16 (kind::f16) as `ab_type` says;
// results and gradients are fp32.
#include <cuda_bf16.h>

#include "common.h"
#include "gemm.h"

namespace dgx {
namespace {

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

struct ConvGeom {
  int N, Cin, H, W, Cout, KH, KW, pad, stride, OH, OW;
  int ckk;   // Cin*KH*KW
  int ldk;   // row pitch of colT / dcolT / the kernel copy (ckk rounded up to 8)
  int ldo;   // row pitch of YT / dYT (Cout rounded up to 8)
};

// colT[p][r] = x[n][ci][oh*s - pad + kh][ow*s - pad + kw] (0 outside the
// image, and 0 in the pitch padding r >= ckk), p = n*OH*OW + oh*OW + ow,
// r = (ci*KH + kh)*KW + kw. One warp per position row p (its image
// coordinates computed once), lanes along r: coalesced stores, and the
// gathered loads of neighbouring taps hit the same lines in L1/L2.
template <typename T>
__global__ void im2col_rows_kernel(const float* __restrict__ x, T* __restrict__ col, ConvGeom g) {
  const int rows = g.N * g.OH * g.OW;
  const int kk = g.KH * g.KW, ohw = g.OH * g.OW;
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int p = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; p < rows; p += warps) {
    const int n = p / ohw, rem = p - n * ohw;
    const int oh = rem / g.OW, ow = rem - oh * g.OW;
    const int h0 = oh * g.stride - g.pad, w0 = ow * g.stride - g.pad;
    const float* xn = x + (size_t)n * g.Cin * g.H * g.W;
    T* out = col + (size_t)p * g.ldk;
    for (int r = lane; r < g.ldk; r += 32) {
      float v = 0.f;
      if (r < g.ckk) {
        const int ci = r / kk, t = r - ci * kk;
        const int kh = t / g.KW, kw = t - kh * g.KW;
        const int h = h0 + kh, w = w0 + kw;
        if (h >= 0 && h < g.H && w >= 0 && w < g.W) v = __ldg(xn + ((size_t)ci * g.H + h) * g.W + w);
      }
      out[r] = from_f32<T>(v);
    }
  }
}

// Batched transpose of the last two dims: out[b][c][r] (+)= in[b][r][c] (+ bias[c]).
// 32x32 shared-memory tiles keep both sides coalesced.
template <typename Tout>
__global__ void transpose_kernel(const float* __restrict__ in, Tout* __restrict__ out, int R, int Cc, int ld_in,
                                 int ld_out, long long s_in, long long s_out, const float* __restrict__ bias,
                                 int accumulate) {
  __shared__ float tile[32][33];
  const int b = blockIdx.z;
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  const float* ib = in + (size_t)b * s_in;
  Tout* ob = out + (size_t)b * s_out;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  for (int i = ty; i < 32; i += 8) {
    const int r = r0 + i, c = c0 + tx;
    float v = 0.f;
    if (r < R && c < Cc) v = ib[(size_t)r * ld_in + c] + (bias ? bias[c] : 0.f);
    tile[i][tx] = v;
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int c = c0 + i, r = r0 + tx;
    if (c < Cc && r < R) {
      Tout* o = ob + (size_t)c * ld_out + r;
      const float v = tile[tx][i];
      if constexpr (sizeof(Tout) == 4) {
        *o = accumulate ? *o + v : v;
      } else {
        *o = from_f32<Tout>(v);
      }
    }
  }
}

// dX[n][ci][h][w] (+)= sum over the window taps (kh, kw) whose output
// position (oh, ow) = ((h + pad - kh)/s, (w + pad - kw)/s) is integral and in
// range of dcolT[n*OHW + oh*OW + ow][(ci*KH + kh)*KW + kw]; taps in order.
// blockIdx.y walks the (n, ci) planes, threads the H*W pixels of a plane.
__global__ void col2im_gather_kernel(const float* __restrict__ dcol, float* __restrict__ dx, ConvGeom g,
                                     int accumulate) {
  const int kk = g.KH * g.KW, hw_n = g.H * g.W, planes = g.N * g.Cin;
  for (int pc = blockIdx.y; pc < planes; pc += gridDim.y) {
    const int n = pc / g.Cin, ci = pc - n * g.Cin;
    const float* dc = dcol + (size_t)n * g.OH * g.OW * g.ldk + ci * kk;
    float* dxp = dx + (size_t)pc * hw_n;
    for (int hw = blockIdx.x * blockDim.x + threadIdx.x; hw < hw_n; hw += gridDim.x * blockDim.x) {
      const int h = hw / g.W, w = hw - h * g.W;
      float s = 0.f;
      for (int kh = 0; kh < g.KH; ++kh) {
        const int hh = h + g.pad - kh;
        if (hh < 0 || hh % g.stride) continue;
        const int oh = hh / g.stride;
        if (oh >= g.OH) continue;
        for (int kw = 0; kw < g.KW; ++kw) {
          const int ww = w + g.pad - kw;
          if (ww < 0 || ww % g.stride) continue;
          const int ow = ww / g.stride;
          if (ow >= g.OW) continue;
          s += dc[(size_t)(oh * g.OW + ow) * g.ldk + kh * g.KW + kw];
        }
      }
      dxp[hw] = accumulate ? dxp[hw] + s : s;
    }
  }
}

// Kernel weights [Cout][ckk] (fp32) into the padded GEMM operand [Cout][ldk].
template <typename T>
__global__ void pad_rows_kernel(const float* __restrict__ src, T* __restrict__ dst, int rows, int cols, int ld) {
  const long long total = (long long)rows * ld;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / ld), c = (int)(i % ld);
    dst[i] = from_f32<T>(c < cols ? src[(size_t)r * cols + c] : 0.f);
  }
}

inline int round8(int v) { return (v + 7) & ~7; }

dgx_status make_geom(const char* op, int N, int Cin, int H, int W, int Cout, int KH, int KW, int pad, int stride,
                     ConvGeom* g) {
  if (N < 0 || N > 65535 || Cin <= 0 || H <= 0 || W <= 0 || Cout <= 0 || KH <= 0 || KW <= 0 || pad < 0 ||
      stride <= 0)
    return set_error(DGX_EINVAL, "%s: bad geometry N=%d Cin=%d H=%d W=%d Cout=%d K=%dx%d pad=%d stride=%d", op, N, Cin,
                     H, W, Cout, KH, KW, pad, stride);
  g->N = N;
  g->Cin = Cin;
  g->H = H;
  g->W = W;
  g->Cout = Cout;
  g->KH = KH;
  g->KW = KW;
  g->pad = pad;
  g->stride = stride;
  g->OH = (H + 2 * pad - KH) / stride + 1;
  g->OW = (W + 2 * pad - KW) / stride + 1;
  if (H + 2 * pad < KH || W + 2 * pad < KW || g->OH <= 0 || g->OW <= 0)
    return set_error(DGX_EINVAL, "%s: kernel %dx%d larger than the padded %dx%d input", op, KH, KW, H + 2 * pad,
                     W + 2 * pad);
  const long long ckk = (long long)Cin * KH * KW;
  if (ckk > (1 << 30)) return set_error(DGX_EINVAL, "%s: Cin*KH*KW too large", op);
  if ((long long)N * g->OH * g->OW >= (1LL << 31) || (long long)N * Cin >= (1LL << 31) || (long long)H * W >= (1LL << 31))
    return set_error(DGX_EINVAL, "%s: too many output positions", op);
  g->ckk = (int)ckk;
  g->ldk = round8(g->ckk);
  g->ldo = round8(Cout);
  return DGX_OK;
}

int blocks_for(long long work, int per_block) {
  long long b = (work + per_block - 1) / per_block;
  const long long cap = (long long)num_sms() * 16;
  return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace
}  // namespace dgx

using namespace dgx;

extern "C" {

size_t dgx_conv2d_workspace_size(int N, int Cin, int H, int W, int Cout, int KH, int KW, int pad, int stride,
                                 dgx_dtype ab_type) {
  ConvGeom g;
  if (make_geom("dgx_conv2d_workspace_size", N, Cin, H, W, Cout, KH, KW, pad, stride, &g) != DGX_OK) return 0;
  const size_t esz = ab_type == DGX_BF16 ? 2 : 4;
  const size_t rows = (size_t)N * g.OH * g.OW;
  // colT (operand type) + YT / dYT (fp32 forward, operand type backward) +
  // dcolT (fp32) + the padded kernel copy (operand type).
  return ((rows * g.ldk * esz + 255) & ~size_t(255)) + ((rows * g.ldo * 4 + 255) & ~size_t(255)) +
         ((rows * g.ldk * 4 + 255) & ~size_t(255)) + (((size_t)g.Cout * g.ldk * esz + 255) & ~size_t(255));
}

dgx_status dgx_conv2d_fwd(const float* X, const float* Kw, const float* bias, float* Y, int N, int Cin, int H, int W,
                          int Cout, int KH, int KW, int pad, int stride, dgx_dtype ab_type, void* stream) {
  DGX_FAULT_POINT("dgx_conv2d_fwd");
  ConvGeom g;
  dgx_status st = make_geom("dgx_conv2d_fwd", N, Cin, H, W, Cout, KH, KW, pad, stride, &g);
  if (st != DGX_OK) return st;
  if (ab_type != DGX_F32 && ab_type != DGX_BF16) return set_error(DGX_EINVAL, "dgx_conv2d_fwd: ab_type %d", ab_type);
  if (N == 0) return DGX_OK;
  if (!X || !Kw || !Y) return set_error(DGX_EINVAL, "dgx_conv2d_fwd: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  const size_t need = dgx_conv2d_workspace_size(N, Cin, H, W, Cout, KH, KW, pad, stride, ab_type);
  char* ws = (char*)library_scratch_slot(kScratchConv, need, s);
  if (!ws) return set_error(DGX_ENOMEM, "dgx_conv2d_fwd: cannot allocate %zu bytes of scratch", need);
  const size_t esz = ab_type == DGX_BF16 ? 2 : 4;
  const long long rows = (long long)N * g.OH * g.OW;
  void* colT = ws;
  float* yT = (float*)(ws + ((rows * g.ldk * esz + 255) & ~size_t(255)));
  void* kpad = (char*)yT + ((rows * g.ldo * 4 + 255) & ~size_t(255)) + ((rows * g.ldk * 4 + 255) & ~size_t(255));
  const int ib = blocks_for(rows * 32, 256);  // a warp per position row
  if (ab_type == DGX_BF16) {
    im2col_rows_kernel<__nv_bfloat16><<<ib, 256, 0, s>>>(X, (__nv_bfloat16*)colT, g);
    pad_rows_kernel<__nv_bfloat16><<<blocks_for((long long)Cout * g.ldk, 256), 256, 0, s>>>(
        Kw, (__nv_bfloat16*)kpad, Cout, g.ckk, g.ldk);
  } else {
    im2col_rows_kernel<float><<<ib, 256, 0, s>>>(X, (float*)colT, g);
    pad_rows_kernel<float><<<blocks_for((long long)Cout * g.ldk, 256), 256, 0, s>>>(Kw, (float*)kpad, Cout, g.ckk,
                                                                                   g.ldk);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, "dgx_conv2d_fwd im2col");
  // YT[rows][Cout] = colT . K^T (K stored [Cout][ldk]: the [N][K] operand).
  st = dgx_gemm(colT, kpad, yT, (int)rows, Cout, g.ckk, g.ldk, g.ldk, g.ldo, 0, 1, ab_type, DGX_F32, DGX_F32_3XTF32,
                nullptr, DGX_EPI_NONE, 0.f, nullptr, 0, stream);
  if (st != DGX_OK) return st;
  // Y[n][co][p] = YT[n*OHW + p][co] + bias[co]
  const int ohw = g.OH * g.OW;
  dim3 tg((Cout + 31) / 32, (ohw + 31) / 32, N);
  transpose_kernel<float><<<tg, 256, 0, s>>>(yT, Y, ohw, Cout, g.ldo, ohw, (long long)ohw * g.ldo,
                                             (long long)Cout * ohw, bias, 0);
  return cuda_status(cudaGetLastError(), "dgx_conv2d_fwd");
}

dgx_status dgx_conv2d_bwd(const float* X, const float* Kw, const float* dY, float* dX, float* dK, int N, int Cin, int H,
                          int W, int Cout, int KH, int KW, int pad, int stride, dgx_dtype ab_type, int accumulate,
                          void* stream) {
  DGX_FAULT_POINT("dgx_conv2d_bwd");
  ConvGeom g;
  dgx_status st = make_geom("dgx_conv2d_bwd", N, Cin, H, W, Cout, KH, KW, pad, stride, &g);
  if (st != DGX_OK) return st;
  if (ab_type != DGX_F32 && ab_type != DGX_BF16) return set_error(DGX_EINVAL, "dgx_conv2d_bwd: ab_type %d", ab_type);
  if (N == 0) return DGX_OK;
  if (!X || !Kw || !dY || (!dX && !dK)) return set_error(DGX_EINVAL, "dgx_conv2d_bwd: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  const size_t need = dgx_conv2d_workspace_size(N, Cin, H, W, Cout, KH, KW, pad, stride, ab_type);
  char* ws = (char*)library_scratch_slot(kScratchConv, need, s);
  if (!ws) return set_error(DGX_ENOMEM, "dgx_conv2d_bwd: cannot allocate %zu bytes of scratch", need);
  const size_t esz = ab_type == DGX_BF16 ? 2 : 4;
  const long long rows = (long long)N * g.OH * g.OW;
  const int ohw = g.OH * g.OW;
  void* colT = ws;
  void* dyT = ws + ((rows * g.ldk * esz + 255) & ~size_t(255));
  float* dcolT = (float*)((char*)dyT + ((rows * g.ldo * 4 + 255) & ~size_t(255)));
  void* kpad = (char*)dcolT + ((rows * g.ldk * 4 + 255) & ~size_t(255));
  // dYT[n*OHW + p][co] = dY[n][co][p], in the operand type (the pitch
  // padding columns are never read: the GEMM's K / M extents stop at Cout).
  dim3 tg((ohw + 31) / 32, (Cout + 31) / 32, N);
  if (ab_type == DGX_BF16)
    transpose_kernel<__nv_bfloat16><<<tg, 256, 0, s>>>(dY, (__nv_bfloat16*)dyT, Cout, ohw, ohw, g.ldo,
                                                       (long long)Cout * ohw, (long long)ohw * g.ldo, nullptr, 0);
  else
    transpose_kernel<float><<<tg, 256, 0, s>>>(dY, (float*)dyT, Cout, ohw, ohw, g.ldo, (long long)Cout * ohw,
                                               (long long)ohw * g.ldo, nullptr, 0);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, "dgx_conv2d_bwd transpose");
  if (dK) {
    // dK[Cout][ckk] (+)= dYT^T . colT: A = dYT stored [K = rows][M = Cout].
    const int ib = blocks_for(rows * 32, 256);  // a warp per position row
    if (ab_type == DGX_BF16)
      im2col_rows_kernel<__nv_bfloat16><<<ib, 256, 0, s>>>(X, (__nv_bfloat16*)colT, g);
    else
      im2col_rows_kernel<float><<<ib, 256, 0, s>>>(X, (float*)colT, g);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e, "dgx_conv2d_bwd im2col");
    st = dgx_gemm(dyT, colT, dK, Cout, g.ckk, (int)rows, g.ldo, g.ldk, g.ckk, 1, 0, ab_type, DGX_F32, DGX_F32_3XTF32,
                  nullptr, DGX_EPI_NONE, accumulate ? 1.f : 0.f, nullptr, 0, stream);
    if (st != DGX_OK) return st;
  }
  if (dX) {
    // dcolT[rows][ckk] = dYT . K (K stored [Cout][ldk]: the [K][N] operand), then the gather.
    if (ab_type == DGX_BF16)
      pad_rows_kernel<__nv_bfloat16><<<blocks_for((long long)Cout * g.ldk, 256), 256, 0, s>>>(
          Kw, (__nv_bfloat16*)kpad, Cout, g.ckk, g.ldk);
    else
      pad_rows_kernel<float><<<blocks_for((long long)Cout * g.ldk, 256), 256, 0, s>>>(Kw, (float*)kpad, Cout, g.ckk,
                                                                                     g.ldk);
    st = dgx_gemm(dyT, kpad, dcolT, (int)rows, g.ckk, Cout, g.ldo, g.ldk, g.ldk, 0, 0, ab_type, DGX_F32,
                  DGX_F32_3XTF32, nullptr, DGX_EPI_NONE, 0.f, nullptr, 0, stream);
    if (st != DGX_OK) return st;
    const int hw = H * W, planes = N * Cin;
    dim3 cg((hw + 255) / 256 < 64 ? (hw + 255) / 256 : 64, planes < 65535 ? planes : 65535);
    col2im_gather_kernel<<<cg, 256, 0, s>>>(dcolT, dX, g, accumulate);
  }
  return cuda_status(cudaGetLastError(), "dgx_conv2d_bwd");
}

}  // extern "C"
