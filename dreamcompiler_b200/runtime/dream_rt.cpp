// Dream runtime ops of the GEMM / FlashAttention hot path on top of libdgx.
//
// Mirrors the reference runtime's interface for these ops (heellowdsf/
// DreamCompiler runtime/): tensor_matmul (ops/elementwise.inc:971-1213),
// dream_linear[_relu] (:1432-1521), dream_bmm (:1218-1252),
// dream_flash_attention (nn/training.inc:284-401), dream_tp_matmul_column
// (:1604-1630) and the backward branches for them (ops/autograd.inc). The
// OpenCL/cuBLAS auto-dispatch and the CPU/GPU threshold (backend/gpu.inc:
// 293-361) are gone: every op runs its sm_100a kernel through the C ABI.
//
// Precision: f64 and f32 tensors run the 3xTF32 GEMM (fp32-level error);
// after dream_enable_fp16() GEMMs take bf16 operands as the reference's
// fp16 GemmEx switch did; FlashAttention computes in bf16 with fp32 softmax
// statistics. Host storage stays f64 so every reader sees `data` as before.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <unordered_set>
#include <vector>

#include "dgx.h"
#include "dream_b200.h"

namespace {

enum class Fn { None, Matmul, Linear, LinearRelu, Bmm, Flash, Conv, Mul, Sum };

struct FlashSaved;

// Runtime-private layout after the LLVM-visible prefix (runtime/runtime.h:49-54).
struct TensorImpl {
  double* data;
  double* grad;
  int size;
  int d0, d1, d2, d3;
  // private
  int refcount;
  int dtype;      // 0 f64, 1 f32 mirror live
  float* fdata;
  Fn fn;
  TensorImpl* parents[3];
  int nparents;
  int meta[8];    // op dimensions (B,S,dk,causal / batch,M,K,N / H,W,KH,KW,pad,stride,Cin,Cout)
  FlashSaved* flash;
};

cudaStream_t g_stream = nullptr;
bool g_ready = false;
bool g_use_bf16 = false;

bool ensure_device() {
  if (g_ready) return true;
  const char* dev = std::getenv("DGX_DEVICE");
  if (dgx_init(dev ? std::atoi(dev) : 0) != DGX_OK) {
    std::fprintf(stderr, "RUNTIME ERROR: libdgx device init failed: %s\n", dgx_last_error());
    return false;
  }
  if (cudaStreamCreateWithFlags(&g_stream, cudaStreamNonBlocking) != cudaSuccess) return false;
  g_ready = true;
  return true;
}

void report(const char* op, const char* msg) {
  std::fprintf(stderr, "RUNTIME ERROR in %s: %s\n", op, msg);
  std::fflush(stderr);
}

// Device buffer scoped to one op (stream-ordered allocator).
struct DevBuf {
  void* p = nullptr;
  explicit DevBuf(size_t bytes) {
    if (bytes && cudaMallocAsync(&p, bytes, g_stream) != cudaSuccess) p = nullptr;
  }
  ~DevBuf() {
    if (p) cudaFreeAsync(p, g_stream);
  }
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  template <typename T>
  T* as() const {
    return static_cast<T*>(p);
  }
};

struct FlashSaved {
  void* q = nullptr;  // bf16 Q, K, V, O and fp32 LSE kept for the backward
  void* k = nullptr;
  void* v = nullptr;
  void* o = nullptr;
  float* lse = nullptr;
  ~FlashSaved() {
    for (void* p : {q, k, v, o, (void*)lse})
      if (p) cudaFree(p);
  }
};

TensorImpl* impl(Tensor* t) { return reinterpret_cast<TensorImpl*>(t); }
Tensor* pub(TensorImpl* t) { return reinterpret_cast<Tensor*>(t); }

TensorImpl* new_tensor(int d0, int d1, int d2, int d3) {
  if (d0 < 0 || d1 < 0 || d2 < 0 || d3 < 0) {
    report("alloc", "negative tensor dimension");
    d0 = d1 = d2 = d3 = 1;
  }
  long long sz = (long long)d0 * d1 * d2 * d3;
  if (sz > 500000000LL) {  // the reference's MAX_ELEMS (core/tensor.inc:154)
    report("alloc", "tensor too large");
    d0 = d1 = d2 = d3 = 1;
    sz = 1;
  }
  if (sz <= 0) sz = 1;
  TensorImpl* t = new TensorImpl();
  t->data = static_cast<double*>(std::calloc((size_t)sz, sizeof(double)));
  t->grad = static_cast<double*>(std::calloc((size_t)sz, sizeof(double)));
  t->size = (int)sz;
  t->d0 = d0;
  t->d1 = d1;
  t->d2 = d2;
  t->d3 = d3;
  t->refcount = 1;
  return t;
}

void set_parents(TensorImpl* out, Fn fn, std::initializer_list<TensorImpl*> ps) {
  out->fn = fn;
  out->nparents = 0;
  for (TensorImpl* p : ps) {
    p->refcount++;
    out->parents[out->nparents++] = p;
  }
}

// Host f64 (or the live f32 mirror) -> device buffer of `type`.
bool upload(const TensorImpl* t, void* dst, dgx_dtype type) {
  const size_t n = (size_t)t->size;
  if (t->dtype == 1 && t->fdata) {
    if (type == DGX_F32) return cudaMemcpyAsync(dst, t->fdata, n * 4, cudaMemcpyHostToDevice, g_stream) == cudaSuccess;
    DevBuf tmp(n * 4);
    if (!tmp.p || cudaMemcpyAsync(tmp.p, t->fdata, n * 4, cudaMemcpyHostToDevice, g_stream) != cudaSuccess)
      return false;
    return dgx_convert(tmp.p, DGX_F32, dst, type, n, 0, g_stream) == DGX_OK;
  }
  DevBuf tmp(n * 8);
  if (!tmp.p || cudaMemcpyAsync(tmp.p, t->data, n * 8, cudaMemcpyHostToDevice, g_stream) != cudaSuccess) return false;
  return dgx_convert(tmp.p, DGX_F64, dst, type, n, 0, g_stream) == DGX_OK;
}

// Device buffer of `type` -> host f64 array (overwrite or add).
bool download(const void* src, dgx_dtype type, double* host, size_t n, bool add) {
  DevBuf tmp(n * 8);
  if (!tmp.p) return false;
  if (add) {
    if (cudaMemcpyAsync(tmp.p, host, n * 8, cudaMemcpyHostToDevice, g_stream) != cudaSuccess) return false;
  }
  if (dgx_convert(src, type, tmp.p, DGX_F64, n, add ? 1 : 0, g_stream) != DGX_OK) return false;
  if (cudaMemcpyAsync(host, tmp.p, n * 8, cudaMemcpyDeviceToHost, g_stream) != cudaSuccess) return false;
  return cudaStreamSynchronize(g_stream) == cudaSuccess;
}

dgx_dtype gemm_type() { return g_use_bf16 ? DGX_BF16 : DGX_F32; }
size_t esize(dgx_dtype t) { return t == DGX_BF16 ? 2 : 4; }

// C(f32, device) = op(A) op(B) with operands uploaded from host tensors.
bool device_gemm(const void* A, const void* B, float* C, int M, int N, int K, int transA, int transB, dgx_dtype ab,
                 const float* bias, int epi, float beta) {
  const int lda = transA ? M : K, ldb = transB ? K : N;
  return dgx_gemm(A, B, C, M, N, K, lda, ldb, N, transA, transB, ab, DGX_F32, DGX_F32_3XTF32, bias, epi, beta,
                  nullptr, 0, g_stream) == DGX_OK;
}

void free_tensor(TensorImpl* t);

}  // namespace

extern "C" {

Tensor* alloc_tensor(int d0, int d1, int d2, int d3) { return pub(new_tensor(d0, d1, d2, d3)); }

Tensor* create_scalar(double v) {
  TensorImpl* t = new_tensor(1, 1, 1, 1);
  t->data[0] = v;
  return pub(t);
}

Tensor* tensor_incref(Tensor* t) {
  if (t) impl(t)->refcount++;
  return t;
}

Tensor* tensor_decref(Tensor* t) {
  if (!t) return nullptr;
  TensorImpl* ti = impl(t);
  if (--ti->refcount <= 0) free_tensor(ti);
  return nullptr;
}

Tensor* tensor_get_grad(Tensor* t) {
  if (!t) return create_scalar(0.0);
  TensorImpl* ti = impl(t);
  TensorImpl* g = new_tensor(ti->d0, ti->d1, ti->d2, ti->d3);
  std::memcpy(g->data, ti->grad, sizeof(double) * ti->size);
  return pub(g);
}

Tensor* zero_grad(Tensor* t) {
  if (t) std::memset(impl(t)->grad, 0, sizeof(double) * impl(t)->size);
  return tensor_incref(t);
}

Tensor* dream_set_precision(Tensor* t, int code) {
  if (!t) return nullptr;
  TensorImpl* ti = impl(t);
  if (code == 1) {
    if (!ti->fdata) ti->fdata = new float[ti->size]();
    for (int i = 0; i < ti->size; ++i) ti->fdata[i] = (float)ti->data[i];
    ti->dtype = 1;
  } else {
    if (ti->dtype == 1 && ti->fdata)
      for (int i = 0; i < ti->size; ++i) ti->data[i] = (double)ti->fdata[i];
    ti->dtype = 0;
  }
  return tensor_incref(t);
}

Tensor* dream_enable_fp16(void) {
  g_use_bf16 = true;
  return create_scalar(1.0);
}

Tensor* tensor_matmul(Tensor* a_, Tensor* b_) {
  if (!a_ || !b_) {
    report("matmul (@)", "null operand");
    return alloc_tensor(1, 1, 1, 1);
  }
  TensorImpl *a = impl(a_), *b = impl(b_);
  if (a->d1 != b->d0) {
    char msg[160];
    std::snprintf(msg, sizeof(msg), "shape mismatch (%dx%d @ %dx%d) — inner dimensions must match", a->d0, a->d1,
                  b->d0, b->d1);
    report("matmul (@)", msg);
    return alloc_tensor(1, 1, 1, 1);
  }
  const int M = a->d0, K = a->d1, N = b->d1;
  TensorImpl* c = new_tensor(M, N, 1, 1);
  set_parents(c, Fn::Matmul, {a, b});
  if (!ensure_device()) return pub(c);
  const dgx_dtype ab = gemm_type();
  DevBuf dA((size_t)M * K * esize(ab)), dB((size_t)K * N * esize(ab)), dC((size_t)M * N * 4);
  bool ok = dA.p && dB.p && dC.p && upload(a, dA.p, ab) && upload(b, dB.p, ab) &&
            device_gemm(dA.p, dB.p, dC.as<float>(), M, N, K, 0, 0, ab, nullptr, DGX_EPI_NONE, 0.f) &&
            download(dC.p, DGX_F32, c->data, (size_t)M * N, false);
  if (!ok) report("matmul (@)", dgx_last_error());
  if (a->dtype == 1 && b->dtype == 1) {  // f32 in, f32 out (elementwise.inc:1000-1016)
    c->fdata = new float[c->size];
    for (int i = 0; i < c->size; ++i) c->fdata[i] = (float)c->data[i];
    c->dtype = 1;
  }
  return pub(c);
}

static Tensor* linear_impl(Tensor* x_, Tensor* W_, Tensor* b_, bool relu) {
  const char* op = relu ? "linear_relu" : "linear";
  if (!x_ || !W_ || !b_) {
    report(op, "null arg");
    return alloc_tensor(1, 1, 1, 1);
  }
  TensorImpl *x = impl(x_), *W = impl(W_), *b = impl(b_);
  const int N = x->d0, din = x->d1, dout = W->d0;
  if (din != W->d1) {
    report(op, "x.d1 != W.d1");
    return alloc_tensor(1, 1, 1, 1);
  }
  TensorImpl* y = new_tensor(N, dout, 1, 1);
  set_parents(y, relu ? Fn::LinearRelu : Fn::Linear, {x, W, b});
  if (!ensure_device()) return pub(y);
  const dgx_dtype ab = gemm_type();
  DevBuf dX((size_t)N * din * esize(ab)), dW((size_t)dout * din * esize(ab)), dbias((size_t)dout * 4),
      dY((size_t)N * dout * 4);
  bool ok = dX.p && dW.p && dbias.p && dY.p && upload(x, dX.p, ab) && upload(W, dW.p, ab) &&
            upload(b, dbias.p, DGX_F32) &&
            device_gemm(dX.p, dW.p, dY.as<float>(), N, dout, din, 0, 1, ab, dbias.as<float>(),
                        relu ? DGX_EPI_BIAS_RELU : DGX_EPI_BIAS, 0.f) &&
            download(dY.p, DGX_F32, y->data, (size_t)N * dout, false);
  if (!ok) report(op, dgx_last_error());
  return pub(y);
}

Tensor* dream_linear(Tensor* x, Tensor* W, Tensor* b) { return linear_impl(x, W, b, false); }
Tensor* dream_linear_relu(Tensor* x, Tensor* W, Tensor* b) { return linear_impl(x, W, b, true); }

Tensor* dream_bmm(Tensor* a_, Tensor* b_, Tensor* batch_t, Tensor* m_t, Tensor* k_t, Tensor* n_t) {
  if (!a_ || !b_ || !batch_t || !m_t || !k_t || !n_t) {
    report("bmm", "null arg");
    return alloc_tensor(1, 1, 1, 1);
  }
  TensorImpl *a = impl(a_), *b = impl(b_);
  const int B = (int)batch_t->data[0], M = (int)m_t->data[0], K = (int)k_t->data[0], N = (int)n_t->data[0];
  if (B <= 0 || M <= 0 || K <= 0 || N <= 0 || a->size < B * M * K || b->size < B * K * N) {
    report("bmm", "size mismatch");
    return alloc_tensor(1, 1, 1, 1);
  }
  TensorImpl* c = new_tensor(B, M * N, 1, 1);
  set_parents(c, Fn::Bmm, {a, b});
  c->meta[0] = B;
  c->meta[1] = M;
  c->meta[2] = K;
  c->meta[3] = N;
  if (!ensure_device()) return pub(c);
  const dgx_dtype ab = gemm_type();
  DevBuf dA((size_t)a->size * esize(ab)), dB((size_t)b->size * esize(ab)), dC((size_t)B * M * N * 4);
  bool ok = dA.p && dB.p && dC.p && upload(a, dA.p, ab) && upload(b, dB.p, ab) &&
            dgx_bmm(dA.p, dB.p, dC.p, B, M, N, K, ab, DGX_F32, g_stream) == DGX_OK &&
            download(dC.p, DGX_F32, c->data, (size_t)B * M * N, false);
  if (!ok) report("bmm", dgx_last_error());
  return pub(c);
}

}  // extern "C"

namespace {

// The three attention ops share one device path: softmax(Q K^T / sqrt(dk)) V
// per batch row on the FlashAttention kernels (bf16 operands, fp32 softmax),
// causal for flash_attention / attention_causal, full for attention. The
// backward recomputes nothing on the host: it runs dgx_flash_bwd from the
// saved bf16 Q, K, V, O and the LSE.
Tensor* attention_impl(const char* op, Tensor* Q_, Tensor* K_, Tensor* V_, Tensor* batch_t, Tensor* seq_t,
                       Tensor* dk_t, int causal) {
  if (!Q_ || !K_ || !V_ || !batch_t || !seq_t || !dk_t) return create_scalar(0.0);
  TensorImpl *Q = impl(Q_), *K = impl(K_), *V = impl(V_);
  const int B = (int)batch_t->data[0], S = (int)seq_t->data[0], dk = (int)dk_t->data[0];
  const long long n = (long long)B * S * dk;
  if (B <= 0 || S <= 0 || dk <= 0 || Q->size < n || K->size < n || V->size < n) {
    report(op, "Q/K/V smaller than batch*seq*dk");
    return alloc_tensor(1, 1, 1, 1);
  }
  TensorImpl* out = new_tensor(B, S * dk, 1, 1);
  set_parents(out, Fn::Flash, {Q, K, V});
  out->meta[0] = B;
  out->meta[1] = S;
  out->meta[2] = dk;
  out->meta[3] = causal;
  if (!ensure_device()) return pub(out);
  FlashSaved* fs = new FlashSaved();
  const size_t bytes = (size_t)n * 2;
  bool ok = cudaMalloc(&fs->q, bytes) == cudaSuccess && cudaMalloc(&fs->k, bytes) == cudaSuccess &&
            cudaMalloc(&fs->v, bytes) == cudaSuccess && cudaMalloc(&fs->o, bytes) == cudaSuccess &&
            cudaMalloc(&fs->lse, (size_t)B * S * 4) == cudaSuccess;
  ok = ok && upload(Q, fs->q, DGX_BF16) && upload(K, fs->k, DGX_BF16) && upload(V, fs->v, DGX_BF16) &&
       dgx_flash_fwd(fs->q, fs->k, fs->v, fs->o, fs->lse, B, S, dk, (float)(1.0 / std::sqrt((double)dk)), causal,
                     DGX_BF16, g_stream) == DGX_OK &&
       download(fs->o, DGX_BF16, out->data, (size_t)n, false);
  if (!ok) {
    report(op, dgx_last_error());
    delete fs;
    return pub(out);
  }
  out->flash = fs;
  return pub(out);
}

}  // namespace

extern "C" {

Tensor* dream_flash_attention(Tensor* Q, Tensor* K, Tensor* V, Tensor* batch_t, Tensor* seq_t, Tensor* dk_t,
                              Tensor* block_t) {
  (void)block_t;  // the device tiles are 128 x 128; the result does not depend on the CPU block size
  return attention_impl("flash_attention", Q, K, V, batch_t, seq_t, dk_t, 1);
}

// dream_attention (runtime/nn/training.inc:177-220): full (non-causal) SDPA.
Tensor* dream_attention(Tensor* Q, Tensor* K, Tensor* V, Tensor* batch_t, Tensor* seq_t, Tensor* dk_t) {
  return attention_impl("attention", Q, K, V, batch_t, seq_t, dk_t, 0);
}

// dream_attention_causal (runtime/nn/training.inc:222-263): the materialised
// causal SDPA; the same function as flash_attention.
Tensor* dream_attention_causal(Tensor* Q, Tensor* K, Tensor* V, Tensor* batch_t, Tensor* seq_t, Tensor* dk_t) {
  return attention_impl("attention_causal", Q, K, V, batch_t, seq_t, dk_t, 1);
}

}  // extern "C"

namespace {

// dream_conv2d / dream_conv2d_padded: NCHW rows (N, Cin*H*W) and kernel
// (Cout, Cin*KH*KW) as the reference stores them, one batched device
// convolution (dgx_conv2d_fwd). The graph keeps input and kernel as parents
// (the reference's lhs / rhs; bias is not differentiated there either).
Tensor* conv_impl(const char* op, Tensor* input_, Tensor* kernel_, Tensor* bias_, Tensor* h_t, Tensor* w_t,
                  Tensor* kh_t, Tensor* kw_t, int pad, int stride) {
  if (!input_ || !kernel_ || !h_t || !w_t || !kh_t || !kw_t) {
    report(op, "null arg");
    return alloc_tensor(1, 1, 1, 1);
  }
  TensorImpl *x = impl(input_), *k = impl(kernel_), *b = bias_ ? impl(bias_) : nullptr;
  const int H = (int)h_t->data[0], W = (int)w_t->data[0], KH = (int)kh_t->data[0], KW = (int)kw_t->data[0];
  if (stride < 1) stride = 1;
  if (pad < 0 || H <= 0 || W <= 0 || KH <= 0 || KW <= 0 || H + 2 * pad < KH || W + 2 * pad < KW) {
    report(op, "kernel larger than input");
    return alloc_tensor(1, 1, 1, 1);
  }
  const int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
  const int N = x->d0, Cout = k->d0;
  int Cin = x->d1 / (H * W);
  if (Cin < 1) Cin = 1;
  if ((long long)N * Cin * H * W > x->size || (long long)Cout * Cin * KH * KW > k->size) {
    report(op, "input / kernel smaller than their geometry");
    return alloc_tensor(1, 1, 1, 1);
  }
  TensorImpl* out = new_tensor(N, Cout * OH * OW, 1, 1);
  set_parents(out, Fn::Conv, {x, k});
  const int geo[8] = {H, W, KH, KW, pad, stride, Cin, Cout};
  for (int i = 0; i < 8; ++i) out->meta[i] = geo[i];
  if (!ensure_device()) return pub(out);
  const dgx_dtype ab = gemm_type();
  DevBuf dX((size_t)x->size * 4), dK((size_t)k->size * 4), dB((size_t)Cout * 4), dY((size_t)N * Cout * OH * OW * 4);
  bool ok = dX.p && dK.p && dB.p && dY.p && upload(x, dX.p, DGX_F32) && upload(k, dK.p, DGX_F32);
  if (ok && b) {
    // bias entries past its size add nothing (conv_add_bias, conv.inc:5-10)
    TensorImpl bb{};
    std::vector<double> host((size_t)Cout, 0.0);
    for (int i = 0; i < Cout && i < b->size; ++i) host[i] = b->data[i];
    bb.data = host.data();
    bb.size = Cout;
    ok = upload(&bb, dB.p, DGX_F32) && cudaStreamSynchronize(g_stream) == cudaSuccess;
  }
  ok = ok && dgx_conv2d_fwd(dX.as<float>(), dK.as<float>(), b ? dB.as<float>() : nullptr, dY.as<float>(), N, Cin, H,
                            W, Cout, KH, KW, pad, stride, ab, g_stream) == DGX_OK &&
       download(dY.p, DGX_F32, out->data, (size_t)N * Cout * OH * OW, false);
  if (!ok) report(op, dgx_last_error());
  return pub(out);
}

}  // namespace

extern "C" {

// dream_conv2d (runtime/nn/conv.inc:12-110): valid convolution, stride 1.
Tensor* dream_conv2d(Tensor* input, Tensor* kernel, Tensor* bias, Tensor* h_t, Tensor* w_t, Tensor* kh_t,
                     Tensor* kw_t) {
  return conv_impl("conv2d", input, kernel, bias, h_t, w_t, kh_t, kw_t, 0, 1);
}

// dream_conv2d_padded (runtime/nn/conv.inc:111-187): zero padding and stride.
// Its backward is the gradient of this geometry (the reference's reuses the
// unpadded one).
Tensor* dream_conv2d_padded(Tensor* input, Tensor* kernel, Tensor* bias, Tensor* h_t, Tensor* w_t, Tensor* kh_t,
                            Tensor* kw_t, Tensor* pad_t, Tensor* stride_t) {
  return conv_impl("conv2d", input, kernel, bias, h_t, w_t, kh_t, kw_t, pad_t ? (int)pad_t->data[0] : 0,
                   stride_t ? (int)stride_t->data[0] : 1);
}

Tensor* dream_tp_matmul_column(Tensor* X_, Tensor* W_, Tensor* gpus_t) {
  if (!X_ || !W_) {
    report("tp_matmul_column", "null operand");
    return alloc_tensor(1, 1, 1, 1);
  }
  TensorImpl *X = impl(X_), *W = impl(W_);
  int G = gpus_t ? (int)gpus_t->data[0] : 1;
  if (G < 1) G = 1;
  const int M = X->d0, K = X->d1, N = W->d1;
  if (K != W->d0) {
    report("tp_matmul_column", "shape mismatch");
    return alloc_tensor(1, 1, 1, 1);
  }
  // No graph node, as in the reference (training.inc:1604-1630).
  TensorImpl* Y = new_tensor(M, N, 1, 1);
  if (!ensure_device()) return pub(Y);
  const dgx_dtype ab = gemm_type();
  DevBuf dX((size_t)M * K * esize(ab)), dW((size_t)K * N * esize(ab)), dY((size_t)M * N * 4);
  bool ok = dX.p && dW.p && dY.p && upload(X, dX.p, ab) && upload(W, dW.p, ab);
  // Shard g computes Y[:, col:col+ncol] = X . W[:, col:col+ncol]; the shard is
  // addressed in place through the row pitch, so the gather is the store itself.
  for (int g = 0; ok && g < G; ++g) {
    int col = 0, ncol = 0;
    dgx_tp_shard(N, G, g, &col, &ncol);
    if (ncol <= 0) continue;
    ok = dgx_gemm(dX.as<char>(), dW.as<char>() + (size_t)col * esize(ab), dY.as<float>() + col, M, ncol, K, K, N, N,
                  0, 0, ab, DGX_F32, DGX_F32_3XTF32, nullptr, DGX_EPI_NONE, 0.f, nullptr, 0, g_stream) == DGX_OK;
  }
  ok = ok && download(dY.p, DGX_F32, Y->data, (size_t)M * N, false);
  if (!ok) report("tp_matmul_column", dgx_last_error());
  return pub(Y);
}

Tensor* tensor_mul(Tensor* a_, Tensor* b_) {
  if (!a_ || !b_) return alloc_tensor(1, 1, 1, 1);
  TensorImpl *a = impl(a_), *b = impl(b_);
  TensorImpl* big = a->size >= b->size ? a : b;
  TensorImpl* c = new_tensor(big->d0, big->d1, big->d2, big->d3);
  for (int i = 0; i < c->size; ++i) c->data[i] = a->data[i % a->size] * b->data[i % b->size];
  set_parents(c, Fn::Mul, {a, b});
  return pub(c);
}

Tensor* sum(Tensor* a_) {
  if (!a_) return create_scalar(0.0);
  TensorImpl* a = impl(a_);
  double s = 0;
  for (int i = 0; i < a->size; ++i) s += a->data[i];
  TensorImpl* c = new_tensor(1, 1, 1, 1);
  c->data[0] = s;
  set_parents(c, Fn::Sum, {a});
  return pub(c);
}

}  // extern "C"

namespace {

void free_tensor(TensorImpl* t) {
  for (int i = 0; i < t->nparents; ++i) {
    TensorImpl* p = t->parents[i];
    if (--p->refcount <= 0) free_tensor(p);
  }
  delete t->flash;
  delete[] t->fdata;
  std::free(t->data);
  std::free(t->grad);
  delete t;
}

void topo(TensorImpl* root, std::vector<TensorImpl*>& order) {
  std::unordered_set<TensorImpl*> seen;
  std::vector<std::pair<TensorImpl*, int>> st{{root, 0}};
  seen.insert(root);
  while (!st.empty()) {
    auto& [t, i] = st.back();
    if (i < t->nparents) {
      TensorImpl* p = t->parents[i++];
      if (seen.insert(p).second) st.push_back({p, 0});
    } else {
      order.push_back(t);
      st.pop_back();
    }
  }
}

bool bwd_matmul(TensorImpl* t) {
  TensorImpl *a = t->parents[0], *b = t->parents[1];
  const int M = a->d0, K = a->d1, N = b->d1;
  const dgx_dtype ab = gemm_type();
  DevBuf dA((size_t)M * K * esize(ab)), dB((size_t)K * N * esize(ab)), dY((size_t)M * N * esize(ab));
  DevBuf gA((size_t)M * K * 4), gB((size_t)K * N * 4);
  if (!dA.p || !dB.p || !dY.p || !gA.p || !gB.p || !upload(a, dA.p, ab) || !upload(b, dB.p, ab)) return false;
  TensorImpl g{};
  g.data = t->grad;
  g.size = t->size;
  if (!upload(&g, dY.p, ab)) return false;
  // dA = dY . B^T (autograd.inc:104-113), dB = A^T . dY (:115-124)
  return device_gemm(dY.p, dB.p, gA.as<float>(), M, K, N, 0, 1, ab, nullptr, DGX_EPI_NONE, 0.f) &&
         device_gemm(dA.p, dY.p, gB.as<float>(), K, N, M, 1, 0, ab, nullptr, DGX_EPI_NONE, 0.f) &&
         download(gA.p, DGX_F32, a->grad, (size_t)M * K, true) && download(gB.p, DGX_F32, b->grad, (size_t)K * N, true);
}

bool bwd_linear(TensorImpl* t, bool relu) {
  TensorImpl *x = t->parents[0], *W = t->parents[1], *b = t->parents[2];
  const int N = x->d0, din = x->d1, dout = W->d0;
  // g = dY masked by the ReLU (autograd.inc:156-211); db on the host (O(N*out)).
  std::vector<double> g((size_t)N * dout);
  for (size_t i = 0; i < g.size(); ++i) g[i] = (relu && t->data[i] <= 0.0) ? 0.0 : t->grad[i];
  for (int i = 0; i < N; ++i)
    for (int j = 0; j < dout && j < b->size; ++j) b->grad[j] += g[(size_t)i * dout + j];
  const dgx_dtype ab = gemm_type();
  DevBuf dX((size_t)N * din * esize(ab)), dW((size_t)dout * din * esize(ab)), dG((size_t)N * dout * esize(ab));
  DevBuf gX((size_t)N * din * 4), gW((size_t)dout * din * 4);
  TensorImpl gt{};
  gt.data = g.data();
  gt.size = (int)g.size();
  if (!dX.p || !dW.p || !dG.p || !gX.p || !gW.p || !upload(x, dX.p, ab) || !upload(W, dW.p, ab) ||
      !upload(&gt, dG.p, ab))
    return false;
  // dX = g . W  (N x out . out x in), dW = g^T . X  (out x N . N x in)
  return device_gemm(dG.p, dW.p, gX.as<float>(), N, din, dout, 0, 0, ab, nullptr, DGX_EPI_NONE, 0.f) &&
         device_gemm(dG.p, dX.p, gW.as<float>(), dout, din, N, 1, 0, ab, nullptr, DGX_EPI_NONE, 0.f) &&
         download(gX.p, DGX_F32, x->grad, (size_t)N * din, true) &&
         download(gW.p, DGX_F32, W->grad, (size_t)dout * din, true);
}

bool bwd_bmm(TensorImpl* t) {
  TensorImpl *a = t->parents[0], *b = t->parents[1];
  const int B = t->meta[0], M = t->meta[1], K = t->meta[2], N = t->meta[3];
  const dgx_dtype ab = gemm_type();
  const size_t es = esize(ab);
  DevBuf dA((size_t)a->size * es), dB((size_t)b->size * es), dY((size_t)B * M * N * es);
  DevBuf gA((size_t)B * M * K * 4), gB((size_t)B * K * N * 4);
  TensorImpl g{};
  g.data = t->grad;
  g.size = t->size;
  if (!dA.p || !dB.p || !dY.p || !gA.p || !gB.p || !upload(a, dA.p, ab) || !upload(b, dB.p, ab) ||
      !upload(&g, dY.p, ab))
    return false;
  // One batched launch each: dA_b = dC_b . B_b^T, dB_b = A_b^T . dC_b.
  if (dgx_gemm_batched(dY.p, dB.p, gA.p, B, M, K, N, N, N, K, (long long)M * N, (long long)K * N, (long long)M * K,
                       0, 1, ab, DGX_F32, 0.f, g_stream) != DGX_OK ||
      dgx_gemm_batched(dA.p, dY.p, gB.p, B, K, N, M, K, N, N, (long long)M * K, (long long)M * N, (long long)K * N,
                       1, 0, ab, DGX_F32, 0.f, g_stream) != DGX_OK)
    return false;
  return download(gA.p, DGX_F32, a->grad, (size_t)B * M * K, true) &&
         download(gB.p, DGX_F32, b->grad, (size_t)B * K * N, true);
}

// "conv2d" backward (runtime/ops/autograd.inc:507-535): dK += dY . col^T,
// dX += col2im(K^T . dY), both on the device in one call.
bool bwd_conv(TensorImpl* t) {
  TensorImpl *x = t->parents[0], *k = t->parents[1];
  const int H = t->meta[0], W = t->meta[1], KH = t->meta[2], KW = t->meta[3], pad = t->meta[4], stride = t->meta[5];
  const int Cin = t->meta[6], Cout = t->meta[7], N = x->d0;
  const size_t nx = (size_t)N * Cin * H * W, nk = (size_t)Cout * Cin * KH * KW;
  DevBuf dX((size_t)x->size * 4), dK((size_t)k->size * 4), dY((size_t)t->size * 4), gX(nx * 4), gK(nk * 4);
  TensorImpl g{};
  g.data = t->grad;
  g.size = t->size;
  if (!dX.p || !dK.p || !dY.p || !gX.p || !gK.p || !upload(x, dX.p, DGX_F32) || !upload(k, dK.p, DGX_F32) ||
      !upload(&g, dY.p, DGX_F32))
    return false;
  if (dgx_conv2d_bwd(dX.as<float>(), dK.as<float>(), dY.as<float>(), gX.as<float>(), gK.as<float>(), N, Cin, H, W,
                     Cout, KH, KW, pad, stride, gemm_type(), 0, g_stream) != DGX_OK)
    return false;
  return download(gX.p, DGX_F32, x->grad, nx, true) && download(gK.p, DGX_F32, k->grad, nk, true);
}

bool bwd_flash(TensorImpl* t) {
  FlashSaved* fs = t->flash;
  if (!fs) return false;
  const int B = t->meta[0], S = t->meta[1], dk = t->meta[2];
  const size_t n = (size_t)B * S * dk;
  DevBuf ddO(n * 2), dQ(n * 2), dK(n * 2), dV(n * 2);
  TensorImpl g{};
  g.data = t->grad;
  g.size = (int)n;
  if (!ddO.p || !dQ.p || !dK.p || !dV.p || !upload(&g, ddO.p, DGX_BF16)) return false;
  if (dgx_flash_bwd(fs->q, fs->k, fs->v, fs->o, ddO.p, fs->lse, dQ.p, dK.p, dV.p, B, S, dk,
                    (float)(1.0 / std::sqrt((double)dk)), t->meta[3], DGX_BF16, nullptr, 0, g_stream) != DGX_OK)
    return false;
  return download(dQ.p, DGX_BF16, t->parents[0]->grad, n, true) &&
         download(dK.p, DGX_BF16, t->parents[1]->grad, n, true) &&
         download(dV.p, DGX_BF16, t->parents[2]->grad, n, true);
}

}  // namespace

extern "C" Tensor* backward(Tensor* root_) {
  if (!root_) {
    std::fprintf(stderr, "error: backward(null)\n");
    return create_scalar(0);
  }
  TensorImpl* root = impl(root_);
  for (int i = 0; i < root->size; ++i) root->grad[i] = 1.0;  // autograd.inc:34
  std::vector<TensorImpl*> order;
  topo(root, order);
  for (int i = (int)order.size() - 1; i >= 0; --i) {
    TensorImpl* t = order[i];
    bool ok = true;
    const char* op = "";
    switch (t->fn) {
      case Fn::Sum:
        for (int j = 0; j < t->parents[0]->size; ++j) t->parents[0]->grad[j] += t->grad[0];
        break;
      case Fn::Mul: {
        TensorImpl *a = t->parents[0], *b = t->parents[1];
        for (int j = 0; j < t->size; ++j) {
          a->grad[j % a->size] += t->grad[j] * b->data[j % b->size];
          b->grad[j % b->size] += t->grad[j] * a->data[j % a->size];
        }
        break;
      }
      case Fn::Matmul:
        op = "matmul";
        ok = ensure_device() && bwd_matmul(t);
        break;
      case Fn::Linear:
      case Fn::LinearRelu:
        op = "linear";
        ok = ensure_device() && bwd_linear(t, t->fn == Fn::LinearRelu);
        break;
      case Fn::Bmm:
        op = "bmm";
        ok = ensure_device() && bwd_bmm(t);
        break;
      case Fn::Flash:
        op = "flash_attention";
        ok = ensure_device() && bwd_flash(t);
        break;
      case Fn::Conv:
        op = "conv2d";
        ok = ensure_device() && bwd_conv(t);
        break;
      case Fn::None:
        break;
    }
    if (!ok) {
      char msg[96];
      std::snprintf(msg, sizeof(msg), "backward of %s: ", op);
      report(msg, dgx_last_error());
    }
  }
  return create_scalar(1.0);
}
