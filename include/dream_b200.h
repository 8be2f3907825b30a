/*
 * libdream_b200 — the Dream tensor runtime's op signatures for the GEMM and
 * FlashAttention hot path, computing on a B200 through libdgx.
 *
 * Drop-in for the reference runtime's ops on this path (heellowdsf/
 * DreamCompiler runtime/): same names, same argument meaning (scalars arrive
 * as 1x1 tensors), same ownership (+1 reference returned, arguments never
 * stolen, interop/dream.h:13-17) and the same error behaviour (a
 * "RUNTIME ERROR in <op>" line on stderr and a 1x1 result, never an abort,
 * runtime/ops/elementwise.inc:972-989). `struct Tensor` keeps the fields
 * compiled Dream code addresses by index (runtime/runtime.h:49-54): data,
 * grad, size, d0..d3; everything after them is private to this runtime.
 *
 * Host data stays f64 as in the reference; each op moves its operands to the
 * device, runs the sm_100a kernel and writes the result back into `data`.
 */
#ifndef DREAM_B200_H_
#define DREAM_B200_H_

#ifdef __cplusplus
extern "C" {
#endif

typedef struct Tensor {
  double* data; /* 0 */
  double* grad; /* 1 */
  int size;     /* 2 */
  int d0, d1, d2, d3; /* 3-6 */
  /* runtime-private fields follow (see dream_rt.cpp) */
} Tensor;

/* tensors and scalars (runtime/core/tensor.inc:143-200, :444) */
Tensor* alloc_tensor(int d0, int d1, int d2, int d3);
Tensor* create_scalar(double v);
Tensor* tensor_incref(Tensor* t);
Tensor* tensor_decref(Tensor* t);
Tensor* tensor_get_grad(Tensor* t);      /* runtime/ops/autograd.inc:1 */
Tensor* zero_grad(Tensor* t);            /* runtime/ops/autograd.inc:15 */

/* seeded inputs (runtime/ops/elementwise.inc:30-55): same stream as the reference */
Tensor* dream_set_seed(Tensor* seed_t);
Tensor* dream_randn(Tensor* d0, Tensor* d1);

/* precision (runtime/io/builtins.inc:1168-1185, :465) */
Tensor* dream_set_precision(Tensor* t, int code); /* 1 = f32 mirror, 0 = f64 */
Tensor* dream_enable_fp16(void);  /* route GEMMs through the bf16 tensor-core path */

/* the hot path */
Tensor* tensor_matmul(Tensor* a, Tensor* b);                       /* elementwise.inc:971 */
Tensor* dream_linear(Tensor* x, Tensor* W, Tensor* b);             /* elementwise.inc:1432 */
Tensor* dream_linear_relu(Tensor* x, Tensor* W, Tensor* b);        /* elementwise.inc:1508 */
Tensor* dream_bmm(Tensor* a, Tensor* b, Tensor* batch_t, Tensor* m_t, Tensor* k_t, Tensor* n_t); /* :1218 */
Tensor* dream_flash_attention(Tensor* Q, Tensor* K, Tensor* V, Tensor* batch_t, Tensor* seq_t, Tensor* dk_t,
                              Tensor* block_t);                    /* training.inc:284 */
Tensor* dream_attention(Tensor* Q, Tensor* K, Tensor* V, Tensor* batch_t, Tensor* seq_t,
                        Tensor* dk_t);                             /* training.inc:177 */
Tensor* dream_attention_causal(Tensor* Q, Tensor* K, Tensor* V, Tensor* batch_t, Tensor* seq_t,
                               Tensor* dk_t);                      /* training.inc:222 */
Tensor* dream_conv2d(Tensor* input, Tensor* kernel, Tensor* bias, Tensor* h_t, Tensor* w_t, Tensor* kh_t,
                     Tensor* kw_t);                                 /* conv.inc:12 */
Tensor* dream_conv2d_padded(Tensor* input, Tensor* kernel, Tensor* bias, Tensor* h_t, Tensor* w_t, Tensor* kh_t,
                            Tensor* kw_t, Tensor* pad_t, Tensor* stride_t); /* conv.inc:116 */
Tensor* dream_tp_matmul_column(Tensor* X, Tensor* W, Tensor* gpus_t); /* training.inc:1604 */

/* the two ops programs use to seed a gradient: backward(sum(Y * G)) */
Tensor* tensor_mul(Tensor* a, Tensor* b);
Tensor* sum(Tensor* a);

/* reverse-mode autograd over the ops above (runtime/ops/autograd.inc:26-887) */
Tensor* backward(Tensor* root);

#ifdef __cplusplus
}
#endif
#endif /* DREAM_B200_H_ */
