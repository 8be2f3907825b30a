/*
 * libdgx — the C ABI between the Dream tensor runtime and its B200 (sm_100a)
 * kernels. Plain pointers, sizes and status codes only; no C++ or torch types.
 *
 * All tensors are row-major and live in device memory unless a function says
 * otherwise. Every call is asynchronous on `stream` (a cudaStream_t, NULL for
 * the legacy default stream) and returns a status; on failure
 * dgx_last_error() holds a one-line message for the calling thread. No call
 * throws, aborts or falls back to the CPU.
 *
 * Library scratch: calls given no workspace (and the ones that take none:
 * split-K partials, int8 activation planes, conv im2col matrices) use
 * buffers the library owns per device and grows with cudaMalloc on demand,
 * syncing the calling stream before it frees a smaller one. Calls that use
 * the library's buffers must be ordered (one stream, or streams joined by
 * events); calls that overlap on the GPU from different streams would share
 * them. Pass a workspace where the entry point takes one to avoid that.
 *
 * Each entry point names the reference interface it replaces
 * (heellowdsf/DreamCompiler, paths relative to the project root).
 */
#ifndef DGX_H_
#define DGX_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  DGX_OK = 0,
  DGX_EINVAL = 1,        /* bad argument (null pointer, negative size, bad enum) */
  DGX_ECUDA = 2,         /* a CUDA runtime call failed */
  DGX_ENCCL = 3,         /* a collective or peer-memory step failed */
  DGX_ETIMEOUT = 4,      /* a bounded device or host wait ran out */
  DGX_EUNSUPPORTED = 5,  /* shape/type combination this build does not handle */
  DGX_ENOMEM = 6,        /* workspace too small or allocation failed */
} dgx_status;

typedef enum { DGX_F32 = 0, DGX_BF16 = 1, DGX_I8 = 2, DGX_F64 = 3 } dgx_dtype;  /* F64: dgx_convert only */

enum { DGX_EPI_NONE = 0, DGX_EPI_BIAS = 1, DGX_EPI_BIAS_RELU = 2, DGX_EPI_RELU = 3 };
enum { DGX_F32_3XTF32 = 0, DGX_F32_FFMA = 1 };

/* Library identification and error reporting. */
const char* dgx_version(void);
const char* dgx_last_error(void);

/* Select and initialise a device for the calling thread.
 * Replaces initBackend() (runtime/backend/gpu.inc:313-361): no OpenCL/cuBLAS
 * probing and no CPU/GPU threshold (gpu.inc:293-307); the device always runs. */
dgx_status dgx_init(int device);

/* Wait for `stream`, then read and clear the device error word that bounded
 * waits in the kernels report into. DGX_ETIMEOUT if any wait ran out. */
dgx_status dgx_sync_check(void* stream);

/* Device memory, streams and copies for callers that do not include the CUDA
 * headers (the Dream runtime loads CUDA dynamically and defines its own
 * names for it, runtime/backend/gpu.inc:1-110). dgx_copy is asynchronous on
 * `stream`: direction 0 host -> device, 1 device -> host, 2 device -> device
 * (pageable host memory makes it return after the host side is read or
 * written, as cudaMemcpyAsync does). */
dgx_status dgx_stream_create(void** stream);
dgx_status dgx_device_alloc(size_t bytes, void** ptr);
dgx_status dgx_device_free(void* ptr);
dgx_status dgx_copy(void* dst, const void* src, size_t bytes, int direction, void* stream);

/* Failure detection without a device fault.
 *
 * dgx_fault_inject: host-side fault injection. Every entry point that
 * launches device work (and dgx_sync_check, dgx_tp_open) counts its calls
 * from 1; call number `at_call` returns `status` (an error status) with the
 * message "injected fault at call n (<entry point>)" and launches nothing.
 * at_call = 0 turns injection off. The counter restarts on every
 * dgx_fault_inject. The environment variable DGX_FAIL_AT=<n>[:<status>]
 * (status defaults to DGX_ETIMEOUT) sets the same thing at the first call.
 * Calls a convolution makes through dgx_gemm count as well. The reference
 * has no counterpart; its error path (RUNTIME ERROR and a 1x1 result,
 * runtime/ops/elementwise.inc:972-989) is what the Dream op mirror turns a
 * non-OK status into, and this lets callers test that path.
 * dgx_fault_calls: calls counted so far. */
dgx_status dgx_fault_inject(long long at_call, int status);
long long dgx_fault_calls(void);

/* dgx_wait_probe: run one of the library's bounded device waits in a
 * one-warp kernel on `stream`, so a caller can check on one GPU that a wait
 * which never completes ends with DGX_ETIMEOUT from dgx_sync_check and
 * leaves the context usable.
 *   kind 0: the cross-rank completion wait of dgx_tp_gemm_colsplit: wait
 *           until *flag (device memory) >= expect, at most timeout_us.
 *   kind 1: the mbarrier wait of every tensor-core kernel's pipeline, with
 *           its fixed budget of about one second; expect = 0 completes the
 *           barrier first (the wait succeeds), anything else leaves it
 *           incomplete (flag and timeout_us are not used). */
dgx_status dgx_wait_probe(int kind, const unsigned long long* flag, unsigned long long expect, int timeout_us,
                          void* stream);

/* Profiling hook: the next main kernel this thread launches (the tensor-core
 * kernel behind dgx_gemm, dgx_flash_fwd or dgx_flash_bwd) is bracketed by
 * cudaEventRecord(start) / cudaEventRecord(stop) on the stream it runs on,
 * then the hook clears itself. start/stop are cudaEvent_t handles; NULL
 * clears. Lets a benchmark time the dominant kernel live, inside its loop.
 * (No reference counterpart: the reference only has host wall-clock
 * regions, runtime/nn/training.inc:2223-2291.) */
void dgx_set_timer_events(void* start, void* stop);

/*
 * Device-side element conversion dst[i] = (dst_type) src[i] for n elements
 * (f64/f32 -> bf16 round to nearest even, as dream_to_bf16,
 * runtime/nn/training.inc:1969-1976; f64 -> f32 round to nearest). With
 * accumulate=1 the converted value is ADDED to dst (f64/f32 dst only), which
 * is how autograd's `grad +=` (runtime/ops/autograd.inc:112,123) lands.
 * Lets a caller whose tensors are f64 (the Dream runtime's `data`/`grad`)
 * move them to the device at 8 B/element and convert there.
 */
dgx_status dgx_convert(const void* src, dgx_dtype src_type, void* dst, dgx_dtype dst_type, size_t n, int accumulate,
                       void* stream);

/*
 * Content fingerprint of `bytes` bytes of device memory into *out (device
 * memory, 8 bytes): the sum mod 2^64 over 8-byte little-endian words w_i
 * (a shorter tail zero-padded into one last word) of
 * splitmix64(w_i + (i + 1) * 0x9E3779B97F4A7C15). A host computes the same
 * value over the same bytes, so a caller holding a device copy of a host
 * buffer can tell whether the host buffer still holds those bytes. No
 * counterpart in the reference: the B200 backend of the Dream runtime uses it
 * to keep device copies of tensors across ops (the reference re-uploads every
 * operand on every call, runtime/ops/elementwise.inc:1033-1090).
 */
dgx_status dgx_fingerprint(const void* data, size_t bytes, unsigned long long* out, void* stream);

/*
 * C[M,N] = beta*C + op(A)[M,K] . op(B)[K,N] (+bias[N]) (ReLU)
 *   A stored [M,K] (transA=0) or [K,M] (transA=1), row pitch lda elements
 *   B stored [K,N] (transB=0) or [N,K] (transB=1), row pitch ldb elements
 *   ab_type: DGX_BF16 (tcgen05 kind::f16) or DGX_F32 (f32_mode 3xTF32 on
 *            tcgen05 kind::tf32, or FFMA); accumulation is always fp32
 *   c_type : DGX_F32 or DGX_BF16
 *   epilogue: DGX_EPI_* (bias is required for the BIAS forms)
 *   workspace: device scratch for the 3xTF32 split planes, at least
 *            dgx_gemm_workspace_size() bytes; NULL lets the library use its
 *            own per-device buffer.
 * Replaces: tensor_matmul (runtime/ops/elementwise.inc:971-1213) incl. the
 * f32 mirror path dream_gemm_f32 (:689-738) and cuBLAS Sgemm/GemmEx (:1046-1090);
 * the "matmul" backward dA = dY.B^T (transB=1, beta=1) and dB = A^T.dY
 * (transA=1, beta=1) (runtime/ops/autograd.inc:91-125); dream_linear /
 * dream_linear_relu Y = X.W^T + b (transB=1, epilogue BIAS[_RELU])
 * (runtime/ops/elementwise.inc:1432-1521).
 */
dgx_status dgx_gemm(const void* A, const void* B, void* C, int M, int N, int K, int lda, int ldb, int ldc,
                    int transA, int transB, dgx_dtype ab_type, dgx_dtype c_type, int f32_mode, const float* bias,
                    int epilogue, float beta, void* workspace, size_t workspace_bytes, void* stream);

/*
 * C[M,N] = beta*C + op(A)[M,K] . op(B)[K,N] (+bias[N]) (ReLU), all in f64:
 * every product and sum an f64 fused multiply-add, so results carry the
 * reference's float64 precision (no tensor-core splitting).
 *   Operand layouts, pitches, transA/transB and epilogue as dgx_gemm; bias is
 *   f64 [N]; beta any value (0: C is not read).
 * Replaces, for the reference's default float64 tensors: dream_gemm_d
 * (runtime/ops/elementwise.inc:516-638, the CPU branch of tensor_matmul
 * :1020-1031), the f64 "matmul" backward loops (runtime/ops/autograd.inc:91-125)
 * and the f64 dream_linear / "linear" backward (elementwise.inc:1432-1521,
 * autograd.inc:156-211).
 */
dgx_status dgx_gemm_f64(const double* A, const double* B, double* C, int M, int N, int K, int lda, int ldb, int ldc,
                        int transA, int transB, const double* bias, int epilogue, double beta, void* stream);
size_t dgx_gemm_workspace_size(int M, int N, int K, int transA, int transB, dgx_dtype ab_type, int f32_mode);
/* bf16 GEMM kernel selection: 0 = single-CTA tiles (128 x 256) only;
 * 1 (default) = 2-SM tiles (256 x 256 over a CTA pair, tcgen05 cta_group::2)
 * wherever they apply (A not transposed, beta 0 or fp32 accumulate, K >= 1024,
 * enough tiles), single-CTA tiles elsewhere. Process-wide. */
dgx_status dgx_gemm_set_algo(int algo);

/*
 * Batched GEMM C_b = A_b . B_b over `batch` contiguous [M,K] x [K,N] blocks,
 * all batches in one kernel launch. Replaces dream_bmm
 * (runtime/ops/elementwise.inc:1218-1252).
 */
dgx_status dgx_bmm(const void* A, const void* B, void* C, int batch, int M, int N, int K, dgx_dtype ab_type,
                   dgx_dtype c_type, void* stream);

/*
 * Strided batched GEMM: for b < batch,
 *   C_b = op(A_b) . op(B_b) (+ beta*C_b),  X_b = X + b*strideX (elements),
 * op and leading dimensions as in dgx_gemm (no bias epilogue; f32 inputs run
 * 3xTF32 with library scratch). strideA / strideB may be 0 (one operand
 * shared by every batch); output batches may not overlap (strideC >= M*ldc).
 * One launch for all batches; this is what the "bmm" backward
 * (runtime/ops/autograd.inc:549-574) needs: dA_b = dC_b . B_b^T (transB) and
 * dB_b = A_b^T . dC_b (transA).
 */
dgx_status dgx_gemm_batched(const void* A, const void* B, void* C, int batch, int M, int N, int K, int lda,
                            int ldb, int ldc, long long strideA, long long strideB, long long strideC, int transA,
                            int transB, dgx_dtype ab_type, dgx_dtype c_type, float beta, void* stream);

/*
 * 2-D convolution, NCHW fp32 tensors as the reference stores them:
 * X [N][Cin][H][W], Kw [Cout][Cin*KH*KW] (row = output channel), bias [Cout]
 * (may be NULL), Y [N][Cout][OH][OW], OH = (H + 2*pad - KH)/stride + 1.
 * One tensor-core GEMM for the whole batch over a positions-major im2col
 * matrix (library scratch, dgx_conv2d_workspace_size bytes). ab_type DGX_F32
 * runs 3xTF32, DGX_BF16 bf16 operands (fp32 accumulate either way).
 * Replaces dream_conv2d (runtime/nn/conv.inc:12-110, pad 0, stride 1) and
 * dream_conv2d_padded (:111-187), im2col (runtime/nn/im2col.inc:2-13).
 */
dgx_status dgx_conv2d_fwd(const float* X, const float* Kw, const float* bias, float* Y, int N, int Cin, int H, int W,
                          int Cout, int KH, int KW, int pad, int stride, dgx_dtype ab_type, void* stream);
/*
 * Convolution backward: dK = sum_n dY_n . col_n^T and dX = col2im(K^T . dY)
 * (either may be NULL to skip it); accumulate = 1 adds into dX / dK, as
 * autograd's `grad +=` does. Replaces the "conv2d" backward branch
 * (runtime/ops/autograd.inc:507-535) and col2im (runtime/nn/im2col.inc:14-25);
 * with pad / stride it is the gradient of dgx_conv2d_fwd's geometry.
 */
dgx_status dgx_conv2d_bwd(const float* X, const float* Kw, const float* dY, float* dX, float* dK, int N, int Cin, int H,
                          int W, int Cout, int KH, int KW, int pad, int stride, dgx_dtype ab_type, int accumulate,
                          void* stream);
size_t dgx_conv2d_workspace_size(int N, int Cin, int H, int W, int Cout, int KH, int KW, int pad, int stride,
                                 dgx_dtype ab_type);

/*
 * FlashAttention forward. Q, K, V, O: [BH][S][D] (heads folded into the batch,
 * as dream_flash_attention's `(B, S*dk)` layout), dtype DGX_BF16.
 * LSE [BH][S] fp32 receives the natural-log row log-sum-exp of scale*QK^T
 * (may be NULL when no backward follows). causal=1 masks j > i.
 * Replaces dream_flash_attention (runtime/nn/training.inc:284-401) and its
 * OpenCL kernel flash_attention_v1 (:310-363).
 */
dgx_status dgx_flash_fwd(const void* Q, const void* K, const void* V, void* O, float* LSE, int BH, int S, int D,
                         float scale, int causal, dgx_dtype dtype, void* stream);

/*
 * Reproducibility of the FlashAttention backward (process-wide, default 0).
 * Head dims <= 64 normally take one kernel whose dQ sums each key tile's
 * part by fp32 reduce-adds in completion order: dK and dV are the same bits
 * on every run, dQ can differ in the last bits. With on = 1 they take the
 * two-kernel form that 64 < D <= 128 always uses (dK/dV per key tile, dQ per
 * query tile, no accumulation through memory): every gradient is the same
 * bits on every run, at the cost of computing S and dP twice. The reference
 * promises byte-identical seeded runs (tests/16_determinism.dream).
 */
dgx_status dgx_flash_set_deterministic(int on);

/*
 * FlashAttention backward: dQ, dK, dV ([BH][S][D], dtype) from Q, K, V, O, dO
 * and the forward's LSE. workspace: at least dgx_flash_bwd_workspace_size()
 * bytes of device scratch (fp32 dQ accumulator and the row terms
 * D_i = dO_i . O_i); NULL lets the library use its own per-device buffer.
 * A workspace of the caller's is cleared while the kernel issued just before
 * the call may still be running (it must not be that kernel's operand).
 * Replaces the "flash_attention" backward branch
 * (runtime/ops/autograd.inc:779-840), without its 3-pass recompute.
 */
dgx_status dgx_flash_bwd(const void* Q, const void* K, const void* V, const void* O, const void* dO,
                         const float* LSE, void* dQ, void* dK, void* dV, int BH, int S, int D, float scale,
                         int causal, dgx_dtype dtype, void* workspace, size_t workspace_bytes, void* stream);
size_t dgx_flash_bwd_workspace_size(int BH, int S, int D);

/*
 * FlashAttention forward / backward on heads stored inside token rows (bf16):
 * head h of batch b, position s of tensor X starts at element
 * (b*S + s)*ldX + h*D of X's pointer, BH = B*H. This is how a fused QKV
 * projection writes its output ([B*S][3*H*D]: pass Q = qkv, K = qkv + H*D,
 * V = qkv + 2*H*D, all with ld = 3*H*D) and how the output projection reads
 * O ([B*S][H*D], ld = H*D), so no head transposes run around the kernels.
 * LSE stays [BH][S]; the workspace is dgx_flash_bwd_workspace_size(B*H, S, D).
 * Tensor-core kernels only: D % 8 == 0, D <= 64, 16-byte aligned pointers,
 * pitches multiples of 8 elements. No reference counterpart: the
 * reference's flash_attention takes one head per batch row ((B, S*dk)); this
 * form lets a caller that keeps heads inside token rows skip the transposes.
 */
dgx_status dgx_flash_fwd_rows(const void* Q, int ldq, const void* K, int ldk, const void* V, int ldv, void* O,
                              int ldo, float* LSE, int B, int H, int S, int D, float scale, int causal, void* stream);
dgx_status dgx_flash_bwd_rows(const void* Q, int ldq, const void* K, int ldk, const void* V, int ldv, const void* O,
                              int ldo, const void* dO, int lddo, const float* LSE, void* dQ, int lddq, void* dK,
                              int lddk, void* dV, int lddv, int B, int H, int S, int D, float scale, int causal,
                              void* workspace, size_t workspace_bytes, void* stream);

/*
 * int8 weight-only dense layer, Y[B,N] = bias[N] + scale[n] * sum_k W[n,k] * X[b,k].
 *   W int8 [N][K] (row n = output channel, the dense_q layout), scale [N] fp32
 *   per output channel (a per-tensor scale is N copies of one value), bias [N]
 *   or NULL, X [B][K] fp32, Y [B][N] fp32.
 *   mode 0 (W8A32): fp32 products and accumulation, the arithmetic of the
 *          exported dense_q (runtime/nn/training.inc:3738-3752).
 *   mode 1 (W8A8): X quantised per row (sx = max|x|/127, round half away from
 *          zero, clamp [-127,127]), exact int32 accumulation, then
 *          Y = bias + scale[n]*sx[b]*acc.
 * Replaces the export-only int8 path dense_q / export_c_header_int8
 * (runtime/nn/training.inc:3492-3817) with an on-device kernel.
 */
dgx_status dgx_gemm_w8(const float* X, const int8_t* W, const float* scale, const float* bias, float* Y, int B,
                       int N, int K, int mode, void* stream);
/*
 * dgx_gemm_w8 mode 1 (W8A8) for callers that cannot let a library allocate
 * device memory: a deployment that gives the whole device budget to its own
 * pool at start-up, or a serving loop that must not call cudaMalloc once it
 * runs (cudaMalloc can synchronise the device and take unbounded time). It has
 * no counterpart in the reference.
 *   Same arguments and result as dgx_gemm_w8(..., mode = 1), without `mode`.
 *   The quantised activations and row scales live in a fixed array inside
 *   libdgx's device image (4 MiB + 16 KiB, held on every GPU that loads the
 *   library until the process exits), so the call allocates nothing.
 *   Limits: B <= 4096 and B*K <= 4,194,304; larger problems return DGX_EINVAL.
 *   Every call looks up the array's device address (cudaGetSymbolAddress,
 *   which allocates nothing); make the first call on a device before any
 *   stream capture. dgx_init is not required first: the device error word
 *   the kernels report into is a fixed word in the same image as well.
 *   All calls share the array and it keeps the last call's contents: calls
 *   that overlap on the GPU (other streams, other host threads) race on it,
 *   so issue them in order on one stream.
 */
dgx_status dgx_gemm_w8a8_noalloc(const float* X, const int8_t* W, const float* scale, const float* bias, float* Y,
                                 int B, int N, int K, void* stream);
/*
 * One layer of the C inference code export_c_header_int8 writes
 * (runtime/nn/training.inc:3694-3752), for a batch of B inputs at once:
 *   Y[b][j] = relu?( bias[j] + s_j * sum_k W[j][k] * X[b][k] ),
 * with W the emitted `static const int8_t <layer>_weight[out_dim*in_dim]`
 * array as is ([out][in], row = output channel), s_j = `scale` (the emitted
 * per-tensor `<layer>_weight_scale`) when `scales` is NULL, else scales[j]
 * (the per-channel variant of the exporter), bias the emitted float array,
 * relu = 1 for every layer but the last (the emitted relu_inplace). The
 * products are exact (the fp32 activations go through the 3-plane int8
 * split) and each output is rounded once, where the emitted dense_q adds
 * fp32 terms one by one.
 */
dgx_status dgx_dense_q(const float* X, const int8_t* W, float scale, const float* scales, const float* bias,
                       float* Y, int B, int out_dim, int in_dim, int relu, void* stream);
/* Exact int32 accumulators acc[b,n] = sum_k Xq[b,k]*W[n,k] (the W8A8 core). */
dgx_status dgx_gemm_i8i32(const int8_t* Xq, const int8_t* W, int32_t* acc, int B, int N, int K, void* stream);
/* Per-row symmetric quantisation used by mode 1: Xq = clamp(round(X/sx)), sx = max|X_b|/127. */
dgx_status dgx_quantize_rows_i8(const float* X, int8_t* Xq, float* sx, int B, int K, void* stream);

/*
 * Building blocks of the GPT training step: the device
 * forms of the reference NN ops between the GEMMs and attention, so the step
 * stays on the GPU. fp32 activations and master data; bf16 where the next
 * consumer is a GEMM. Rows are contiguous ([R][C] row-major).
 */
/* y16 = bf16(layer_norm(x)) per row (no affine, eps 1e-5); mean/rstd [R] saved
 * for the backward. Replaces dream_layer_norm (runtime/io/builtins.inc:167-197). */
dgx_status dgx_layernorm_fwd(const float* x, void* y16, float* mean, float* rstd, int R, int C, void* stream);
/* dx (+)= rstd/C * (C*dy - sum(dy) - y*sum(dy*y)), y recomputed from x
 * (runtime/ops/autograd.inc:453-470); accumulate = 1 adds into dx. */
dgx_status dgx_layernorm_bwd(const float* x, const float* mean, const float* rstd, const float* dy, float* dx, int R,
                             int C, int accumulate, void* stream);
/* dgx_layernorm_bwd that also writes bf16(dx) into dx16 ([R][C]): the
 * residual gradient and the bf16 operand of the next GEMMs in one pass. */
dgx_status dgx_layernorm_bwd_x16(const float* x, const float* mean, const float* rstd, const float* dy, float* dx,
                                 void* dx16, int R, int C, int accumulate, void* stream);
/* y16 = bf16(gelu(x)), tanh form (runtime/io/builtins.inc:548-560); x DGX_F32 or DGX_BF16. */
dgx_status dgx_gelu_fwd(const void* x, int x_type, void* y16, long long n, void* stream);
/* dx16 = bf16(gelu'(x) * dy) (runtime/ops/autograd.inc:293-303); x, dy DGX_F32 or DGX_BF16. */
dgx_status dgx_gelu_bwd(const void* x, int x_type, const void* dy, int dy_type, void* dx16, long long n, void* stream);
/* x[i] = W[tok[i]] + P[i % S] (P may be NULL): dream_embedding
 * (runtime/nn/training.inc:579-600) plus the broadcast position add. */
dgx_status dgx_embedding_fwd(const int* tok, const float* W, const float* P, float* x, int n, int S, int d, int V,
                             void* stream);
/* dW[tok[i]] += dx[i] (fp32 atomics), dP[s] += sum over rows i % S == s
 * (runtime/ops/autograd.inc:330-341). dP may be NULL. */
dgx_status dgx_embedding_bwd(const int* tok, const float* dx, float* dW, float* dP, int n, int S, int d, int V,
                             void* stream);
/* loss = nll_loss(log_softmax(logits), target) over n rows of pitch ld (the
 * first V columns valid), device scalar; dlogits (may be NULL; DGX_F32 or
 * DGX_BF16, pitch ld) = (softmax - onehot(target)) / n, zero past V.
 * runtime/ops/elementwise.inc:1550-1603, runtime/ops/autograd.inc:212-245. */
dgx_status dgx_softmax_nll(const float* logits, int ld, int V, const int* target, int n, float* loss, void* dlogits,
                           int dlogits_type, void* stream);
/* One AdamW step, grad zeroed: dream_adamw_update
 * (runtime/io/builtins.inc:578-617) with fp32 state. The 1-based step count
 * is `step`, or *step_dev (device int) when step_dev is not NULL, so that a
 * captured CUDA graph replays correct bias corrections. */
dgx_status dgx_adamw(float* param, float* grad, float* m, float* v, long long n, float lr, float b1, float b2,
                     float eps, float wd, int step, const int* step_dev, void* stream);
/* db[j] (+)= sum_r dy[r][j] (bias gradients of dream_linear,
 * runtime/ops/autograd.inc:156-211); dy DGX_F32 or DGX_BF16. Deterministic. */
dgx_status dgx_colsum(const void* dy, int dy_type, float* db, int R, int N, int accumulate, void* stream);
/* Head layouts for attention: rows [B*S][ld] with head h at columns
 * col0 + h*D  <->  heads [B*H][S][D] (bf16, the dgx_flash_* layout). */
dgx_status dgx_rows_to_heads(const void* src, int src_type, int ld, int col0, void* dst, int B, int S, int H, int D,
                             void* stream);
dgx_status dgx_heads_to_rows(const void* src, void* dst, int ld, int col0, int B, int S, int H, int D, void* stream);

/*
 * Column-parallel tensor-parallel GEMM over `world` GPUs, one process per GPU.
 * Each rank holds all of A [M,K] and its column shard of B ([K, n_r] with the
 * reference's widths: base = N/world, the first N%world shards one wider).
 * The GEMM epilogue writes every output tile straight into C_full [M,N] on
 * every rank through NVLink peer stores, so the all-gather overlaps the GEMM
 * tile by tile; the call returns after a bounded cross-rank completion flag.
 * Replaces dream_tp_matmul_column (runtime/nn/training.inc:1604-1630), whose
 * "all-gather" is a host copy into Y[:, col:col+ncol].
 */
/* C_full is complete on every rank when the call's stream reaches the end of
 * the call (the last step is a bounded cross-rank completion wait; a missing
 * rank shows up as DGX_ETIMEOUT from dgx_sync_check). It stays valid until
 * any rank's next dgx_tp_gemm_colsplit, whose stores may land in it: callers
 * that keep a result while another call starts must synchronise or copy. */
/* Shard width and first column of `rank`, as dream_tp_matmul_column computes them. */
void dgx_tp_shard(int N, int world, int rank, int* col0, int* ncol);
/* Export this rank's C_full + flag buffers as an opaque handle (for exchange). */
dgx_status dgx_tp_export(void* C_full, size_t c_bytes, void* handle_out, size_t handle_bytes);
size_t dgx_tp_handle_size(void);
/* Open all ranks' handles (handles: world * dgx_tp_handle_size() bytes). */
dgx_status dgx_tp_open(int rank, int world, const void* handles);
dgx_status dgx_tp_gemm_colsplit(const void* A, const void* B_shard, int M, int N, int K, dgx_dtype ab_type,
                                dgx_dtype c_type, int timeout_ms, void* stream);
dgx_status dgx_tp_close(void);

#ifdef __cplusplus
}
#endif
#endif /* DGX_H_ */
