// C ABI entry points of libdgx: argument validation, dispatch to the sm_100a
// kernels, error reporting. See include/dgx.h for the contract.
#include <atomic>
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.h"
#include "gemm.h"

namespace dgx {

static thread_local char g_err[512] = "";

dgx_status set_error(dgx_status st, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return st;
}

dgx_status cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return DGX_OK;
  return set_error(DGX_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

TensorMapEncodeFn get_tensor_map_encoder() {
  static TensorMapEncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<TensorMapEncodeFn>(p);
  });
  return fn;
}

static int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

int num_sms() {
  static int cache[64] = {0};
  const int d = current_device();
  if (d < 0 || d >= 64) return 148;
  if (!cache[d]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
    cache[d] = n > 0 ? n : 148;
  }
  return cache[d];
}

struct DeviceState {
  uint32_t* err_word = nullptr;
  void* scratch[kScratchSlots] = {};
  size_t scratch_bytes[kScratchSlots] = {};
};
static std::mutex g_dev_mu;
static DeviceState g_dev[64];

// The error word lives in libdgx's device image (zero when the module
// loads), so no entry point allocates to get it. Its device address is
// looked up once per device; dgx_init looks it up again, so a caller that
// reset the device calls dgx_init before the next op.
static __device__ uint32_t g_error_word;

static uint32_t* lookup_error_word() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_error_word) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return static_cast<uint32_t*>(p);
}

uint32_t* device_error_word() {
  const int d = current_device();
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceState& st = g_dev[d & 63];
  if (!st.err_word) st.err_word = lookup_error_word();
  return st.err_word;
}

static uint32_t* refresh_error_word() {
  const int d = current_device();
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceState& st = g_dev[d & 63];
  st.err_word = lookup_error_word();
  return st.err_word;
}

void* library_scratch_slot(int slot, size_t bytes, cudaStream_t s) {
  if (slot < 0 || slot >= kScratchSlots) return nullptr;
  const int d = current_device();
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceState& st = g_dev[d & 63];
  if (st.scratch_bytes[slot] < bytes) {
    // The old buffer may still be read by queued work on `s`.
    if (st.scratch[slot]) {
      cudaStreamSynchronize(s);
      cudaFree(st.scratch[slot]);
      st.scratch[slot] = nullptr;
      st.scratch_bytes[slot] = 0;
    }
    size_t want = bytes < (64u << 20) ? (64u << 20) : bytes;
    if (cudaMalloc(&st.scratch[slot], want) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    st.scratch_bytes[slot] = want;
  }
  return st.scratch[slot];
}

void* library_scratch(size_t bytes, cudaStream_t s) { return library_scratch_slot(kScratchGeneral, bytes, s); }

// Fault injection state: calls counted since the last dgx_fault_inject (or
// process start), the call that fails (0: none) and its status.
static std::atomic<long long> g_fault_calls{0};
static std::atomic<long long> g_fault_at{-1};  // -1: environment not read yet
static std::atomic<int> g_fault_status{DGX_ETIMEOUT};

static void fault_from_env() {
  long long at = 0;
  int st = DGX_ETIMEOUT;
  if (const char* v = getenv("DGX_FAIL_AT")) {
    char* end = nullptr;
    at = strtoll(v, &end, 10);
    if (end && *end == ':') st = (int)strtol(end + 1, nullptr, 10);
    if (at < 0) at = 0;
    if (st <= DGX_OK || st > DGX_ENOMEM) st = DGX_ETIMEOUT;
  }
  long long expect = -1;
  if (g_fault_at.compare_exchange_strong(expect, at)) g_fault_status.store(st);
}

bool fault_fires(const char* entry, dgx_status* st) {
  if (g_fault_at.load(std::memory_order_relaxed) < 0) fault_from_env();
  const long long at = g_fault_at.load(std::memory_order_relaxed);
  if (at <= 0) return false;
  const long long n = g_fault_calls.fetch_add(1) + 1;
  if (n != at) return false;
  *st = set_error((dgx_status)g_fault_status.load(), "injected fault at call %lld (%s)", n, entry);
  return true;
}

static thread_local cudaEvent_t g_timer_start = nullptr, g_timer_stop = nullptr;

TimerScope::TimerScope(cudaStream_t st) : s(st), stop(g_timer_stop) {
  if (g_timer_start && g_timer_stop) cudaEventRecord(g_timer_start, s);
  else stop = nullptr;
  g_timer_start = g_timer_stop = nullptr;
}
TimerScope::~TimerScope() {
  if (stop) cudaEventRecord(stop, s);
}

}  // namespace dgx

using namespace dgx;

extern "C" {

const char* dgx_version(void) { return "libdgx 0.1 (sm_100a)"; }

const char* dgx_last_error(void) { return g_err; }

void dgx_set_timer_events(void* start, void* stop) {
  g_timer_start = (cudaEvent_t)start;
  g_timer_stop = (cudaEvent_t)stop;
}

dgx_status dgx_fault_inject(long long at_call, int status) {
  if (at_call < 0) return set_error(DGX_EINVAL, "dgx_fault_inject: negative call index");
  if (at_call > 0 && (status <= DGX_OK || status > DGX_ENOMEM))
    return set_error(DGX_EINVAL, "dgx_fault_inject: status %d is not an error status", status);
  g_fault_at.store(-2);  // keep the environment from overriding this setting
  g_fault_status.store(at_call > 0 ? status : DGX_ETIMEOUT);
  g_fault_calls.store(0);
  g_fault_at.store(at_call);
  return DGX_OK;
}

long long dgx_fault_calls(void) { return g_fault_calls.load(); }

dgx_status dgx_stream_create(void** stream) {
  if (!stream) return set_error(DGX_EINVAL, "dgx_stream_create: null pointer");
  cudaStream_t s = nullptr;
  const cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  if (e != cudaSuccess) return cuda_status(e, "dgx_stream_create");
  *stream = s;
  return DGX_OK;
}

dgx_status dgx_device_alloc(size_t bytes, void** ptr) {
  if (!ptr) return set_error(DGX_EINVAL, "dgx_device_alloc: null pointer");
  *ptr = nullptr;
  const cudaError_t e = cudaMalloc(ptr, bytes ? bytes : 1);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(DGX_ENOMEM, "dgx_device_alloc: %zu bytes: %s", bytes, cudaGetErrorString(e));
  }
  return DGX_OK;
}

dgx_status dgx_device_free(void* ptr) { return cuda_status(cudaFree(ptr), "dgx_device_free"); }

dgx_status dgx_copy(void* dst, const void* src, size_t bytes, int direction, void* stream) {
  if (bytes == 0) return DGX_OK;
  if (!dst || !src) return set_error(DGX_EINVAL, "dgx_copy: null pointer");
  const cudaMemcpyKind kinds[3] = {cudaMemcpyHostToDevice, cudaMemcpyDeviceToHost, cudaMemcpyDeviceToDevice};
  if (direction < 0 || direction > 2) return set_error(DGX_EINVAL, "dgx_copy: direction %d", direction);
  return cuda_status(cudaMemcpyAsync(dst, src, bytes, kinds[direction], (cudaStream_t)stream), "dgx_copy");
}

dgx_status dgx_gemm_set_algo(int algo) {
  if (algo != 0 && algo != 1) return set_error(DGX_EINVAL, "dgx_gemm_set_algo: %d", algo);
  gemm_set_algo(algo);
  return DGX_OK;
}

dgx_status dgx_init(int device) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDeviceCount");
  if (device < 0 || device >= n) return set_error(DGX_EINVAL, "dgx_init: device %d of %d", device, n);
  e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_status(e, "cudaSetDevice");
  cudaDeviceProp p;
  e = cudaGetDeviceProperties(&p, device);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDeviceProperties");
  if (p.major != 10) return set_error(DGX_EUNSUPPORTED, "dgx_init: device is sm_%d%d, libdgx is built for sm_100a",
                                      p.major, p.minor);
  if (!get_tensor_map_encoder()) return set_error(DGX_ECUDA, "cuTensorMapEncodeTiled unavailable");
  if (!refresh_error_word()) return set_error(DGX_ECUDA, "dgx_init: cannot find the device error word");
  return DGX_OK;
}

dgx_status dgx_sync_check(void* stream) {
  DGX_FAULT_POINT("dgx_sync_check");
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_status(e, "dgx_sync_check");
  uint32_t* w = device_error_word();
  if (!w) return set_error(DGX_ECUDA, "dgx_sync_check: no device error word");
  uint32_t v = 0;
  e = cudaMemcpy(&v, w, sizeof(v), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_status(e, "dgx_sync_check: read error word");
  if (v) {
    cudaMemset(w, 0, sizeof(uint32_t));
    return set_error(DGX_ETIMEOUT, "device error word 0x%x (1=wait timeout, 2=tmem, 4=bounds)", v);
  }
  return DGX_OK;
}

size_t dgx_gemm_workspace_size(int M, int N, int K, int transA, int transB, dgx_dtype ab_type, int f32_mode) {
  if (ab_type != DGX_F32 || f32_mode != DGX_F32_3XTF32 || M <= 0 || N <= 0 || K <= 0) return 0;
  GemmArgs a{};
  a.M = M;
  a.N = N;
  a.K = K;
  a.transA = transA;
  a.transB = transB;
  return gemm_f32_scratch_floats(a) * sizeof(float);
}

dgx_status dgx_gemm(const void* A, const void* B, void* C, int M, int N, int K, int lda, int ldb, int ldc,
                    int transA, int transB, dgx_dtype ab_type, dgx_dtype c_type, int f32_mode, const float* bias,
                    int epilogue, float beta, void* workspace, size_t workspace_bytes, void* stream) {
  DGX_FAULT_POINT("dgx_gemm");
  if (M < 0 || N < 0 || K < 0) return set_error(DGX_EINVAL, "dgx_gemm: negative size %dx%dx%d", M, N, K);
  if (M == 0 || N == 0) return DGX_OK;
  if (!C || (K > 0 && (!A || !B))) return set_error(DGX_EINVAL, "dgx_gemm: null operand");
  if (ab_type != DGX_F32 && ab_type != DGX_BF16) return set_error(DGX_EINVAL, "dgx_gemm: ab_type %d", ab_type);
  if (c_type != DGX_F32 && c_type != DGX_BF16) return set_error(DGX_EINVAL, "dgx_gemm: c_type %d", c_type);
  if (epilogue < DGX_EPI_NONE || epilogue > DGX_EPI_RELU) return set_error(DGX_EINVAL, "dgx_gemm: epilogue");
  if ((epilogue == DGX_EPI_BIAS || epilogue == DGX_EPI_BIAS_RELU) && !bias)
    return set_error(DGX_EINVAL, "dgx_gemm: bias epilogue without bias");
  const int min_lda = transA ? M : K, min_ldb = transB ? K : N;
  if (lda < min_lda || ldb < min_ldb || ldc < N)
    return set_error(DGX_EINVAL, "dgx_gemm: leading dimension too small (lda %d ldb %d ldc %d)", lda, ldb, ldc);
  cudaStream_t s = (cudaStream_t)stream;
  GemmArgs a{};
  a.M = M;
  a.N = N;
  a.K = K;
  a.lda = lda;
  a.ldb = ldb;
  a.ldc = ldc;
  a.transA = transA ? 1 : 0;
  a.transB = transB ? 1 : 0;
  a.C = C;
  a.c_bf16 = c_type == DGX_BF16;
  a.bias = (epilogue == DGX_EPI_BIAS || epilogue == DGX_EPI_BIAS_RELU) ? bias : nullptr;
  a.relu = (epilogue == DGX_EPI_BIAS_RELU || epilogue == DGX_EPI_RELU);
  a.beta = beta;
  a.err = device_error_word();
  return gemm_run(a, A, B, ab_type, f32_mode, workspace, workspace_bytes, s);
}

}  // extern "C"

namespace dgx {

// Kernel choice for a validated GemmArgs (single or batched product).
dgx_status gemm_run(const GemmArgs& a, const void* A, const void* B, dgx_dtype ab_type, int f32_mode,
                    void* workspace, size_t workspace_bytes, cudaStream_t s) {
  if (a.K == 0) {
    // Degenerate contraction: C = beta*C (+bias)(relu); the SIMT kernel handles it.
    return cuda_status(gemm_simt(a, A, B, ab_type == DGX_BF16, s), "dgx_gemm simt");
  }
  const int esz = ab_type == DGX_BF16 ? 2 : 4;
  const bool tc = gemm_tc_supported(a, esz, A, B);
  if (ab_type == DGX_BF16) {
    if (tc) return cuda_status(gemm_bf16_tc(a, A, B, s), "dgx_gemm bf16");
    return cuda_status(gemm_simt(a, A, B, 1, s), "dgx_gemm bf16 simt");
  }
  // f32 inputs
  if (f32_mode == DGX_F32_3XTF32) {
    const size_t need = gemm_f32_scratch_floats(a) * sizeof(float);
    void* ws = workspace;
    if (ws && workspace_bytes < need)
      return set_error(DGX_ENOMEM, "dgx_gemm: workspace %zu bytes < %zu", workspace_bytes, need);
    if (!ws) ws = library_scratch(need, s);
    if (!ws) return set_error(DGX_ENOMEM, "dgx_gemm: cannot allocate %zu bytes of scratch", need);
    return cuda_status(gemm_f32_3xtf32(a, (const float*)A, (const float*)B, (float*)ws, s), "dgx_gemm 3xtf32");
  }
  if (f32_mode != DGX_F32_3XTF32 && f32_mode != DGX_F32_FFMA)
    return set_error(DGX_EINVAL, "dgx_gemm: f32_mode %d", f32_mode);
  return cuda_status(gemm_simt(a, A, B, 0, s), "dgx_gemm f32 simt");
}

}  // namespace dgx

extern "C" {

dgx_status dgx_gemm_batched(const void* A, const void* B, void* C, int batch, int M, int N, int K, int lda,
                            int ldb, int ldc, long long strideA, long long strideB, long long strideC, int transA,
                            int transB, dgx_dtype ab_type, dgx_dtype c_type, float beta, void* stream) {
  DGX_FAULT_POINT("dgx_gemm_batched");
  if (batch < 0 || M < 0 || N < 0 || K < 0)
    return set_error(DGX_EINVAL, "dgx_gemm_batched: negative size %d x %dx%dx%d", batch, M, N, K);
  if (batch == 0 || M == 0 || N == 0) return DGX_OK;
  if (!C || (K > 0 && (!A || !B))) return set_error(DGX_EINVAL, "dgx_gemm_batched: null operand");
  if (ab_type != DGX_F32 && ab_type != DGX_BF16) return set_error(DGX_EINVAL, "dgx_gemm_batched: ab_type %d", ab_type);
  if (c_type != DGX_F32 && c_type != DGX_BF16) return set_error(DGX_EINVAL, "dgx_gemm_batched: c_type %d", c_type);
  const int min_lda = transA ? M : K, min_ldb = transB ? K : N;
  if (lda < min_lda || ldb < min_ldb || ldc < N)
    return set_error(DGX_EINVAL, "dgx_gemm_batched: leading dimension too small (lda %d ldb %d ldc %d)", lda, ldb,
                     ldc);
  // Operands may overlap or repeat across batches (stride 0 broadcasts one
  // operand); the outputs may not.
  if (batch > 1 && (strideA < 0 || strideB < 0 || strideC < (long long)M * ldc))
    return set_error(DGX_EINVAL, "dgx_gemm_batched: bad batch strides (%lld %lld %lld)", strideA, strideB, strideC);
  const size_t esz = ab_type == DGX_BF16 ? 2 : 4, csz = c_type == DGX_BF16 ? 2 : 4;
  // One launch per chunk of batches (the grid's z extent bounds the split and
  // fallback kernels to 32767 batches a launch).
  constexpr int kMaxBatch = 32767;
  for (int b0 = 0; b0 < batch; b0 += kMaxBatch) {
    GemmArgs a{};
    a.M = M;
    a.N = N;
    a.K = K;
    a.lda = lda;
    a.ldb = ldb;
    a.ldc = ldc;
    a.transA = transA ? 1 : 0;
    a.transB = transB ? 1 : 0;
    a.C = (char*)C + (size_t)b0 * strideC * csz;
    a.c_bf16 = c_type == DGX_BF16;
    a.beta = beta;
    a.err = device_error_word();
    a.batch = batch - b0 < kMaxBatch ? batch - b0 : kMaxBatch;
    a.sA = strideA;
    a.sB = strideB;
    a.sC = strideC;
    dgx_status st = gemm_run(a, (const char*)A + (size_t)b0 * strideA * esz, (const char*)B + (size_t)b0 * strideB * esz,
                             ab_type, DGX_F32_3XTF32, nullptr, 0, (cudaStream_t)stream);
    if (st != DGX_OK) return st;
  }
  return DGX_OK;
}

dgx_status dgx_bmm(const void* A, const void* B, void* C, int batch, int M, int N, int K, dgx_dtype ab_type,
                   dgx_dtype c_type, void* stream) {
  return dgx_gemm_batched(A, B, C, batch, M, N, K, K, N, N, (long long)M * K, (long long)K * N, (long long)M * N, 0,
                          0, ab_type, c_type, 0.f, stream);
}

}  // extern "C"
