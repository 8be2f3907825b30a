// Column-parallel tensor-parallel GEMM with the all-gather fused into the
// GEMM epilogue, one process per GPU.
//
// Replaces dream_tp_matmul_column (runtime/nn/training.inc:1604-1630): there
// each column shard Y_g = X . W[:, shard g] runs in turn in one process and
// the "all-gather" is a host copy into Y[:, col:col+ncol] (the comment at
// :1622 names ncclAllGather). Here rank r computes its shard on its own GPU
// and the epilogue stores every output tile into C_full of ALL ranks: the
// local copy plus NVLink peer stores through CUDA IPC mappings. The transfer
// of tile t overlaps the MMAs of tile t+1; no separate collective runs.
//
// Completion: after the GEMM kernel, a one-warp kernel raises this call's
// epoch in every rank's flag slot for this rank (system-scope release) and
// then waits, bounded, until every rank's flag in its own slot array shows
// the epoch (system-scope acquire). A rank that never arrives makes the wait
// time out: the kernel records DGX_DEV_ERR_TIMEOUT and returns, and the host
// reports DGX_ETIMEOUT from dgx_sync_check / the call's own check.
#include <cstring>
#include <mutex>

#include "common.h"
#include "gemm.h"
#include "sm100.cuh"

namespace dgx {
namespace {

constexpr int kMaxRanks = 8;

struct TpHandle {  // what one rank publishes (opaque to callers)
  cudaIpcMemHandle_t c_mem;
  uint64_t c_offset;  // C_full - allocation base
  uint64_t c_bytes;
  cudaIpcMemHandle_t flag_mem;
};

struct TpState {
  int rank = -1, world = 0;
  void* c_local = nullptr;
  size_t c_bytes = 0;
  unsigned long long* flags = nullptr;  // [kMaxRanks] slots, written by peers
  void* peer_c[kMaxRanks] = {};
  unsigned long long* peer_flags[kMaxRanks] = {};
  void* opened[2 * kMaxRanks] = {};
  int n_opened = 0;
  unsigned long long epoch = 0;
};

std::mutex g_tp_mu;
TpState g_tp;

typedef CUresult (*AddrRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);
AddrRangeFn addr_range_fn() {
  static AddrRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddrRangeFn>(p);
  });
  return fn;
}

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

struct SignalArgs {
  unsigned long long* peer_flags[kMaxRanks];  // peer r's slot array (own array for r == rank)
  unsigned long long* my_flags;
  int rank, world;
  unsigned long long epoch;
  long long budget_cycles;
  uint32_t* err;
};

// Wait until *flag >= epoch (system-scope acquire), at most budget_cycles
// SM clocks; on running out record DGX_DEV_ERR_TIMEOUT and return false.
__device__ __forceinline__ bool bounded_flag_wait(const unsigned long long* flag, unsigned long long epoch,
                                                  long long budget_cycles, uint32_t* err) {
  const long long t0 = clock64();
  while (ld_acquire_sys(flag) < epoch) {
    if (clock64() - t0 > budget_cycles) {
      if (err) atomicOr(err, DGX_DEV_ERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

// Lane i < world: publish "rank done" into rank i's slot array, then wait for
// slot i of our own array. Runs after the GEMM kernel on the same stream, so
// every peer store of this rank's tiles precedes the release.
__global__ void tp_signal_wait_kernel(SignalArgs a) {
  const int i = threadIdx.x;
  if (i < a.world) {
    __threadfence_system();
    st_release_sys(a.peer_flags[i] + a.rank, a.epoch);
    bounded_flag_wait(a.my_flags + i, a.epoch, a.budget_cycles, a.err);
  }
}

// dgx_wait_probe: one warp runs one of the library's bounded waits.
//   kind 0: the cross-rank completion wait above, on `flag`, `budget_cycles`.
//   kind 1: the mbarrier wait every tensor-core kernel pipeline uses
//           (mbar_wait, its fixed budget of about a second); when `expect` is
//           0 the probe completes the barrier phase itself first.
__global__ void wait_probe_kernel(int kind, const unsigned long long* flag, unsigned long long expect,
                                  long long budget_cycles, uint32_t* err) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x != 0) return;
  if (kind == 0) {
    bounded_flag_wait(flag, expect, budget_cycles, err);
    return;
  }
  abort_flag = 0;
  mbar_init(&bar, 1);
  fence_mbar_init();
  if (expect == 0) mbar_arrive(&bar);
  WaitCtx wc{&abort_flag, err};
  mbar_wait(&bar, 0, wc);
}

}  // namespace
}  // namespace dgx

using namespace dgx;

extern "C" {

void dgx_tp_shard(int N, int world, int rank, int* col0, int* ncol) {
  if (world < 1) world = 1;
  const int base = N / world, rem = N % world;
  *ncol = base + (rank < rem ? 1 : 0);
  *col0 = rank * base + (rank < rem ? rank : rem);
}

size_t dgx_tp_handle_size(void) { return sizeof(TpHandle); }

dgx_status dgx_tp_export(void* C_full, size_t c_bytes, void* handle_out, size_t handle_bytes) {
  if (!C_full || !handle_out) return set_error(DGX_EINVAL, "dgx_tp_export: null pointer");
  if (handle_bytes < sizeof(TpHandle)) return set_error(DGX_EINVAL, "dgx_tp_export: handle buffer too small");
  std::lock_guard<std::mutex> lk(g_tp_mu);
  TpHandle h{};
  CUdeviceptr base = 0;
  size_t size = 0;
  auto range = addr_range_fn();
  if (!range || range(&base, &size, (CUdeviceptr)C_full) != CUDA_SUCCESS)
    return set_error(DGX_ECUDA, "dgx_tp_export: cannot resolve the allocation of C_full");
  cudaError_t e = cudaIpcGetMemHandle(&h.c_mem, (void*)base);
  if (e != cudaSuccess) return cuda_status(e, "dgx_tp_export: cudaIpcGetMemHandle(C_full)");
  h.c_offset = (uint64_t)((CUdeviceptr)C_full - base);
  h.c_bytes = c_bytes;
  if (!g_tp.flags) {
    e = cudaMalloc(&g_tp.flags, kMaxRanks * sizeof(unsigned long long));
    if (e != cudaSuccess) return cuda_status(e, "dgx_tp_export: flags");
    cudaMemset(g_tp.flags, 0, kMaxRanks * sizeof(unsigned long long));
    g_tp.epoch = 0;
  }
  e = cudaIpcGetMemHandle(&h.flag_mem, g_tp.flags);
  if (e != cudaSuccess) return cuda_status(e, "dgx_tp_export: cudaIpcGetMemHandle(flags)");
  g_tp.c_local = C_full;
  g_tp.c_bytes = c_bytes;
  std::memcpy(handle_out, &h, sizeof(h));
  return DGX_OK;
}

dgx_status dgx_tp_open(int rank, int world, const void* handles) {
  DGX_FAULT_POINT("dgx_tp_open");
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
    return set_error(DGX_EINVAL, "dgx_tp_open: rank %d of world %d (max %d)", rank, world, kMaxRanks);
  if (!handles) return set_error(DGX_EINVAL, "dgx_tp_open: null handles");
  std::lock_guard<std::mutex> lk(g_tp_mu);
  if (!g_tp.c_local || !g_tp.flags) return set_error(DGX_EINVAL, "dgx_tp_open: call dgx_tp_export first");
  const TpHandle* hs = static_cast<const TpHandle*>(handles);
  g_tp.rank = rank;
  g_tp.world = world;
  for (int r = 0; r < world; ++r) {
    if (r == rank) {
      g_tp.peer_c[r] = g_tp.c_local;
      g_tp.peer_flags[r] = g_tp.flags;
      continue;
    }
    if (hs[r].c_bytes != g_tp.c_bytes)
      return set_error(DGX_EINVAL, "dgx_tp_open: rank %d exported %llu bytes, this rank %zu", r,
                       (unsigned long long)hs[r].c_bytes, g_tp.c_bytes);
    void* pc = nullptr;
    void* pf = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&pc, hs[r].c_mem, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_status(e, "dgx_tp_open: cudaIpcOpenMemHandle(C)");
    g_tp.opened[g_tp.n_opened++] = pc;
    e = cudaIpcOpenMemHandle(&pf, hs[r].flag_mem, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_status(e, "dgx_tp_open: cudaIpcOpenMemHandle(flags)");
    g_tp.opened[g_tp.n_opened++] = pf;
    g_tp.peer_c[r] = static_cast<char*>(pc) + hs[r].c_offset;
    g_tp.peer_flags[r] = static_cast<unsigned long long*>(pf);
  }
  return DGX_OK;
}

dgx_status dgx_tp_gemm_colsplit(const void* A, const void* B_shard, int M, int N, int K, dgx_dtype ab_type,
                                dgx_dtype c_type, int timeout_ms, void* stream) {
  DGX_FAULT_POINT("dgx_tp_gemm_colsplit");
  if (M < 0 || N < 0 || K < 0) return set_error(DGX_EINVAL, "dgx_tp_gemm_colsplit: negative size");
  if (ab_type != DGX_BF16 && ab_type != DGX_F32) return set_error(DGX_EINVAL, "dgx_tp_gemm_colsplit: ab_type");
  if (c_type != DGX_BF16 && c_type != DGX_F32) return set_error(DGX_EINVAL, "dgx_tp_gemm_colsplit: c_type");
  std::lock_guard<std::mutex> lk(g_tp_mu);
  if (g_tp.world < 1) return set_error(DGX_EINVAL, "dgx_tp_gemm_colsplit: call dgx_tp_open first");
  const size_t csz = c_type == DGX_BF16 ? 2 : 4;
  if ((size_t)M * N * csz > g_tp.c_bytes)
    return set_error(DGX_EINVAL, "dgx_tp_gemm_colsplit: C_full holds %zu bytes, M*N needs %zu", g_tp.c_bytes,
                     (size_t)M * N * csz);
  cudaStream_t s = (cudaStream_t)stream;
  int col0 = 0, ncol = 0;
  dgx_tp_shard(N, g_tp.world, g_tp.rank, &col0, &ncol);
  if (ncol > 0 && M > 0) {
    if (!A || !B_shard) return set_error(DGX_EINVAL, "dgx_tp_gemm_colsplit: null operand");
    GemmArgs a{};
    a.M = M;
    a.N = ncol;
    a.K = K;
    a.lda = K;
    a.ldb = ncol;
    a.ldc = N;
    a.C = static_cast<char*>(g_tp.c_local) + (size_t)col0 * csz;
    a.c_bf16 = c_type == DGX_BF16;
    a.err = device_error_word();
    for (int r = 0; r < g_tp.world; ++r)
      if (r != g_tp.rank) a.C_extra[a.n_extra++] = static_cast<char*>(g_tp.peer_c[r]) + (size_t)col0 * csz;
    cudaError_t e;
    if (ab_type == DGX_BF16 && gemm_tc_supported(a, 2, A, B_shard)) {
      e = gemm_bf16_tc(a, A, B_shard, s);
    } else if (ab_type == DGX_F32) {
      const size_t need = gemm_f32_scratch_floats(a) * sizeof(float);
      void* ws = library_scratch(need, s);
      if (!ws) return set_error(DGX_ENOMEM, "dgx_tp_gemm_colsplit: scratch");
      e = gemm_f32_3xtf32(a, (const float*)A, (const float*)B_shard, (float*)ws, s);
    } else {
      e = gemm_simt(a, A, B_shard, 1, s);
    }
    if (e != cudaSuccess) return cuda_status(e, "dgx_tp_gemm_colsplit gemm");
  }
  SignalArgs sa{};
  for (int r = 0; r < g_tp.world; ++r) sa.peer_flags[r] = g_tp.peer_flags[r];
  sa.my_flags = g_tp.flags;
  sa.rank = g_tp.rank;
  sa.world = g_tp.world;
  sa.epoch = ++g_tp.epoch;
  const long long ms = timeout_ms > 0 ? timeout_ms : 10000;
  sa.budget_cycles = ms * 2000000ll;  // ~2 GHz SM clock
  sa.err = device_error_word();
  tp_signal_wait_kernel<<<1, 32, 0, s>>>(sa);
  return cuda_status(cudaGetLastError(), "dgx_tp_gemm_colsplit signal");
}

dgx_status dgx_wait_probe(int kind, const unsigned long long* flag, unsigned long long expect, int timeout_us,
                          void* stream) {
  DGX_FAULT_POINT("dgx_wait_probe");
  if (kind != 0 && kind != 1) return set_error(DGX_EINVAL, "dgx_wait_probe: kind %d", kind);
  if (kind == 0 && !flag) return set_error(DGX_EINVAL, "dgx_wait_probe: null flag");
  if (timeout_us < 0) return set_error(DGX_EINVAL, "dgx_wait_probe: negative timeout");
  const long long budget = (long long)timeout_us * 2000ll;  // ~2 GHz SM clock
  wait_probe_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(kind, flag, expect, budget, device_error_word());
  return cuda_status(cudaGetLastError(), "dgx_wait_probe");
}

dgx_status dgx_tp_close(void) {
  std::lock_guard<std::mutex> lk(g_tp_mu);
  cudaDeviceSynchronize();
  for (int i = 0; i < g_tp.n_opened; ++i) cudaIpcCloseMemHandle(g_tp.opened[i]);
  if (g_tp.flags) cudaFree(g_tp.flags);
  g_tp = TpState{};
  return DGX_OK;
}

}  // extern "C"
