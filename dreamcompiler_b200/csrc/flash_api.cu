// C ABI entry points of the FlashAttention kernels (include/dgx.h).
#include "common.h"
#include "flash.h"

using namespace dgx;

extern "C" {

dgx_status dgx_flash_set_deterministic(int on) {
  flash_set_deterministic(on != 0);
  return DGX_OK;
}

size_t dgx_flash_bwd_workspace_size(int BH, int S, int D) {
  if (BH <= 0 || S <= 0 || D <= 0) return 0;
  return flash_bwd_scratch_bytes(BH, S, D);
}

dgx_status dgx_flash_fwd(const void* Q, const void* K, const void* V, void* O, float* LSE, int BH, int S, int D,
                         float scale, int causal, dgx_dtype dtype, void* stream) {
  DGX_FAULT_POINT("dgx_flash_fwd");
  if (BH < 0 || S < 0 || D <= 0) return set_error(DGX_EINVAL, "dgx_flash_fwd: bad size BH=%d S=%d D=%d", BH, S, D);
  if (dtype != DGX_BF16) return set_error(DGX_EUNSUPPORTED, "dgx_flash_fwd: dtype %d (bf16 only)", dtype);
  if (BH == 0 || S == 0) return DGX_OK;
  if (!Q || !K || !V || !O) return set_error(DGX_EINVAL, "dgx_flash_fwd: null tensor");
  FlashFwdArgs a{Q, K, V, O, LSE, BH, S, D, scale, causal ? 1 : 0, device_error_word()};
  flash_dense_layout(a);
  cudaStream_t s = (cudaStream_t)stream;
  const void* ptrs[4] = {Q, K, V, O};
  if (flash_tc_supported(D, kFlashFwdMaxD, ptrs, 4)) return cuda_status(flash_fwd_tc(a, s), "dgx_flash_fwd");
  if (D > 256) return set_error(DGX_EUNSUPPORTED, "dgx_flash_fwd: D=%d > 256", D);
  return cuda_status(flash_fwd_simt(a, s), "dgx_flash_fwd simt");
}

dgx_status dgx_flash_bwd(const void* Q, const void* K, const void* V, const void* O, const void* dO,
                         const float* LSE, void* dQ, void* dK, void* dV, int BH, int S, int D, float scale,
                         int causal, dgx_dtype dtype, void* workspace, size_t workspace_bytes, void* stream) {
  DGX_FAULT_POINT("dgx_flash_bwd");
  if (BH < 0 || S < 0 || D <= 0) return set_error(DGX_EINVAL, "dgx_flash_bwd: bad size BH=%d S=%d D=%d", BH, S, D);
  if (dtype != DGX_BF16) return set_error(DGX_EUNSUPPORTED, "dgx_flash_bwd: dtype %d (bf16 only)", dtype);
  if (BH == 0 || S == 0) return DGX_OK;
  if (!Q || !K || !V || !O || !dO || !LSE || !dQ || !dK || !dV)
    return set_error(DGX_EINVAL, "dgx_flash_bwd: null tensor");
  if (D > 256) return set_error(DGX_EUNSUPPORTED, "dgx_flash_bwd: D=%d > 256", D);
  cudaStream_t s = (cudaStream_t)stream;
  const size_t need = flash_bwd_scratch_bytes(BH, S, D);
  void* ws = workspace;
  if (ws && workspace_bytes < need)
    return set_error(DGX_ENOMEM, "dgx_flash_bwd: workspace %zu bytes < %zu", workspace_bytes, need);
  if (ws && ((uintptr_t)ws & 15)) return set_error(DGX_EINVAL, "dgx_flash_bwd: workspace must be 16-byte aligned");
  if (!ws) ws = library_scratch(need, s);
  if (!ws) return set_error(DGX_ENOMEM, "dgx_flash_bwd: cannot allocate %zu bytes of scratch", need);
  FlashBwdArgs a{Q, K, V, O, dO, LSE, dQ, dK, dV, (float*)ws, (float*)ws + (size_t)BH * S * D,
                 BH, S, D, flash_spad(S), scale, causal ? 1 : 0, device_error_word()};
  a.own_ws = workspace != nullptr;
  flash_dense_layout(a);
  const void* ptrs[9] = {Q, K, V, O, dO, dQ, dK, dV, LSE};
  if (flash_tc_supported(D, kFlashBwdMaxD, ptrs, 9)) return cuda_status(flash_bwd_tc(a, s), "dgx_flash_bwd");
  return cuda_status(flash_bwd_simt(a, s), "dgx_flash_bwd simt");
}

// Checks shared by the head-row entry points: the tensor-core kernels take
// D % 8 == 0 up to their limit, and TMA wants 16-byte aligned bases and pitches.
static dgx_status rows_check(const char* op, int B, int H, int S, int D, int max_d, const void* const* ptrs,
                             const int* lds, int n) {
  if (B < 0 || H <= 0 || S < 0 || D <= 0) return set_error(DGX_EINVAL, "%s: bad size B=%d H=%d S=%d D=%d", op, B, H, S, D);
  if (D % 8 || D > max_d)
    return set_error(DGX_EUNSUPPORTED, "%s: D=%d (the head-row form takes D %% 8 == 0, D <= %d)", op, D, max_d);
  if ((long long)B * H * S * D >= (1LL << 31)) return set_error(DGX_EINVAL, "%s: B*H*S*D >= 2^31", op);
  for (int i = 0; i < n; ++i) {
    if (!ptrs[i]) return set_error(DGX_EINVAL, "%s: null tensor", op);
    if ((uintptr_t)ptrs[i] & 15) return set_error(DGX_EINVAL, "%s: tensors must be 16-byte aligned", op);
  }
  for (int i = 0; i < n; ++i)
    if (lds[i] < H * D || lds[i] % 8) return set_error(DGX_EINVAL, "%s: row pitch %d (>= H*D and a multiple of 8)", op, lds[i]);
  return DGX_OK;
}

dgx_status dgx_flash_fwd_rows(const void* Q, int ldq, const void* K, int ldk, const void* V, int ldv, void* O,
                              int ldo, float* LSE, int B, int H, int S, int D, float scale, int causal, void* stream) {
  DGX_FAULT_POINT("dgx_flash_fwd_rows");
  const void* ptrs[4] = {Q, K, V, O};
  const int lds[4] = {ldq, ldk, ldv, ldo};
  dgx_status st = rows_check("dgx_flash_fwd_rows", B, H, S, D, kFlashFwdMaxD, ptrs, lds, 4);
  if (st != DGX_OK) return st;
  if (B == 0 || S == 0) return DGX_OK;
  FlashFwdArgs a{Q, K, V, O, LSE, B * H, S, D, scale, causal ? 1 : 0, device_error_word()};
  a.H = H;
  a.ldq = ldq;
  a.ldk = ldk;
  a.ldv = ldv;
  a.ldo = ldo;
  return cuda_status(flash_fwd_tc(a, (cudaStream_t)stream), "dgx_flash_fwd_rows");
}

dgx_status dgx_flash_bwd_rows(const void* Q, int ldq, const void* K, int ldk, const void* V, int ldv, const void* O,
                              int ldo, const void* dO, int lddo, const float* LSE, void* dQ, int lddq, void* dK,
                              int lddk, void* dV, int lddv, int B, int H, int S, int D, float scale, int causal,
                              void* workspace, size_t workspace_bytes, void* stream) {
  DGX_FAULT_POINT("dgx_flash_bwd_rows");
  const void* ptrs[8] = {Q, K, V, O, dO, dQ, dK, dV};
  const int lds[8] = {ldq, ldk, ldv, ldo, lddo, lddq, lddk, lddv};
  dgx_status st = rows_check("dgx_flash_bwd_rows", B, H, S, D, kFlashBwdMaxD, ptrs, lds, 8);
  if (st != DGX_OK) return st;
  if (!LSE) return set_error(DGX_EINVAL, "dgx_flash_bwd_rows: null LSE");
  if (B == 0 || S == 0) return DGX_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const int BH = B * H;
  const size_t need = flash_bwd_scratch_bytes(BH, S, D);
  void* ws = workspace;
  if (ws && workspace_bytes < need)
    return set_error(DGX_ENOMEM, "dgx_flash_bwd_rows: workspace %zu bytes < %zu", workspace_bytes, need);
  if (ws && ((uintptr_t)ws & 15)) return set_error(DGX_EINVAL, "dgx_flash_bwd_rows: workspace must be 16-byte aligned");
  if (!ws) ws = library_scratch(need, s);
  if (!ws) return set_error(DGX_ENOMEM, "dgx_flash_bwd_rows: cannot allocate %zu bytes of scratch", need);
  FlashBwdArgs a{Q, K, V, O, dO, LSE, dQ, dK, dV, (float*)ws, (float*)ws + (size_t)BH * S * D,
                 BH, S, D, flash_spad(S), scale, causal ? 1 : 0, device_error_word()};
  a.own_ws = workspace != nullptr;
  a.H = H;
  a.ldq = ldq;
  a.ldk = ldk;
  a.ldv = ldv;
  a.ldo = ldo;
  a.lddo = lddo;
  a.lddq = lddq;
  a.lddk = lddk;
  a.lddv = lddv;
  return cuda_status(flash_bwd_tc(a, s), "dgx_flash_bwd_rows");
}

}  // extern "C"
