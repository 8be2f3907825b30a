// C ABI entry points of the FlashAttention kernels (include/dgx.h).
#include "common.h"
#include "flash.h"

using namespace dgx;

extern "C" {

size_t dgx_flash_bwd_workspace_size(int BH, int S, int D) {
  if (BH <= 0 || S <= 0 || D <= 0) return 0;
  return flash_bwd_scratch_bytes(BH, S, D);
}

dgx_status dgx_flash_fwd(const void* Q, const void* K, const void* V, void* O, float* LSE, int BH, int S, int D,
                         float scale, int causal, dgx_dtype dtype, void* stream) {
  if (BH < 0 || S < 0 || D <= 0) return set_error(DGX_EINVAL, "dgx_flash_fwd: bad size BH=%d S=%d D=%d", BH, S, D);
  if (dtype != DGX_BF16) return set_error(DGX_EUNSUPPORTED, "dgx_flash_fwd: dtype %d (bf16 only)", dtype);
  if (BH == 0 || S == 0) return DGX_OK;
  if (!Q || !K || !V || !O) return set_error(DGX_EINVAL, "dgx_flash_fwd: null tensor");
  FlashFwdArgs a{Q, K, V, O, LSE, BH, S, D, scale, causal ? 1 : 0, device_error_word()};
  cudaStream_t s = (cudaStream_t)stream;
  const void* ptrs[4] = {Q, K, V, O};
  if (flash_tc_supported(D, ptrs, 4)) return cuda_status(flash_fwd_tc(a, s), "dgx_flash_fwd");
  if (D > 256) return set_error(DGX_EUNSUPPORTED, "dgx_flash_fwd: D=%d > 256", D);
  return cuda_status(flash_fwd_simt(a, s), "dgx_flash_fwd simt");
}

dgx_status dgx_flash_bwd(const void* Q, const void* K, const void* V, const void* O, const void* dO,
                         const float* LSE, void* dQ, void* dK, void* dV, int BH, int S, int D, float scale,
                         int causal, dgx_dtype dtype, void* workspace, size_t workspace_bytes, void* stream) {
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
  const void* ptrs[9] = {Q, K, V, O, dO, dQ, dK, dV, LSE};
  if (flash_tc_supported(D, ptrs, 9)) return cuda_status(flash_bwd_tc(a, s), "dgx_flash_bwd");
  return cuda_status(flash_bwd_simt(a, s), "dgx_flash_bwd simt");
}

}  // extern "C"
