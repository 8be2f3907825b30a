// Tensor-parallel entry points whose kernels are not in this build yet: they return
// DGX_EUNSUPPORTED so the ABI stays complete and callers fail loudly.
#include "common.h"
using namespace dgx;
extern "C" {
void dgx_tp_shard(int N, int world, int rank, int* col0, int* ncol) {
  int base = N / world, rem = N % world;
  *ncol = base + (rank < rem ? 1 : 0);
  *col0 = rank * base + (rank < rem ? rank : rem);
}
dgx_status dgx_tp_export(void*, size_t, void*, size_t) { return set_error(DGX_EUNSUPPORTED, "not built"); }
size_t dgx_tp_handle_size(void) { return 0; }
dgx_status dgx_tp_open(int, int, const void*) { return set_error(DGX_EUNSUPPORTED, "not built"); }
dgx_status dgx_tp_gemm_colsplit(const void*, const void*, int, int, int, dgx_dtype, dgx_dtype, int, void*) {
  return set_error(DGX_EUNSUPPORTED, "not built");
}
dgx_status dgx_tp_close(void) { return DGX_OK; }
}
