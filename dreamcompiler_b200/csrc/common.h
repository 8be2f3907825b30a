// Host-side plumbing shared by the libdgx translation units: the driver-API
// tensor-map encoder (fetched through the runtime, so libdgx does not link
// libcuda directly), SM count, the per-thread error string and the device
// error word that bounded waits report into.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/dgx.h"

namespace dgx {

typedef CUresult (*TensorMapEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                      const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                      CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                      CUtensorMapFloatOOBfill);

TensorMapEncodeFn get_tensor_map_encoder();
int num_sms();
uint32_t* device_error_word();  // per-device word in global memory

// Host-side fault injection (dgx_fault_inject, or DGX_FAIL_AT=<n>[:<status>]
// in the environment): every entry point that launches device work counts
// its calls; the n-th returns the chosen status with a message, launching
// nothing. Failure handling above the library is tested this way without a
// device fault.
bool fault_fires(const char* entry, dgx_status* st);
#define DGX_FAULT_POINT(entry)                     \
  do {                                             \
    dgx_status fault_st_;                          \
    if (dgx::fault_fires(entry, &fault_st_)) return fault_st_; \
  } while (0)

// Record a message as the calling thread's last error and return `st`.
dgx_status set_error(dgx_status st, const char* fmt, ...);
dgx_status cuda_status(cudaError_t e, const char* what);

// Per-device scratch buffers owned by the library (grown on demand with
// cudaMalloc, reused across calls on the same stream order). Separate slots
// for buffers that are live at the same time within one call: the GEMM's
// split-K partial tiles (kScratchSplitK) while its operands may sit in the
// general buffer (the 3xTF32 planes); the convolution's im2col matrices
// (kScratchConv) while its GEMMs use both.
constexpr int kScratchGeneral = 0, kScratchSplitK = 1, kScratchConv = 2, kScratchSlots = 3;
void* library_scratch_slot(int slot, size_t bytes, cudaStream_t s);
void* library_scratch(size_t bytes, cudaStream_t s);  // the general slot

// Brackets one kernel launch with the events set by dgx_set_timer_events
// (if any), then clears them. Construct right before the launch.
struct TimerScope {
  cudaStream_t s;
  cudaEvent_t stop;
  explicit TimerScope(cudaStream_t st);
  ~TimerScope();
};

}  // namespace dgx
