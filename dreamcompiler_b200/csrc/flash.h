// Internal interface of the FlashAttention kernels.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dgx {

// Head layout of a tensor: head h of batch b, position s, starts at element
// (b*S + s)*ld + h*D of its base pointer, with BH = B*H. [BH][S][D] is H = 1,
// ld = D; the token rows a fused QKV projection writes ([B*S][3*H*D], Q, K, V
// at column offsets 0, H*D, 2*H*D folded into the base) are H heads, ld = 3*H*D.
struct FlashFwdArgs {
  const void* Q;
  const void* K;
  const void* V;
  void* O;
  float* lse;  // [BH*S] natural log, or null
  int BH, S, D;
  float scale;
  int causal;
  uint32_t* err;
  int H;                    // heads per batch row (1: the [BH][S][D] layout)
  int ldq, ldk, ldv, ldo;   // row pitches (elements)
};

struct FlashBwdArgs {
  const void* Q;
  const void* K;
  const void* V;
  const void* O;
  const void* dO;
  const float* lse;
  void* dQ;
  void* dK;
  void* dV;
  float* dq_acc;   // [BH*S*D] fp32 scratch
  float* rowstat;  // [2][BH][Spad] scratch: D_i = dO_i.O_i, then LSE_i*log2(e) (+inf past S)
  int BH, S, D;
  int Spad;        // S rounded up to 128: every 128-row slice of rowstat is in bounds and aligned
  float scale;
  int causal;
  uint32_t* err;
  int zero_acc;    // the row pre-pass also zeroes dq_acc (tensor-core path)
  int H;                                        // heads per batch row (1: [BH][S][D])
  int ldq, ldk, ldv, ldo, lddo, lddq, lddk, lddv;  // row pitches (elements); dq_acc stays [BH][S][D]
  int dense3d;     // set by the launcher: every tensor is [BH][S][D], loaded through 3-D maps
  int own_ws;      // the caller's workspace (not library scratch): its zeroing may overlap the kernel before
};

// The [BH][S][D] layout for every tensor.
inline void flash_dense_layout(FlashFwdArgs& a) {
  a.H = 1;
  a.ldq = a.ldk = a.ldv = a.ldo = a.D;
}
inline void flash_dense_layout(FlashBwdArgs& a) {
  a.H = 1;
  a.ldq = a.ldk = a.ldv = a.ldo = a.lddo = a.lddq = a.lddk = a.lddv = a.D;
}

// Scratch bytes the backward needs (dQ accumulator + padded row statistics).
inline int flash_spad(int S) { return (S + 127) / 128 * 128; }
size_t flash_bwd_scratch_bytes(int BH, int S, int D);

// Head dims the tensor-core kernels take: D % 8 == 0, D <= 128. The backward
// runs one kernel for D <= 64 (dQ reduced through an fp32 accumulator) and two
// for 64 < D <= 128, or for any D in deterministic mode (dK/dV per key tile,
// dQ per query tile).
constexpr int kFlashFwdMaxD = 128, kFlashBwdMaxD = 128;
bool flash_tc_supported(int D, int max_d, const void* const* ptrs, int n);
bool make_head_map(CUtensorMap* map, const void* base, int BH, int H, int S, int D, int ld);
cudaError_t flash_fwd_tc(const FlashFwdArgs& a, cudaStream_t s);
cudaError_t flash_bwd_tc(const FlashBwdArgs& a, cudaStream_t s);
// Two kernels with one owner per gradient element (dK/dV per key tile, dQ
// per query tile): D <= 128, bit-reproducible.
cudaError_t flash_bwd_split_tc(const FlashBwdArgs& a, cudaStream_t s);
// Whether backward calls with D <= 64 take the split, reproducible path too.
void flash_set_deterministic(bool on);
bool flash_deterministic();
// The backward's row pre-pass alone: D_i and LSE_i*log2 e into a.rowstat.
cudaError_t flash_bwd_rowstats(const FlashBwdArgs& a, cudaStream_t s);
// SIMT kernels for head dims the tensor-core kernels do not take (D % 8 != 0,
// or D above the kernel's limit): fp32 math, one thread per query row / key row.
cudaError_t flash_fwd_simt(const FlashFwdArgs& a, cudaStream_t s);
cudaError_t flash_bwd_simt(const FlashBwdArgs& a, cudaStream_t s);

}  // namespace dgx
