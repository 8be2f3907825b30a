// Tensor-core int8 dense layer on sm_100a: tcgen05.mma kind::i8, exact int32
// accumulation in TMEM.
//
// The layer is y[b,n] = bias[n] + scale[n] * sum_k x[b,k]*w[n,k] with an
// int8 weight matrix W[N][K] (the exported dense_q of the reference,
// runtime/nn/training.inc:3738-3752, with per-output-channel scales). At the
// batch sizes it serves (1..256 rows) the weight stream dominates, so the
// problem is laid out "swap-AB": the weight rows are the MMA's M side (128
// output channels per CTA, one per TMEM lane) and the activation rows are
// its N side (16..256 columns). The weights arrive by TMA in 16 KiB stages
// (128 channels x 128 bytes of K) and are read from HBM exactly once.
//
// Activations reach the tensor cores as int8 planes:
//   W8A8 (1 plane)  : the per-row quantised activations; the int32 sums are
//                     the exact integer dot products of the reference's
//                     W8A8 semantics.
//   W8A32 (3 planes): fp32 activations split exactly as
//                     x = 2^e_b * (q0 + q1/2^7 + q2/2^14 + r), |q0| <= 127,
//                     |q1|,|q2| <= 64, |r| <= 2^-15, with 2^e_b the power of
//                     two that puts the row's largest |x| in (63.5, 127].
//                     The three int32 sums combine exactly in int64 and are
//                     rounded once to fp32, so the only error is r: below
//                     5e-7 of the row's largest |x|, less than the fp32
//                     summation error of the reference loop.
//
// Large batches are cut into chunks of activation rows, one CTA per
// (output tile, chunk). Small batches leave too few output tiles (32 for
// N = 4096), so K is split over the CTAs of a thread-block cluster instead:
// each CTA stores its partial int32 sums straight from TMEM into the shared
// memory of the CTA that finishes those activation rows (distributed shared
// memory), one cluster barrier later every CTA sums its rows locally. Integer
// sums are exact, so the result does not depend on the split; there is no
// global scratch and no second launch.
#include <algorithm>

#include "common.h"
#include "sm100.cuh"
#include "w8.h"

namespace dgx {

namespace {

constexpr int TC_BM = 128;        // output channels per CTA
constexpr int TC_BK = 128;        // K bytes per stage: one 128-byte swizzled row
constexpr int TC_THREADS = 192;   // warps 0-3 epilogue, 4 TMA, 5 MMA
constexpr int TC_MAX_STAGES = 8;
constexpr int TC_SMEM_BUDGET = 200 * 1024;
constexpr int TC_W_BYTES = TC_BM * TC_BK;

struct W8TcArgs {
  const float* scale;
  const float* bias;
  const float* rowscale;
  float* Y;
  int32_t* acc_out;
  int B, N, K;
  int planes;       // 1 or 3
  int bc;           // activation rows per chunk (multiple of 16)
  int ncols;        // planes * bc: MMA N and accumulator columns
  int tmem_cols;    // ncols rounded up to a power of two >= 32
  int kblocks;      // ceil(K / 128)
  int kper;         // K blocks per split
  int splits;       // cluster size along K
  int per;          // activation rows each CTA of a cluster finishes
  int stages;
  int stage_bytes;  // TC_W_BYTES + ncols*128
  int ring_bytes;   // stages*stage_bytes
  int inbox_bytes;  // splits > 1: partials received, [splits][planes][per][128] int32
  int tma_out;      // 1: the single output (Y, or acc_out) leaves by one TMA tensor store per CTA
  uint32_t* err;
  float scale_all;  // the scale of every channel when `scale` is null
  int relu;         // Y <- max(Y, 0)
};

// ReLU of the exported-network layers (dgx_dense_q); identity otherwise.
__device__ __forceinline__ float w8_act(const W8TcArgs& a, float y) { return a.relu ? fmaxf(y, 0.f) : y; }

__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::
          : "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_map(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_s32(uint32_t addr, int v) {
  asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void mma_i8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Instruction descriptor, kind::i8: D s32 (2), A and B signed 8-bit (1), both K-major.
__host__ __device__ constexpr uint32_t idesc_i8(uint32_t M, uint32_t N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

// Final value of one output from its per-plane int32 sums (rs: the row scale).
__device__ __forceinline__ void w8_store(const W8TcArgs& a, int b, int n, float sc, float bi, float rs, int a0,
                                         int a1, int a2) {
  const size_t o = (size_t)b * a.N + n;
  if (a.planes == 1) {
    if (a.acc_out) a.acc_out[o] = a0;
    if (a.Y) a.Y[o] = w8_act(a, fmaf(sc * rs, (float)a0, bi));
  } else {
    // exact A0*2^14 + A1*2^7 + A2, rounded once
    const long long t = ((long long)a0 << 14) + ((long long)a1 << 7) + (long long)a2;
    a.Y[o] = w8_act(a, fmaf(sc, __ll2float_rn(t) * (0x1p-14f * rs), bi));
  }
}

__global__ void __launch_bounds__(TC_THREADS, 1)
    w8_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                 const __grid_constant__ CUtensorMap tmOut, W8TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + a.ring_bytes);  // tail: barriers, row scales, inbox
  uint64_t* empty_bar = full_bar + S;
  uint64_t* done_bar = empty_bar + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* rs_s = reinterpret_cast<float*>(smem + a.ring_bytes + 256);  // this chunk's row scales
  int32_t* inbox = reinterpret_cast<int32_t*>(smem + a.ring_bytes + 256 + 1024);

  // Small batches (split K over clusters, a few microseconds per layer): the
  // next layer's activation pre-pass, a programmatic dependent that waits for
  // this grid before it reads anything, may be scheduled now, so its launch
  // and its own dependent's weight stream overlap this layer's tail. Larger
  // batches let it start only at exit: there the next layer's weight stream
  // competing with this one's costs more than the overlap gains.
  if (a.splits > 1) grid_dep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x;
  const int m0 = blockIdx.y * TC_BM;
  const int b0 = blockIdx.z * a.bc;
  const int kb0 = split * a.kper;
  const int nk = min(a.kblocks, kb0 + a.kper) - kb0;  // >= 1 by construction on the host
  // The CTAs of different output tiles read the same activation tiles; each
  // starts its K range at a different block so they do not all ask the same
  // L2 lines at once (the int32 sums do not depend on the order).
  const int krot = (int)((blockIdx.y * 5u) % (unsigned)nk);
  WaitCtx wc{abort_flag, a.err};

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, a.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one_lane()) {
      tma_prefetch_desc(&tmW);
      tma_prefetch_desc(&tmX);
      const uint32_t xbytes = (uint32_t)a.ncols * TC_BK;
      const int pro = min(S, nk);
      // The weights do not depend on the kernel that produces the activation
      // planes: start streaming them before waiting for it.
      auto kx = [&](int i) { return (kb0 + (i + krot) % nk) * TC_BK; };
      for (int i = 0; i < pro; ++i) {
        mbar_arrive_expect_tx(&full_bar[i], TC_W_BYTES + xbytes);
        tma_load_2d(smem + i * a.stage_bytes, &tmW, &full_bar[i], kx(i), m0);
      }
      grid_dep_wait();
      for (int i = 0; i < pro; ++i)
        tma_load_3d(smem + i * a.stage_bytes + TC_W_BYTES, &tmX, &full_bar[i], kx(i), b0, 0);
      int filled = pro;
      for (int i = pro; i < nk; ++i, ++filled) {
        const int s = i % S;
        if (!mbar_wait(&empty_bar[s], ((i / S) & 1) ^ 1, wc)) break;
        uint8_t* st = smem + s * a.stage_bytes;
        mbar_arrive_expect_tx(&full_bar[s], TC_W_BYTES + xbytes);
        tma_load_2d(st, &tmW, &full_bar[s], kx(i), m0);
        tma_load_3d(st + TC_W_BYTES, &tmX, &full_bar[s], kx(i), b0, 0);
      }
      // Teardown: every stage filled must have landed before the CTA leaves.
      for (int f = max(0, filled - S); f < filled; ++f) mbar_drain(&full_bar[f % S], (f / S) & 1);
    }
    __syncwarp();
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one_lane()) {
      const uint32_t idesc = idesc_i8(TC_BM, (uint32_t)a.ncols);
      bool ok = true;
      for (int i = 0; i < nk; ++i) {
        const int s = i % S;
        if (!mbar_wait(&full_bar[s], (i / S) & 1, wc)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + s * a.stage_bytes);
        const uint32_t sb = sa + TC_W_BYTES;
#pragma unroll
        for (int kk = 0; kk < TC_BK / 32; ++kk)
          mma_i8_ss(tmem_base, sw128_desc(sa + kk * 32, 16, 1024), sw128_desc(sb + kk * 32, 16, 1024), idesc,
                    (i > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&empty_bar[s]);
      }
      if (ok) tc_commit(done_bar);
    }
    __syncwarp();
  }

  // ------------------------------------------------------------ epilogue (warps 0-3)
  // TMEM lane quarter q holds output channels m0 + 32q .. m0 + 32q + 31.
  const int row = warp * 32 + lane;
  const int n = m0 + row;
  const int nb = min(a.bc, a.B - b0);  // valid activation rows of this chunk
  bool have = false;
  float sc = 0.f, bi = 0.f;
  if (warp < 4) {
    // Everything the stores need is fetched while the MMAs run.
    grid_dep_wait();  // the row scales come from the producer kernel
    if (n < a.N && a.Y) {
      sc = a.scale ? a.scale[n] : a.scale_all;
      bi = a.bias ? a.bias[n] : 0.f;
    }
    for (int b = threadIdx.x; b < nb; b += 128) rs_s[b] = a.rowscale ? a.rowscale[b0 + b] : 0.f;
    named_bar_sync(1, 128);
    have = mbar_wait(done_bar, 0, wc);
    tc_fence_after();
    const uint32_t taddr = tmem_base + ((uint32_t)(warp * 32) << 16);
    if (have && a.splits == 1 && a.tma_out) {
      // The tile [bc rows][128 channels] is assembled in the free stage ring
      // (each lane writes one channel: conflict-free) and leaves by one TMA
      // store, which also clips rows past B and channels past N.
      float* tile = reinterpret_cast<float*>(smem) + row;
      if (a.planes == 1) {
        const bool acc_only = a.acc_out != nullptr;
        for (int c = 0; c < nb; c += 32) {
          uint32_t v[32];
          tmem_ld32(taddr + c, v);
          tmem_ld_wait();
          if (acc_only) {
#pragma unroll
            for (int j = 0; j < 32; ++j) tile[(c + j) * TC_BM] = __int_as_float((int)v[j]);
          } else {
            // Row scales to registers first: `tile` and `rs_s` are both in
            // shared memory, so a load after a store could not move ahead of it.
            float f[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) f[j] = sc * rs_s[c + j];
#pragma unroll
            for (int j = 0; j < 32; ++j) tile[(c + j) * TC_BM] = w8_act(a, fmaf(f[j], (float)(int)v[j], bi));
          }
        }
      } else {
        for (int c = 0; c < nb; c += 16) {
          uint32_t v0[16], v1[16], v2[16];
          tmem_ld16(taddr + c, v0);
          tmem_ld16(taddr + a.bc + c, v1);
          tmem_ld16(taddr + 2 * a.bc + c, v2);
          tmem_ld_wait();
          float f[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) f[j] = 0x1p-14f * rs_s[c + j];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            // exact A0*2^14 + A1*2^7 + A2, rounded once
            const long long t = ((long long)(int)v0[j] << 14) + ((long long)(int)v1[j] << 7) + (int)v2[j];
            tile[(c + j) * TC_BM] = w8_act(a, fmaf(sc, __ll2float_rn(t) * f[j], bi));
          }
        }
      }
      fence_proxy_async_smem();
      named_bar_sync(1, 128);
      if (threadIdx.x == 0) {
        tma_store_2d(&tmOut, tile, m0, b0);
        bulk_commit();
        bulk_wait0();
      }
    } else if (have && a.splits == 1) {
      // Output row b of this chunk for channel n sits at Y[(b0 + b)*N + n]:
      // for each b the warp's 32 lanes write 128 contiguous bytes.
      const size_t ld = (size_t)a.N;
      float* yp = a.Y ? a.Y + (size_t)b0 * ld + n : nullptr;
      int32_t* ap = a.acc_out ? a.acc_out + (size_t)b0 * ld + n : nullptr;
      const bool live = n < a.N;
      for (int c = 0; c < nb; c += 16) {
        uint32_t v0[16], v1[16], v2[16];
        tmem_ld16(taddr + c, v0);
        if (a.planes == 3) {
          tmem_ld16(taddr + a.bc + c, v1);
          tmem_ld16(taddr + 2 * a.bc + c, v2);
        }
        tmem_ld_wait();
        float rsv[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) rsv[j] = rs_s[c + j];
        if (live) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (c + j < nb) {
              const size_t o = (size_t)(c + j) * ld;
              if (a.planes == 1) {
                if (ap) ap[o] = (int)v0[j];
                if (yp) yp[o] = w8_act(a, fmaf(sc * rsv[j], (float)(int)v0[j], bi));
              } else {
                const long long t = ((long long)(int)v0[j] << 14) + ((long long)(int)v1[j] << 7) + (int)v2[j];
                yp[o] = w8_act(a, fmaf(sc, __ll2float_rn(t) * (0x1p-14f * rsv[j]), bi));
              }
            }
          }
        }
      }
    } else if (have) {
      // Partial sums to the inboxes of the CTAs that finish their rows:
      // column c = p*bc + b goes to CTA b/per, slot [my rank][p][b%per].
      const int me = (int)cluster_rank();
      const uint32_t inbox_row = smem_u32(inbox) + (uint32_t)row * 4;
      for (int p = 0; p < a.planes; ++p) {
        // slot of activation row b in CTA dst's inbox: [me][p][b - dst*per]
        int dst = 0, bl = 0;
        uint32_t slot = inbox_row + (uint32_t)((me * a.planes + p) * a.per * TC_BM * 4);
        uint32_t remote = cluster_map(slot, 0);
        for (int c = 0; c < nb; c += 16) {
          uint32_t v[16];
          tmem_ld16(taddr + p * a.bc + c, v);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (c + j < nb) {
              st_cluster_s32(remote + (uint32_t)(bl * TC_BM * 4), (int)v[j]);
              if (++bl == a.per) {
                bl = 0;
                ++dst;
                remote = cluster_map(slot, (uint32_t)min(dst, a.splits - 1));
              }
            }
          }
        }
      }
    }
  }
  if (a.splits > 1) {
    cluster_sync_all();  // every partial has landed in its inbox
    if (warp < 4 && n < a.N) {
      const int me = (int)cluster_rank();
      const int bs = me * a.per, be = min(nb, bs + a.per);
      for (int b = bs; b < be; ++b) {
        int acc[3] = {0, 0, 0};
        for (int p = 0; p < a.planes; ++p)
          for (int r = 0; r < a.splits; ++r) acc[p] += inbox[((r * a.planes + p) * a.per + (b - bs)) * TC_BM + row];
        w8_store(a, b0 + b, n, sc, bi, rs_s[b], acc[0], acc[1], acc[2]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem_base, a.tmem_cols);
  }
}

// The power-of-two scale of a row with largest magnitude m: s = m/127
// rounded; frexp gives s = f*2^e, f in [0.5,1), so 2^e > m/127 (2^e is
// representable and rounding is monotone) and 2^e <= 2s.
__device__ __forceinline__ int plane_exponent(float m) {
  int e = 0;
  if (m > 0.f) {
    frexpf(m / 127.f, &e);
    e = max(e, -126);  // keep 2^-e finite for rows of tiny magnitude
  }
  return e;
}

// Splits four values (already scaled by 2^-e) into the three int8 planes and
// stores them. Every step is exact in fp32: scaling by a power of two,
// subtracting the nearest integer, scaling by 2^7.
__device__ __forceinline__ void split_store4(float4 v, float inv, int8_t* dst, size_t plane) {
  const float t[4] = {v.x, v.y, v.z, v.w};
  int8_t q0[4], q1[4], q2[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const float s0 = t[u] * inv;
    const float r0 = rintf(s0);
    const float s1 = (s0 - r0) * 128.f;
    const float r1 = rintf(s1);
    const float r2 = rintf((s1 - r1) * 128.f);
    q0[u] = (int8_t)(int)r0;
    q1[u] = (int8_t)(int)r1;
    q2[u] = (int8_t)(int)r2;
  }
  *reinterpret_cast<char4*>(dst) = make_char4(q0[0], q0[1], q0[2], q0[3]);
  *reinterpret_cast<char4*>(dst + plane) = make_char4(q1[0], q1[1], q1[2], q1[3]);
  *reinterpret_cast<char4*>(dst + 2 * plane) = make_char4(q2[0], q2[1], q2[2], q2[3]);
}

__device__ __forceinline__ float block_max256(float m, float* red) {
#pragma unroll
  for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  m = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w]);
  return m;
}

// One CTA of 256 threads per row, the row held in registers (K <= 1024*NV):
// row max, the power-of-two scale 2^e with max|x|/2^e in (63.5, 127], and
// the three int8 planes.
template <int NV>
__global__ void __launch_bounds__(256) split_planes_kernel(const float* __restrict__ X, int8_t* __restrict__ Xp,
                                                           float* __restrict__ rowscale, int B, int K) {
  grid_dep_launch();  // the GEMM may start streaming weights now
  grid_dep_wait();    // X may come from the kernel before (launched as its dependent)
  __shared__ float red[8];
  const int b = blockIdx.x;
  const float* x = X + (size_t)b * K;
  float4 v[NV];
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int k = (threadIdx.x + 256 * j) * 4;
    v[j] = k < K ? __ldg(reinterpret_cast<const float4*>(x + k)) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int j = 0; j < NV; ++j)
    m = fmaxf(m, fmaxf(fmaxf(fabsf(v[j].x), fabsf(v[j].y)), fmaxf(fabsf(v[j].z), fabsf(v[j].w))));
  m = block_max256(m, red);
  const int e = plane_exponent(m);
  const float inv = ldexpf(1.f, -e);
  if (threadIdx.x == 0) rowscale[b] = ldexpf(1.f, e);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int k = (threadIdx.x + 256 * j) * 4;
    if (k < K) split_store4(v[j], inv, Xp + (size_t)b * K + k, (size_t)B * K);
  }
}

// The same split for any K (% 4 == 0): two passes over the row.
__global__ void __launch_bounds__(256) split_planes_loop_kernel(const float* __restrict__ X, int8_t* __restrict__ Xp,
                                                                float* __restrict__ rowscale, int B, int K) {
  grid_dep_launch();
  grid_dep_wait();
  __shared__ float red[8];
  const int b = blockIdx.x;
  const float* x = X + (size_t)b * K;
  float m = 0.f;
  for (int k = threadIdx.x * 4; k < K; k += 1024) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(x + k));
    m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  m = block_max256(m, red);
  const int e = plane_exponent(m);
  const float inv = ldexpf(1.f, -e);
  if (threadIdx.x == 0) rowscale[b] = ldexpf(1.f, e);
  for (int k = threadIdx.x * 4; k < K; k += 1024)
    split_store4(__ldg(reinterpret_cast<const float4*>(x + k)), inv, Xp + (size_t)b * K + k, (size_t)B * K);
}

bool encode_map(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
                const cuuint32_t* box) {
  auto enc = get_tensor_map_encoder();
  if (!enc) return false;
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, (cuuint32_t)rank, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int round16(int x) { return (x + 15) & ~15; }

}  // namespace

cudaError_t w8_tc_gemm(const int8_t* Xp, int planes, const int8_t* W, const float* scale, const float* bias,
                       const float* rowscale, float* Y, int32_t* acc_out, int B, int N, int K, bool after_producer,
                       cudaStream_t s, const W8Epi& epi) {
  W8TcArgs a{};
  a.scale = scale;
  a.scale_all = epi.scale_all;
  a.relu = epi.relu;
  a.bias = bias;
  a.rowscale = rowscale;
  a.Y = Y;
  a.acc_out = acc_out;
  a.B = B;
  a.N = N;
  a.K = K;
  a.planes = planes;
  // Activation rows per chunk (the MMA takes at most 256 columns): as few
  // chunks as give enough (output tile, chunk) CTAs to fill the GPU; when
  // even the smallest chunks leave it idle, one chunk and split K instead.
  const int mtiles = (N + TC_BM - 1) / TC_BM;
  const int max_bc = planes == 1 ? 256 : 80;
  const int min_chunks = (B + max_bc - 1) / max_bc;
  const int want_ctas = num_sms() * 2 / 3;
  int chunks = min_chunks;
  while (mtiles * chunks < want_ctas && (B + chunks) / (chunks + 1) >= 64) ++chunks;
  a.bc = round16((B + chunks - 1) / chunks);
  chunks = (B + a.bc - 1) / a.bc;
  a.ncols = planes * a.bc;
  a.tmem_cols = 32;
  while (a.tmem_cols < a.ncols) a.tmem_cols *= 2;
  a.kblocks = (K + TC_BK - 1) / TC_BK;
  int splits = 1;
  if (mtiles * chunks < want_ctas)
    splits = std::max(1, std::min(num_sms() / std::max(1, mtiles * chunks), std::min(8, a.kblocks)));
  a.kper = (a.kblocks + splits - 1) / splits;
  a.splits = (a.kblocks + a.kper - 1) / a.kper;
  a.per = (std::min(a.bc, B) + a.splits - 1) / a.splits;
  a.inbox_bytes = a.splits > 1 ? a.splits * planes * a.per * TC_BM * 4 : 0;
  a.stage_bytes = TC_W_BYTES + a.ncols * TC_BK;
  const int tail = 256 + 1024 + a.inbox_bytes;  // barriers, row scales, inbox
  a.stages = std::min(TC_MAX_STAGES, std::min(a.kper, (TC_SMEM_BUDGET - tail) / a.stage_bytes));
  if (a.stages < 1) return cudaErrorInvalidConfiguration;
  a.ring_bytes = a.stages * a.stage_bytes;
  a.err = device_error_word();
  // At least 116 KiB so one CTA holds an SM: a second CTA of the same
  // cluster on that SM could otherwise wait for TMEM that the first only
  // frees after the cluster barrier.
  const int smem = std::max(1024 + a.ring_bytes + tail, 116 * 1024);

  CUtensorMap mw{}, mx{}, mo{};
  {
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
    const cuuint64_t strides[1] = {(cuuint64_t)K};
    const cuuint32_t box[2] = {TC_BK, TC_BM};
    if (!encode_map(&mw, W, 2, dims, strides, box)) return cudaErrorInvalidValue;
  }
  {
    const cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)B, (cuuint64_t)planes};
    const cuuint64_t strides[2] = {(cuuint64_t)K, (cuuint64_t)B * (cuuint64_t)K};
    const cuuint32_t box[3] = {TC_BK, (cuuint32_t)a.bc, (cuuint32_t)planes};
    if (!encode_map(&mx, Xp, 3, dims, strides, box)) return cudaErrorInvalidValue;
  }
  // One output, rows of N 4-byte values 16-byte aligned: a TMA store per CTA.
  void* out = Y ? (void*)Y : (void*)acc_out;
  a.tma_out = a.splits == 1 && ((Y == nullptr) != (acc_out == nullptr)) && N % 4 == 0 &&
              ((uintptr_t)out & 15) == 0 && a.ring_bytes >= ((a.bc + 31) & ~31) * TC_BM * 4;
  if (a.tma_out) {
    auto enc = get_tensor_map_encoder();
    const cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)B};
    const cuuint64_t strides[1] = {(cuuint64_t)N * 4};
    const cuuint32_t box[2] = {TC_BM, (cuuint32_t)a.bc};
    const cuuint32_t estr[2] = {1, 1};
    if (!enc || enc(&mo, Y ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_INT32, 2, out, dims, strides,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  } else {
    mo = mw;  // unused
  }

  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e =
        cudaFuncSetAttribute(w8_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 1024 + TC_SMEM_BUDGET);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(a.splits, mtiles, chunks);
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  attrs[na].id = cudaLaunchAttributeClusterDimension;
  attrs[na].val.clusterDim.x = a.splits;
  attrs[na].val.clusterDim.y = 1;
  attrs[na].val.clusterDim.z = 1;
  ++na;
  if (after_producer) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  TimerScope timer(s);
  return cudaLaunchKernelEx(&cfg, w8_tc_kernel, mw, mx, mo, a);
}

cudaError_t w8_split_planes(const float* X, int8_t* Xp, float* rowscale, int B, int K, cudaStream_t s) {
  if (K <= 1024) return launch_dependent(split_planes_kernel<1>, B, 256, s, X, Xp, rowscale, B, K);
  if (K <= 2048) return launch_dependent(split_planes_kernel<2>, B, 256, s, X, Xp, rowscale, B, K);
  if (K <= 4096) return launch_dependent(split_planes_kernel<4>, B, 256, s, X, Xp, rowscale, B, K);
  if (K <= 8192) return launch_dependent(split_planes_kernel<8>, B, 256, s, X, Xp, rowscale, B, K);
  return launch_dependent(split_planes_loop_kernel, B, 256, s, X, Xp, rowscale, B, K);
}

}  // namespace dgx
