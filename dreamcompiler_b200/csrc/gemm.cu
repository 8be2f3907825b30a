// Dense GEMM for the Dream `@` operator and its autograd GEMMs on sm_100a.
//
//   C[M,N] = op(A)[M,K] . op(B)[K,N]  (+ beta*C) (+ bias[N]) (ReLU)
//
// Replaces the reference's CPU/OpenCL/cuBLAS dispatch in `tensor_matmul`
// (runtime/ops/elementwise.inc:971-1213), the "matmul" backward GEMMs
// dA = dY.B^T and dB = A^T.dY (runtime/ops/autograd.inc:91-125) and the fused
// `dream_linear` Y = X.W^T + b (+ReLU) (runtime/ops/elementwise.inc:1432-1521).
//
// Design: one persistent CTA per SM. Warp 0 issues TMA tile loads into a
// ring of shared-memory stages; warp 1 issues tcgen05.mma into one of two TMEM
// accumulators; warps 2-9 (two per TMEM lane quarter) drain the other
// accumulator (tcgen05.ld), apply the epilogue and store, so the epilogue of
// tile i overlaps the main loop of tile i+1. Transposed operands are handled by the shared-memory descriptor's
// major-ness (K-major or MN-major), never by a copy.
//
// bf16 inputs run kind::f16 with fp32 accumulation. f32 inputs run the
// 3xTF32 split (a = a_hi + a_lo, C = A_hi.B_hi + A_hi.B_lo + A_lo.B_hi) on
// kind::tf32, which keeps the error near fp32 level (<= 1e-4 normwise); the
// hi/lo planes are produced by `split_tf32_kernel` into caller-visible scratch.
#include <algorithm>

#include "sm100.cuh"
#include "gemm.h"

namespace dgx {

// ---------------------------------------------------------------------------
// Tile configuration
// ---------------------------------------------------------------------------
// BN_: the default output tile width (256 bf16 / 128 tf32), or half of it for
// problems whose default tiles would leave SMs idle.
template <bool TF32, int BN_ = (TF32 ? 128 : 256)>
struct GemmCfg {
  static constexpr int BM = 128;
  static constexpr int BN = BN_;
  static constexpr int ESZ = TF32 ? 4 : 2;                 // bytes per element
  static constexpr int BK = 128 / ESZ;                       // one 128-byte swizzle row of K
  static constexpr int MMA_K = 32 / ESZ;                     // K per tcgen05.mma (32 bytes)
  static constexpr int A_BYTES = BM * BK * ESZ;              // 16 KB
  static constexpr int B_BYTES = BN * BK * ESZ;              // 32 KB (bf16) / 16 KB (tf32)
  static constexpr int PLANES = TF32 ? 2 : 1;                // hi (+ lo) planes per operand
  static constexpr int STAGE_BYTES = PLANES * (A_BYTES + B_BYTES);
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES > 8 ? 8 : (192 * 1024) / STAGE_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;                   // double-buffered accumulator
  static constexpr int CHUNK = 128 / ESZ;                    // MN elements per 128-byte chunk
  // Epilogue staging for the TMA-store path: 8 warps x (32 rows x 128 B).
  static constexpr int OUT_STAGE_BYTES = 8 * 4096;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + OUT_STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static constexpr uint32_t FMT = TF32 ? 2u : 1u;
};

struct TileSched {
  int tiles_m, tiles_n, group_m;
  __device__ __forceinline__ void coords(int t, int& tm, int& tn) const {
    const int per_group = group_m * tiles_n;
    const int g = t / per_group;
    const int first_m = g * group_m;
    const int gsize = min(tiles_m - first_m, group_m);
    const int r = t - g * per_group;
    tm = first_m + r % gsize;
    tn = r / gsize;
  }
};

// Shared-memory offset of the K-major or MN-major operand tile for MMA step kk
// (each step consumes 32 bytes of K).
template <bool MN, int ESZ>
__device__ __forceinline__ uint32_t kstep_offset(int kk) {
  // K-major: advance 32 bytes inside the 128-byte swizzled row.
  // MN-major: advance (32/ESZ) K rows of 128 bytes each.
  return MN ? (uint32_t)kk * (32 / ESZ) * 128 : (uint32_t)kk * 32;
}

// EXTRA: the TMA-store epilogue also stores every staged box to the extra
// destinations (tmX); plain instantiations carry none of that code.
// Warps: 0 TMA producer, 1 MMA issuer, 2..9 epilogue (two per TMEM lane
// quarter, taking alternate column chunks of the accumulator).
constexpr int kGemmThreads = 320;

template <bool TF32, bool A_MN, bool B_MN, int BN_, bool EXTRA = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2,
                   const __grid_constant__ CUtensorMap tmC, const __grid_constant__ ExtraOutMaps tmX,
                   GemmArgs args) {
  using Cfg = GemmCfg<TF32, BN_>;
  constexpr int BM = Cfg::BM, BN = Cfg::BN, BK = Cfg::BK, STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* out_stage = smem + STAGES * Cfg::STAGE_BYTES;  // 1024-aligned
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(out_stage + Cfg::OUT_STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* accf_bar = empty_bar + STAGES;  // [2]
  uint64_t* acce_bar = accf_bar + 2;        // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  WaitCtx wc{abort_flag, args.err};

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf_bar[b], 1);
      mbar_init(&acce_bar[b], 8);  // every epilogue warp releases the accumulator
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (TF32) {
      tma_prefetch_desc(&tmA2);
      tma_prefetch_desc(&tmB2);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const TileSched sched{args.tiles_m, args.tiles_n, args.group_m};
  // Work units: (batch, output tile, K slice); unit u -> batch u / per_batch,
  // tile (u % per_batch) / splits, slice u % splits.
  const int splits = args.splits;
  const int per_batch = args.tiles_m * args.tiles_n * splits;
  const int num_tiles = per_batch * (args.batch > 1 ? args.batch : 1);
  const int nk_all = (args.K + BK - 1) / BK;
  const int kper = (nk_all + splits - 1) / splits;
  auto kslice = [&](int u, int& kb0, int& kb1) {
    kb0 = (u % splits) * kper;
    kb1 = min(nk_all, kb0 + kper);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one_lane()) {
      uint32_t fill = 0;
      for (int t = blockIdx.x; t < num_tiles && !*abort_flag; t += gridDim.x) {
        int tm, tn, kb0, kb1;
        const int bz = t / per_batch;
        sched.coords((t - bz * per_batch) / splits, tm, tn);
        kslice(t, kb0, kb1);
        const int m0 = tm * BM, n0 = tn * BN;
        for (int kb = kb0; kb < kb1; ++kb, ++fill) {
          const int s = fill % STAGES;
          const uint32_t round = fill / STAGES;
          if (!mbar_wait(&empty_bar[s], (round & 1) ^ 1, wc)) break;
          uint8_t* sa = smem + s * Cfg::STAGE_BYTES;
          uint8_t* sb = sa + Cfg::PLANES * Cfg::A_BYTES;
          mbar_arrive_expect_tx(&full_bar[s], Cfg::STAGE_BYTES);
          const int k0 = kb * BK;
#pragma unroll
          for (int p = 0; p < Cfg::PLANES; ++p) {
            const CUtensorMap* ma = p == 0 ? &tmA : &tmA2;
            const CUtensorMap* mb = p == 0 ? &tmB : &tmB2;
            uint8_t* pa = sa + p * Cfg::A_BYTES;
            uint8_t* pb = sb + p * Cfg::B_BYTES;
            if (A_MN) {
#pragma unroll
              for (int c = 0; c < BM / Cfg::CHUNK; ++c)
                tma_load_3d(pa + c * BK * 128, ma, &full_bar[s], m0 + c * Cfg::CHUNK, k0, bz);
            } else {
              tma_load_3d(pa, ma, &full_bar[s], k0, m0, bz);
            }
            if (B_MN) {
#pragma unroll
              for (int c = 0; c < BN / Cfg::CHUNK; ++c)
                tma_load_3d(pb + c * BK * 128, mb, &full_bar[s], n0 + c * Cfg::CHUNK, k0, bz);
            } else {
              tma_load_3d(pb, mb, &full_bar[s], k0, n0, bz);
            }
          }
        }
        if (*abort_flag) break;
      }
      // Teardown: every stage we filled must have landed before we leave.
      const uint32_t first = fill > (uint32_t)STAGES ? fill - STAGES : 0;
      for (uint32_t f = first; f < fill; ++f) mbar_drain(&full_bar[f % STAGES], (f / STAGES) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = make_idesc(Cfg::FMT, A_MN ? 1u : 0u, B_MN ? 1u : 0u, BM, BN);
    const uint32_t a_lbo = A_MN ? BK * 128 : 16, b_lbo = B_MN ? BK * 128 : 16;
    if (elect_one_lane()) {
      uint32_t fill = 0, use = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++use) {
        const int buf = use & 1;
        if (!mbar_wait(&acce_bar[buf], ((use >> 1) & 1) ^ 1, wc)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        bool ok = true;
        int kb0, kb1;
        kslice(t, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb, ++fill) {
          const int s = fill % STAGES;
          if (!mbar_wait(&full_bar[s], (fill / STAGES) & 1, wc)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * Cfg::STAGE_BYTES);
          const uint32_t sb = sa + Cfg::PLANES * Cfg::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / Cfg::MMA_K; ++kk) {
            const uint32_t ao = kstep_offset<A_MN, Cfg::ESZ>(kk), bo = kstep_offset<B_MN, Cfg::ESZ>(kk);
            const uint64_t adesc = sw128_desc(sa + ao, a_lbo, 1024);
            const uint64_t bdesc = sw128_desc(sb + bo, b_lbo, 1024);
            const uint32_t acc = (kb > kb0 || kk > 0) ? 1u : 0u;
            if (TF32) {
              const uint64_t adesc_lo = sw128_desc(sa + Cfg::A_BYTES + ao, a_lbo, 1024);
              const uint64_t bdesc_lo = sw128_desc(sb + Cfg::B_BYTES + bo, b_lbo, 1024);
              // small terms first, then the dominant hi.hi product
              mma_tf32_ss(d_tmem, adesc_lo, bdesc, idesc, acc);
              mma_tf32_ss(d_tmem, adesc, bdesc_lo, idesc, 1u);
              mma_tf32_ss(d_tmem, adesc, bdesc, idesc, 1u);
            } else {
              mma_f16_ss(d_tmem, adesc, bdesc, idesc, acc);
            }
          }
          tc_commit(&empty_bar[s]);  // stage is free once these MMAs have read it
        }
        if (!ok) break;
        tc_commit(&accf_bar[buf]);  // accumulator ready for the epilogue
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..9)
    // Two warps per TMEM lane quarter: `half` 0 takes the even column chunks
    // of the accumulator, 1 the odd ones, so the drain, the epilogue math
    // and the stores of one tile run on 8 warps (at small K the epilogue,
    // not the main loop, sets the tile period).
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;
    const int row_in_tile = q * 32 + lane;
    uint32_t use = 0;
    // TMA-store path: each warp stages its 32 rows x 128 bytes (32 fp32 or 64
    // bf16 columns) in its shared-memory buffer with the 128-byte swizzle
    // (16-byte unit u of row r at u ^ (r & 7): conflict-free) and issues one
    // TMA store / reduce-add per chunk.
    uint8_t* my_stage = out_stage + (warp - 2) * 4096;
    uint32_t issued = 0;  // stores issued by this warp
    if (args.tma_out && lane == 0) {
      tma_prefetch_desc(&tmC);
      if (EXTRA)
        for (int e = 0; e < args.n_extra; ++e) tma_prefetch_desc(&tmX.m[e]);
    }
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++use) {
      const int buf = use & 1;
      int tm, tn;
      const int bz = t / per_batch;
      sched.coords((t - bz * per_batch) / splits, tm, tn);
      if (args.tma_out && args.tma_out != 3) prefetch_bias_l1(args.bias, tn * BN, BN, args.N, lane);
      if (!mbar_wait(&accf_bar[buf], (use >> 1) & 1, wc)) break;
      tc_fence_after();
      const int m = tm * BM + row_in_tile;
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + buf * BN;
      if (args.tma_out) {
        constexpr int CW32 = 32;  // fp32 columns per 32-column TMEM load
        const int cw = (args.c_bf16 && args.tma_out != 3) ? 64 : 32;  // columns per 128-byte staged row
        if (half * cw >= BN) {  // no chunk for this warp (one-chunk tiles): release at once
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acce_bar[buf]);
        }
#pragma unroll 1
        for (int c = half * cw; c < BN; c += 2 * cw) {
          uint32_t r[64];
          tmem_ld32(taddr + c, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
          if (cw == 64) tmem_ld32(taddr + c + CW32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
          float bq[64];  // this chunk's bias: the loads overlap the TMEM load
          if (args.bias && args.tma_out != 3) {
#pragma unroll
            for (int j8 = 0; j8 < 64; j8 += 8)
              if (j8 < cw) {
                float b8[8];
                load_bias8(args.bias, tn * BN + c + j8, args.N, b8);
#pragma unroll
                for (int i = 0; i < 8; ++i) bq[j8 + i] = b8[i];
              }
          }
          tmem_ld_wait();
          if (c + 2 * cw >= BN) {  // this warp's last loads of the accumulator: release it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce_bar[buf]);
          }
          const int n0 = tn * BN + c;
          if (n0 >= args.N) continue;
          uint8_t* st = my_stage;
          if (lane == 0 && issued >= 1) bulk_wait_read0();  // the previous store has read the buffer
          __syncwarp();
          uint32_t w[32];
          if (args.tma_out == 3) {  // raw partial sums
#pragma unroll
            for (int j = 0; j < 32; ++j) w[j] = r[j];
          } else if (args.c_bf16) {
#pragma unroll
            for (int j8 = 0; j8 < 64; j8 += 8) {
#pragma unroll
              for (int i = 0; i < 8; i += 2) {
                float v0 = __uint_as_float(r[j8 + i]), v1 = __uint_as_float(r[j8 + i + 1]);
                if (args.bias) {
                  v0 += bq[j8 + i];
                  v1 += bq[j8 + i + 1];
                }
                if (args.relu) {
                  v0 = fmaxf(v0, 0.f);
                  v1 = fmaxf(v1, 0.f);
                }
                w[(j8 + i) / 2] = pack_bf16x2(v0, v1);
              }
            }
          } else {
#pragma unroll
            for (int j8 = 0; j8 < 32; j8 += 8) {
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                float v = __uint_as_float(r[j8 + i]);
                if (args.bias) v += bq[j8 + i];
                if (args.relu) v = fmaxf(v, 0.f);
                w[j8 + i] = __float_as_uint(v);
              }
            }
          }
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<uint4*>(st + lane * 128 + ((u ^ (lane & 7)) << 4)) =
                make_uint4(w[4 * u], w[4 * u + 1], w[4 * u + 2], w[4 * u + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            // z: the K slice for split-K partials (unbatched), else the batch.
            if (args.tma_out == 3)
              tma_store_3d(&tmC, st, n0, tm * BM + q * 32, t % splits);
            else if (args.tma_out == 2)
              tma_reduce_add_3d(&tmC, st, n0, tm * BM + q * 32, bz);
            else {
              tma_store_3d(&tmC, st, n0, tm * BM + q * 32, bz);
              if (EXTRA)
                for (int e = 0; e < args.n_extra; ++e) tma_store_3d(&tmX.m[e], st, n0, tm * BM + q * 32, bz);
            }
            bulk_commit();  // one group per staged buffer, all its destinations
          }
          ++issued;
        }
        (void)m;
      } else {
#pragma unroll 1
        for (int c = half * 32; c < BN; c += 64) {
          uint32_t r[32];
          tmem_ld32(taddr + c, r);
          tmem_ld_wait();
          const int n0 = tn * BN + c;
          if (m < args.M && n0 < args.N)
            gemm_store_row32(args, m, n0, reinterpret_cast<float*>(r), (long long)bz * args.sC);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acce_bar[buf]);
      }
    }
    if (args.tma_out && lane == 0) bulk_wait0();  // staged tiles read and stored before the CTA leaves
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// 3xTF32 operand split: hi = x with the low 13 mantissa bits cleared (exactly
// representable in tf32), lo = x - hi (exact in fp32). The planes are always
// written K-major ([rows][kpad], kpad = K rounded up to 4 with zero fill), so
// the tf32 MMA only ever reads K-major tiles: 32-bit MN-major operands would
// need the 32-byte-atom swizzle, which the plain 128B TMA swizzle does not
// produce. `src_t` = the source is stored [K][rows] (transposed); a 32x32
// shared-memory tile keeps both the read and the write coalesced.
// ---------------------------------------------------------------------------
struct SplitJob {
  const float* x;
  int rows, ld, src_t;
  float* hi;
  float* lo;
  long long sx;  // source batch stride (elements); the planes of batch b start at b * rows * kpad
};
// blockIdx.z = 2 * batch + operand: both operands of every batch are split by
// one launch.
__global__ void split_tf32_kernel(SplitJob ja, SplitJob jb, int K, int kpad) {
  __shared__ float tile[32][33];
  const SplitJob& j = (blockIdx.z & 1) == 0 ? ja : jb;
  const long long bz = blockIdx.z >> 1;
  const float* __restrict__ x = j.x + bz * j.sx;
  float* __restrict__ hi = j.hi + bz * (long long)j.rows * kpad;
  float* __restrict__ lo = j.lo + bz * (long long)j.rows * kpad;
  const int rows = j.rows, ld = j.ld, src_t = j.src_t;
  const int r0 = blockIdx.y * 32, k0 = blockIdx.x * 32;
  if (r0 >= rows) return;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
  for (int i = ty; i < 32; i += 8) {
    float v = 0.f;
    if (src_t) {  // coalesced along rows: x[k*ld + r]
      const int k = k0 + i, r = r0 + tx;
      if (k < K && r < rows) v = x[(long long)k * ld + r];
      tile[tx][i] = v;
    } else {      // coalesced along K: x[r*ld + k]
      const int r = r0 + i, k = k0 + tx;
      if (k < K && r < rows) v = x[(long long)r * ld + k];
      tile[i][tx] = v;
    }
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int r = r0 + i, k = k0 + tx;
    if (r < rows && k < kpad) {
      const float v = tile[i][tx];
      const float h = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
      hi[(long long)r * kpad + k] = h;
      lo[(long long)r * kpad + k] = v - h;
    }
  }
}

// ---------------------------------------------------------------------------
// SIMT fallback/FFMA kernel: any shape, stride or alignment. Used for the
// "FFMA" f32 mode and for operands TMA cannot describe (row pitch not a
// multiple of 16 bytes). 64x64 output tile per 256-thread block, 4x4 per
// thread, fp32 accumulate.
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float ldf(const T* p) {
  if constexpr (sizeof(T) == 2)
    return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(p));
  else
    return *p;
}

template <typename T>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const T* __restrict__ A, const T* __restrict__ B,
                                                        GemmArgs args) {
  __shared__ float As[16][64 + 1];
  __shared__ float Bs[16][64 + 1];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  A += blockIdx.z * args.sA;  // batch (gridDim.z = 1 for a single product)
  B += blockIdx.z * args.sB;
  const long long boff = blockIdx.z * args.sC;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < args.K; k0 += 16) {
    for (int i = threadIdx.x; i < 16 * 64; i += 256) {
      const int kk = i / 64, mm = i % 64;
      const int m = m0 + mm, k = k0 + kk;
      float va = 0.f, vb = 0.f;
      if (m < args.M && k < args.K)
        va = ldf(A + (args.transA ? (long long)k * args.lda + m : (long long)m * args.lda + k));
      const int n = n0 + mm;
      if (n < args.N && k < args.K)
        vb = ldf(B + (args.transB ? (long long)n * args.ldb + k : (long long)k * args.ldb + n));
      As[kk][mm] = va;
      Bs[kk][mm] = vb;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= args.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n < args.N) gemm_store_one(args, m, n, acc[i][j], boff);
    }
  }
}

// ---------------------------------------------------------------------------
// Split-K reduction: C = epilogue(sum over slices of the fp32 partial tiles),
// four columns per thread, slices added in order (deterministic).
// ---------------------------------------------------------------------------
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, int ldw, GemmArgs a) {
  const int nq = (a.N + 3) / 4;
  const long long total = (long long)a.M * nq;
  const size_t slice = (size_t)a.M * ldw;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int m = (int)(i / nq), n = (int)(i % nq) * 4;
    float4 acc = *reinterpret_cast<const float4*>(ws + (size_t)m * ldw + n);
    for (int s = 1; s < splits; ++s) {
      const float4 v = *reinterpret_cast<const float4*>(ws + s * slice + (size_t)m * ldw + n);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    const float r[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (n + j < a.N) gemm_store_one(a, m, n + j, r[j]);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
// 3-D tiled map [batch][outer][inner]; a single product is batch 1.
static bool encode_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t inner, uint64_t outer,
                      uint64_t batch, uint64_t row_pitch_bytes, uint64_t batch_pitch_bytes, uint32_t box_inner,
                      uint32_t box_outer, CUtensorMapL2promotion l2) {
  auto enc = get_tensor_map_encoder();
  if (!enc) return false;
  if (batch <= 1) {
    batch = 1;
    batch_pitch_bytes = (row_pitch_bytes * outer + 15) & ~uint64_t(15);
  }
  cuuint64_t dims[3] = {inner, outer, batch};
  cuuint64_t strides[2] = {row_pitch_bytes, batch_pitch_bytes};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, l2, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Operand descriptor: logical [rows(MN), K] operand, stored either K-major
// (row r at base + r*ld, K contiguous) or MN-major (K row k at base + k*ld);
// `batch` such operands `bstride` elements apart.
template <bool TF32>
static bool make_operand_map(CUtensorMap* map, const void* base, bool mn_major, int mn, int K, int ld,
                             int box_mn, int batch, long long bstride) {
  using Cfg = GemmCfg<TF32>;  // element size, BK and the MN chunk do not depend on the tile width
  const CUtensorMapDataType dt = TF32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint64_t pitch = (uint64_t)ld * Cfg::ESZ, bpitch = (uint64_t)bstride * Cfg::ESZ;
  if (mn_major)
    return encode_3d(map, base, dt, (uint64_t)mn, (uint64_t)K, batch, pitch, bpitch, Cfg::CHUNK, Cfg::BK,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  return encode_3d(map, base, dt, (uint64_t)K, (uint64_t)mn, batch, pitch, bpitch, Cfg::BK, box_mn,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
}

int gemm_tc_supported(const GemmArgs& a, int esz, const void* A, const void* B) {
  // TMA wants 16-byte aligned bases and row / batch pitches that are multiples
  // of 16 bytes (a broadcast operand, batch stride 0, takes the SIMT kernel).
  if (((uintptr_t)A & 15) || ((uintptr_t)B & 15)) return 0;
  if (((long long)a.lda * esz) % 16 || ((long long)a.ldb * esz) % 16) return 0;
  if (a.batch > 1 && ((a.sA * esz) % 16 || (a.sB * esz) % 16 || a.sA <= 0 || a.sB <= 0)) return 0;
  if (a.M <= 0 || a.N <= 0 || a.K <= 0) return 0;
  return 1;
}

template <bool TF32, bool A_MN, bool B_MN, int BN_>
static cudaError_t launch_tc_bn(const GemmArgs& args, const void* A, const void* B, const void* A2, const void* B2,
                             cudaStream_t stream) {
  using Cfg = GemmCfg<TF32, BN_>;
  CUtensorMap ma{}, mb{}, ma2{}, mb2{};
  const int nb = args.batch > 1 ? args.batch : 1;
  if (!make_operand_map<TF32>(&ma, A, A_MN, args.M, args.K, args.lda, Cfg::BM, nb, args.sA))
    return cudaErrorInvalidValue;
  if (!make_operand_map<TF32>(&mb, B, B_MN, args.N, args.K, args.ldb, Cfg::BN, nb, args.sB))
    return cudaErrorInvalidValue;
  if (TF32) {
    if (!make_operand_map<TF32>(&ma2, A2, A_MN, args.M, args.K, args.lda, Cfg::BM, nb, args.sA))
      return cudaErrorInvalidValue;
    if (!make_operand_map<TF32>(&mb2, B2, B_MN, args.N, args.K, args.ldb, Cfg::BN, nb, args.sB))
      return cudaErrorInvalidValue;
  } else {
    ma2 = ma;
    mb2 = mb;
  }
  GemmArgs a = args;
  a.tiles_m = (args.M + Cfg::BM - 1) / Cfg::BM;
  a.tiles_n = (args.N + Cfg::BN - 1) / Cfg::BN;
  a.group_m = 16;
  // Split K over CTAs when the output tiles alone would leave most SMs idle
  // (the weight-gradient GEMMs dW = dY^T X: small outputs, K = tokens).
  a.splits = 1;
  float* ws = nullptr;
  int ldw = 0;
  {
    const int tiles = a.tiles_m * a.tiles_n;
    const int nk_all = (args.K + Cfg::BK - 1) / Cfg::BK;
    if (a.n_extra == 0 && nb == 1 && tiles * 2 <= num_sms() && nk_all >= 16) {
      const int sp = std::min(std::min(num_sms() / tiles, nk_all / 8), 16);
      ldw = (a.N + 3) & ~3;
      if (sp >= 2 && (ws = (float*)library_scratch_slot(kScratchSplitK, (size_t)sp * a.M * ldw * sizeof(float), stream)) !=
              nullptr)
        a.splits = sp;
    }
  }
  // Epilogue path (see GemmArgs::tma_out).
  CUtensorMap mc{};
  ExtraOutMaps mx{};
  if (a.splits > 1) {
    auto enc = get_tensor_map_encoder();
    const cuuint64_t dims[3] = {(cuuint64_t)a.N, (cuuint64_t)a.M, (cuuint64_t)a.splits};
    const cuuint64_t strides[2] = {(cuuint64_t)ldw * 4, (cuuint64_t)a.M * ldw * 4};
    const cuuint32_t box[3] = {32, 32, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (!enc || enc(&mc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, ws, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
    a.tma_out = 3;
  } else {
    const int esz = a.c_bf16 ? 2 : 4;
    const bool aligned = ((uintptr_t)a.C & 15) == 0 && ((long long)a.ldc * esz) % 16 == 0 &&
                         (nb == 1 || (a.sC * esz) % 16 == 0);
    int mode = 0;
    // TMA stores to extra destinations: bf16 operands with A K-major only
    // (the column-parallel GEMM); other extras take per-thread stores.
    const bool extra_ok = a.n_extra == 0 || (!TF32 && !A_MN && extras_tma_aligned(a));
    if (aligned && extra_ok) {
      if (a.beta == 0.f)
        mode = 1;
      else if (a.n_extra == 0 && a.beta == 1.f && !a.c_bf16 && !a.relu)
        mode = 2;
    }
    const CUtensorMapDataType cdt = a.c_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    if (mode && !encode_3d(&mc, a.C, cdt, (uint64_t)a.N, (uint64_t)a.M, nb, (uint64_t)a.ldc * esz,
                           (uint64_t)a.sC * esz, 128 / esz, 32, CU_TENSOR_MAP_L2_PROMOTION_NONE))
      mode = 0;
    for (int e = 0; mode && e < a.n_extra; ++e)  // every extra destination, same box
      if (!encode_3d(&mx.m[e], a.C_extra[e], cdt, (uint64_t)a.N, (uint64_t)a.M, nb, (uint64_t)a.ldc * esz,
                     (uint64_t)a.sC * esz, 128 / esz, 32, CU_TENSOR_MAP_L2_PROMOTION_NONE))
        mode = 0;
    a.tma_out = mode;
    if (!mode) mc = ma;  // unused
  }
  auto kern = gemm_tc_kernel<TF32, A_MN, B_MN, BN_, false>;
  const bool extra = a.tma_out == 1 && a.n_extra > 0;
  if constexpr (!TF32 && !A_MN) {
    if (extra) kern = gemm_tc_kernel<TF32, A_MN, B_MN, BN_, true>;
  }
  static bool attr_done[2] = {false, false};  // per template instantiation
  if (!attr_done[extra]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    attr_done[extra] = true;
  }
  const long long units = (long long)a.tiles_m * a.tiles_n * a.splits * nb;
  const int grid = units < num_sms() ? (int)units : num_sms();
  {
    TimerScope timer(stream);
    kern<<<grid, kGemmThreads, Cfg::SMEM_BYTES, stream>>>(ma, mb, ma2, mb2, mc, mx, a);
  }
  if (a.splits > 1) {
    const long long quads = (long long)a.M * ((a.N + 3) / 4);
    const int rb = (int)std::min<long long>((quads + 255) / 256, (long long)num_sms() * 8);
    splitk_reduce_kernel<<<rb, 256, 0, stream>>>(ws, a.splits, ldw, a);
  }
  return cudaGetLastError();
}

// Full-width tiles, or half-width ones when the full-width tiles would leave
// more than a quarter of the SMs idle (small problems such as the 1024^3
// f32 GEMMs of the autograd step).
template <bool TF32, bool A_MN, bool B_MN>
static cudaError_t launch_tc(const GemmArgs& args, const void* A, const void* B, const void* A2, const void* B2,
                             cudaStream_t stream) {
  constexpr int BN_FULL = GemmCfg<TF32>::BN;
  const long long tiles = (long long)((args.M + 127) / 128) * ((args.N + BN_FULL - 1) / BN_FULL) *
                          (args.batch > 1 ? args.batch : 1);
  if (tiles * 4 < (long long)num_sms() * 3)
    return launch_tc_bn<TF32, A_MN, B_MN, BN_FULL / 2>(args, A, B, A2, B2, stream);
  return launch_tc_bn<TF32, A_MN, B_MN, BN_FULL>(args, A, B, A2, B2, stream);
}

template <bool TF32>
static cudaError_t dispatch_tc(const GemmArgs& args, const void* A, const void* B, const void* A2, const void* B2,
                               cudaStream_t s) {
  // A is MN-major when stored transposed ([K,M]); B is MN-major when stored
  // as [K,N] (the plain row-major right operand of `@`).
  const bool a_mn = args.transA != 0, b_mn = args.transB == 0;
  if (!a_mn && !b_mn) return launch_tc<TF32, false, false>(args, A, B, A2, B2, s);
  if (!a_mn && b_mn) return launch_tc<TF32, false, true>(args, A, B, A2, B2, s);
  if (a_mn && !b_mn) return launch_tc<TF32, true, false>(args, A, B, A2, B2, s);
  return launch_tc<TF32, true, true>(args, A, B, A2, B2, s);
}

// 0: single-CTA kernel only; 1 (default): the 2-SM kernel (gemm2.cu) where eligible.
static int g_gemm_algo = 1;
void gemm_set_algo(int algo) { g_gemm_algo = algo; }

cudaError_t gemm_bf16_tc(const GemmArgs& args, const void* A, const void* B, cudaStream_t s) {
  if (g_gemm_algo == 1 && gemm2_eligible(args, A, B)) return gemm2_launch(args, A, B, s);
  return dispatch_tc<false>(args, A, B, nullptr, nullptr, s);
}

static int kpad4(int K) { return (K + 3) & ~3; }

size_t gemm_f32_scratch_floats(const GemmArgs& a) {
  const size_t kp = (size_t)kpad4(a.K);
  return 2 * ((size_t)a.M * kp + (size_t)a.N * kp) * (size_t)(a.batch > 1 ? a.batch : 1);
}

cudaError_t gemm_f32_3xtf32(const GemmArgs& args, const float* A, const float* B, float* scratch,
                            cudaStream_t s) {
  const int kp = kpad4(args.K);
  const int nb = args.batch > 1 ? args.batch : 1;
  // Planes [batch][rows][kp], K-major.
  float* a_hi = scratch;
  float* a_lo = a_hi + (size_t)nb * args.M * kp;
  float* b_hi = a_lo + (size_t)nb * args.M * kp;
  float* b_lo = b_hi + (size_t)nb * args.N * kp;
  const SplitJob ja{A, args.M, args.lda, args.transA, a_hi, a_lo, args.sA};
  const SplitJob jb{B, args.N, args.ldb, !args.transB, b_hi, b_lo, args.sB};
  dim3 grid((kp + 31) / 32, (std::max(args.M, args.N) + 31) / 32, 2 * nb);
  split_tf32_kernel<<<grid, 256, 0, s>>>(ja, jb, args.K, kp);
  GemmArgs a = args;
  a.K = kp;  // zero-filled tail contributes nothing
  a.lda = kp;
  a.ldb = kp;
  a.sA = (long long)args.M * kp;
  a.sB = (long long)args.N * kp;
  a.transA = 0;
  a.transB = 1;
  return launch_tc<true, false, false>(a, a_hi, b_hi, a_lo, b_lo, s);
}

cudaError_t gemm_simt(const GemmArgs& args, const void* A, const void* B, int bf16_in, cudaStream_t s) {
  dim3 grid((args.N + 63) / 64, (args.M + 63) / 64, args.batch > 1 ? args.batch : 1);
  if (bf16_in)
    gemm_simt_kernel<uint16_t><<<grid, 256, 0, s>>>((const uint16_t*)A, (const uint16_t*)B, args);
  else
    gemm_simt_kernel<float><<<grid, 256, 0, s>>>((const float*)A, (const float*)B, args);
  return cudaGetLastError();
}

}  // namespace dgx
