// Two-SM bf16 GEMM on sm_100a: tcgen05.mma.cta_group::2 over a CTA pair.
//
// Same contract as gemm_tc_kernel (C = op(A).op(B) (+beta C) (+bias) (ReLU),
// fp32 accumulate), for bf16 operands with A K-major and large enough outputs.
// A CTA pair (a cluster of 2) owns a 256 x 256 output tile: each CTA loads
// its own 128 rows of A and its own 128 columns of B (the pair's MMA reads the
// peer's half through the pair), so every SM streams 32 KB of operands per
// 64-wide K step instead of the 48 KB of a 128 x 256 single-CTA tile, and each
// CTA's TMEM holds its 128 rows of the tile, double-buffered (2 x 256 columns)
// so the epilogue of one tile overlaps the main loop of the next.
//
// Protocol (leader = cluster rank 0):
//   full[s]   leader only; the leader's producer expects both CTAs' bytes,
//             both CTAs' TMA loads complete on it (pair form, peer bit clear)
//   empty[s]  each CTA; the leader's MMA commit arrives on both (multicast)
//   accf[b]   each CTA; MMA commit to both when accumulator b is complete
//   acce[b]   leader only; the 4 epilogue warps of both CTAs release it
// No TMA load uses cluster multicast: each CTA fetches its own operand halves.
#include <algorithm>

#include "gemm.h"
#include "sm100.cuh"

namespace dgx {

namespace {

constexpr int G2_BM = 128;  // rows per CTA (256 per pair)
constexpr int G2_BN = 256;  // columns per pair tile (128 of B per CTA)
constexpr int G2_BK = 64;   // one 128-byte swizzled row of bf16 K
constexpr int G2_A_BYTES = G2_BM * G2_BK * 2;         // 16 KB
constexpr int G2_B_BYTES = (G2_BN / 2) * G2_BK * 2;   // 16 KB
constexpr int G2_STAGE = G2_A_BYTES + G2_B_BYTES;     // 32 KB per CTA
// Operand stages and output staging per instantiation: 6 stages and two
// 4 KB staging boxes per epilogue warp; with extra destinations (the
// column-parallel GEMM's peer stores, four or more TMA stores per box, whose
// reads of the box wait on NVLink) 5 stages and four boxes per warp, so a
// warp can stage two more boxes before it waits for earlier stores to leave.
template <bool EXTRA>
struct G2Cfg {
  static constexpr int STAGES = EXTRA ? 5 : 6;
  static constexpr int OUT_BUFS = EXTRA ? 4 : 2;
  static constexpr int OUT_STAGE = 4 * OUT_BUFS * 4096;
  static constexpr int SMEM = STAGES * G2_STAGE + OUT_STAGE + 1024 + 256;
};
constexpr uint32_t G2_TMEM_COLS = 512;
constexpr uint32_t kPeerBitMask = 0xFEFFFFFFu;  // shared::cluster address of the pair leader's copy

__device__ __forceinline__ uint32_t cluster_rank_u32() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all2() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::
          : "memory");
}
__device__ __forceinline__ void tmem_alloc2(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void mma2_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the barrier at this offset in every CTA of `mask` once the
// tcgen05 ops issued so far by this thread complete.
__device__ __forceinline__ void tc_commit2_mc(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}
// TMA load into this CTA's shared memory that completes on the pair leader's barrier.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar) & kPeerBitMask), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint64_t* bar, uint32_t cta) {
  asm volatile(
      "{\n\t.reg .b32 ra;\n\t"
      "mapa.shared::cluster.u32 ra, %0, %1;\n\t"
      "mbarrier.arrive.release.cluster.shared::cluster.b64 _, [ra];\n\t}" ::"r"(smem_u32(bar)),
      "r"(cta)
      : "memory");
}

struct Sched2 {
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

// EXTRA: every staged box also goes to the extra destinations (tmX).
template <bool B_MN, bool EXTRA>
__global__ void __launch_bounds__(192, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ CUtensorMap tmC, const __grid_constant__ ExtraOutMaps tmX,
                 GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int G2_STAGES = G2Cfg<EXTRA>::STAGES, OUT_BUFS = G2Cfg<EXTRA>::OUT_BUFS;
  uint8_t* out_stage = smem + G2_STAGES * G2_STAGE;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(out_stage + G2Cfg<EXTRA>::OUT_STAGE);
  uint64_t* empty_bar = full_bar + G2_STAGES;
  uint64_t* accf_bar = empty_bar + G2_STAGES;  // [2]
  uint64_t* acce_bar = accf_bar + 2;           // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank_u32();
  const bool leader = rank == 0;
  WaitCtx wc{abort_flag, args.err};

  if (threadIdx.x == 0) {
    for (int s = 0; s < G2_STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf_bar[b], 1);
      mbar_init(&acce_bar[b], 8);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {  // same warp in both CTAs, same destination offset
    tmem_alloc2(tmem_slot, G2_TMEM_COLS);
    tmem_relinquish2();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all2();  // both CTAs' barriers are initialised before any cross-CTA traffic
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const Sched2 sched{args.tiles_m, args.tiles_n, args.group_m};
  const int num_tiles = args.tiles_m * args.tiles_n;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int nk = (args.K + G2_BK - 1) / G2_BK;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (elect_one_lane()) {
      uint32_t fill = 0;
      for (int t = pair; t < num_tiles && !*abort_flag; t += npairs) {
        int tm, tn;
        sched.coords(t, tm, tn);
        const int m0 = tm * 2 * G2_BM + (int)rank * G2_BM;  // this CTA's 128 rows
        const int n0 = tn * G2_BN + (int)rank * (G2_BN / 2);  // this CTA's 128 columns of B
        for (int kb = 0; kb < nk; ++kb, ++fill) {
          const int s = fill % G2_STAGES;
          if (!mbar_wait(&empty_bar[s], ((fill / G2_STAGES) & 1) ^ 1, wc)) break;
          uint8_t* sa = smem + s * G2_STAGE;
          uint8_t* sb = sa + G2_A_BYTES;
          if (leader) mbar_arrive_expect_tx(&full_bar[s], 2 * G2_STAGE);
          const int k0 = kb * G2_BK;
          tma_load_2d_pair(sa, &tmA, &full_bar[s], k0, m0);
          if (B_MN) {
#pragma unroll
            for (int c = 0; c < 2; ++c) tma_load_2d_pair(sb + c * G2_BK * 128, &tmB, &full_bar[s], n0 + c * 64, k0);
          } else {
            tma_load_2d_pair(sb, &tmB, &full_bar[s], k0, n0);
          }
        }
        if (*abort_flag) break;
      }
      // Teardown: this CTA's copies must have landed (they complete on the
      // leader's barrier; the empty barriers of the last rounds mean the MMA
      // consumed them).
      const uint32_t first = fill > (uint32_t)G2_STAGES ? fill - G2_STAGES : 0;
      for (uint32_t f = first; f < fill; ++f) mbar_drain(&empty_bar[f % G2_STAGES], (f / G2_STAGES) & 1);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (leader && elect_one_lane()) {
      const uint32_t idesc = make_idesc(1, 0, B_MN ? 1u : 0u, 2 * G2_BM, G2_BN);
      const uint32_t b_lbo = B_MN ? G2_BK * 128 : 16;
      uint32_t fill = 0, use = 0;
      for (int t = pair; t < num_tiles; t += npairs, ++use) {
        const int buf = use & 1;
        if (!mbar_wait(&acce_bar[buf], ((use >> 1) & 1) ^ 1, wc)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * G2_BN;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb, ++fill) {
          const int s = fill % G2_STAGES;
          if (!mbar_wait(&full_bar[s], (fill / G2_STAGES) & 1, wc)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * G2_STAGE), sb = sa + G2_A_BYTES;
#pragma unroll
          for (int kk = 0; kk < G2_BK / 16; ++kk) {
            const uint64_t adesc = sw128_desc(sa + kk * 32, 16, 1024);
            const uint64_t bdesc = sw128_desc(sb + (B_MN ? kk * 16 * 128 : kk * 32), b_lbo, 1024);
            mma2_f16_ss(d_tmem, adesc, bdesc, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit2_mc(&empty_bar[s], 0x3);  // stage free in both CTAs
        }
        if (!ok) break;
        tc_commit2_mc(&accf_bar[buf], 0x3);  // accumulator complete in both CTAs
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5, both CTAs)
    const int q = warp & 3;
    uint8_t* my_stage = out_stage + (warp - 2) * OUT_BUFS * 4096;
    uint32_t issued = 0, use = 0;
    if (lane == 0) {
      tma_prefetch_desc(&tmC);
      if (EXTRA)
        for (int e = 0; e < args.n_extra; ++e) tma_prefetch_desc(&tmX.m[e]);
    }
    for (int t = pair; t < num_tiles; t += npairs, ++use) {
      const int buf = use & 1;
      int tm, tn;
      sched.coords(t, tm, tn);
      prefetch_bias_l1(args.bias, tn * G2_BN, G2_BN, args.N, lane);
      if (!mbar_wait(&accf_bar[buf], (use >> 1) & 1, wc)) break;
      tc_fence_after();
      const int row0 = tm * 2 * G2_BM + (int)rank * G2_BM + q * 32;
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + buf * G2_BN;
      const int cw = args.c_bf16 ? 64 : 32;
#pragma unroll 1
      for (int c = 0; c < G2_BN; c += cw) {
        uint32_t r[64];
        tmem_ld32(taddr + c, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
        if (cw == 64) tmem_ld32(taddr + c + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
        float bq[64];  // this chunk's bias: the loads overlap the TMEM load
        if (args.bias) {
#pragma unroll
          for (int j8 = 0; j8 < 64; j8 += 8)
            if (j8 < cw) {
              float b8[8];
              load_bias8(args.bias, tn * G2_BN + c + j8, args.N, b8);
#pragma unroll
              for (int i = 0; i < 8; ++i) bq[j8 + i] = b8[i];
            }
        }
        tmem_ld_wait();
        if (c + cw >= G2_BN) {  // accumulator read out: release it to the leader's MMA warp
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (leader)
              mbar_arrive(&acce_bar[buf]);
            else
              mbar_arrive_remote(&acce_bar[buf], 0);
          }
        }
        const int n0 = tn * G2_BN + c;
        if (n0 >= args.N) continue;
        uint8_t* st = my_stage + (issued % OUT_BUFS) * 4096;
        if (lane == 0 && issued >= (uint32_t)OUT_BUFS) {
          if constexpr (OUT_BUFS == 4)
            bulk_wait_read3();
          else
            bulk_wait_read1();
        }
        __syncwarp();
        uint32_t w[32];
        if (args.c_bf16) {
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
          if (args.tma_out == 2)
            tma_reduce_add_2d(&tmC, st, n0, row0);
          else {
            tma_store_2d(&tmC, st, n0, row0);
            if (EXTRA)
              for (int e = 0; e < args.n_extra; ++e) tma_store_2d(&tmX.m[e], st, n0, row0);
          }
          bulk_commit();  // one group per staged buffer, all its destinations
        }
        ++issued;
      }
    }
    if (lane == 0) bulk_wait0();
  }

  // Neither CTA leaves (or frees TMEM) while its pair may still use its
  // shared memory or TMEM.
  tc_fence_before();
  __syncthreads();
  cluster_sync_all2();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc2(tmem_base, G2_TMEM_COLS);
  }
}

bool encode_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t pitch_bytes,
                    uint32_t box_inner, uint32_t box_outer) {
  auto enc = get_tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {pitch_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// Whether the 2-SM kernel serves this bf16 GEMM: A K-major, one output with a
// TMA-storable layout (beta 0, or 1 with fp32 C), extra destinations only
// with beta 0, B stored [K][N] and 16-byte aligned pointers (each staged box
// is stored to all), enough 256 x 256 tiles to occupy the GPU's SM pairs, and
// K >= 1024 (below that the single-CTA 128 x 256 tiles measured faster on
// this GPU: more tiles for the short main loops).
bool gemm2_eligible(const GemmArgs& a, const void* A, const void* B) {
  if (a.transA || a.batch > 1) return false;
  if (a.n_extra && (a.beta != 0.f || a.transB || !extras_tma_aligned(a))) return false;
  const int esz = a.c_bf16 ? 2 : 4;
  if ((((uintptr_t)a.C | (uintptr_t)A | (uintptr_t)B) & 15) || ((long long)a.ldc * esz) % 16) return false;
  if (((long long)a.lda * 2) % 16 || ((long long)a.ldb * 2) % 16) return false;
  if (!(a.beta == 0.f || (a.beta == 1.f && !a.c_bf16 && !a.relu))) return false;
  const long long tiles = (long long)((a.M + 255) / 256) * ((a.N + 255) / 256);
  return a.K >= 1024 && tiles * 2 >= num_sms();
}

cudaError_t gemm2_launch(const GemmArgs& args, const void* A, const void* B, cudaStream_t stream) {
  const bool b_mn = args.transB == 0;
  CUtensorMap ma{}, mb{}, mc{};
  ExtraOutMaps mx{};
  if (!encode_2d_bf16(&ma, A, (uint64_t)args.K, (uint64_t)args.M, (uint64_t)args.lda * 2, G2_BK, G2_BM))
    return cudaErrorInvalidValue;
  if (b_mn) {  // B stored [K][N]: boxes of 64 columns x 64 K rows
    if (!encode_2d_bf16(&mb, B, (uint64_t)args.N, (uint64_t)args.K, (uint64_t)args.ldb * 2, 64, G2_BK))
      return cudaErrorInvalidValue;
  } else {  // B stored [N][K]
    if (!encode_2d_bf16(&mb, B, (uint64_t)args.K, (uint64_t)args.N, (uint64_t)args.ldb * 2, G2_BK, G2_BN / 2))
      return cudaErrorInvalidValue;
  }
  GemmArgs a = args;
  a.tiles_m = (args.M + 255) / 256;
  a.tiles_n = (args.N + G2_BN - 1) / G2_BN;
  a.group_m = 8;
  a.splits = 1;
  a.tma_out = args.beta == 0.f ? 1 : 2;
  {
    auto enc = get_tensor_map_encoder();
    const int esz = a.c_bf16 ? 2 : 4;
    const cuuint64_t dims[2] = {(cuuint64_t)a.N, (cuuint64_t)a.M};
    const cuuint64_t strides[1] = {(cuuint64_t)a.ldc * esz};
    const cuuint32_t box[2] = {(cuuint32_t)(128 / esz), 32};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType cdt = a.c_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    if (!enc) return cudaErrorInvalidValue;
    for (int e = -1; e < a.n_extra; ++e)  // C, then every extra destination
      if (enc(e < 0 ? &mc : &mx.m[e], cdt, 2, e < 0 ? a.C : a.C_extra[e], dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
  }
  const bool extra = a.n_extra > 0;  // B stored [K][N] (gemm2_eligible)
  auto kern = extra ? gemm2_kernel<true, true> : b_mn ? gemm2_kernel<true, false> : gemm2_kernel<false, false>;
  const int variant = extra ? 2 : b_mn;
  const int smem = extra ? G2Cfg<true>::SMEM : G2Cfg<false>::SMEM;
  static bool attr_done[3] = {false, false, false};
  if (!attr_done[variant]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_done[variant] = true;
  }
  const int tiles = a.tiles_m * a.tiles_n;
  const int pairs = std::min(tiles, num_sms() / 2);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  TimerScope timer(stream);
  return cudaLaunchKernelEx(&cfg, kern, ma, mb, mc, mx, a);
}

}  // namespace dgx
