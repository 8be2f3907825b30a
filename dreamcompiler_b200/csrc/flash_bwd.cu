// FlashAttention backward on sm_100a (tcgen05 + TMEM + TMA).
//
// Replaces the "flash_attention" branch of backward()
// (runtime/ops/autograd.inc:779-840). The reference recomputes each row's
// softmax statistics (pass 1), D_i = dO_i.O_i (pass 2) and then P, dS and the
// three gradients (pass 3) in f64 scalar loops. Here the forward's LSE
// replaces pass 1, a small kernel computes D_i (pass 2), and one tensor-core
// kernel does pass 3 with the same identities:
//   P = exp(scale*QK^T - LSE),  dV = P^T dO,  dP = dO V^T,
//   dS = P o (dP - D),  dQ = scale * dS K,  dK = scale * dS^T Q.
//
// The kernel is persistent (one CTA per SM). Each work item is one 128-key
// K/V tile of one head, kept resident in shared memory (two buffers, so the
// next item's tile loads during the current one) while the CTA walks the
// 128-row Q tiles that can see it (causal: i >= j). Per Q tile the MMA warp
// issues
//   S^T = K Q^T, dP^T = V dO^T           (TMEM, lanes = keys)
//   dV += P^T dO, dK += dS^T Q           (P^T, dS^T read from TMEM)
//   dQ_part = dS K                       (dS staged in shared memory)
// The Q tile's two 64-query halves (query groups 0-1 and 2-3, eight compute
// warps each) run their own chains: S^T and dP^T are issued per half (N =
// 64), and the halves take turns on the exponentials (MUFU), so one half's
// dS work and hand-offs run while the other's exponentials do. The MMA warp
// issues, per Q tile,
//   dV(i) of half 0, S(i+1) of half 0 | dV(i) of half 1, S(i+1) of half 1 |
//   dK(i) of half 0, dP(i+1) of half 0 | dK(i) of half 1, dQ(i), dP(i+1) of
//   half 1,
// the order in which the halves' P^T and dS^T hand-offs arrive; dV and dK go
// out in parts of one query group of four warps each. dQ partials go
// through two TMEM buffers to 4 drain warps that add them into an fp32
// accumulator: each partial tile is staged in shared memory and added with one
// TMA bulk reduce (cp.reduce.async.bulk.tensor .add) per tile; a last kernel
// scales the accumulator and casts it to bf16.
#include <math.h>

#include <atomic>

#include "common.h"
#include "flash.h"
#include "sm100.cuh"

namespace dgx {

namespace {

constexpr int BKV = 128;  // keys per CTA
constexpr int BQ = 128;   // queries per step
constexpr int DP = 64;
// A query half hands the exponentials over to the other half after the
// first 16 of its 32 columns: the other half's wait ends while these still
// keep MUFU busy (328 us at config 2, against 333 handing over after all 32).
constexpr int TURN_CC = 0;
constexpr int Q_STAGES = 3;   // Q tiles (with their row statistics): released after dK
constexpr int DO_STAGES = 2;  // dO tiles: released after dV
constexpr int TILE = 128 * DP * 2;  // 16 KB
// Warps 0-15 compute (four groups of four, one per 32 queries of the Q tile),
// 16-19 dQ drain, 20 TMA, 21 MMA, 22-23 idle: four compute warps per SM
// sub-partition, so one warp's TMEM loads and exponentials hide behind the
// others'.
constexpr int NUM_THREADS = 768;
constexpr int W_DRAIN = 16, W_TMA = 20, W_MMA = 21;
// setmaxnreg split (per thread): 16 x 88 + 4 x 72 + 4 x 56 = 24 x 80 (the launch allocation).
constexpr uint32_t REG_COMPUTE = 88, REG_DRAIN = 72, REG_CTRL = 56;

constexpr int SM_K = 0, SM_V = 2 * TILE, SM_Q = 4 * TILE, SM_DO = SM_Q + Q_STAGES * TILE;  // K, V: 2 buffers
constexpr int SM_DS = SM_DO + DO_STAGES * TILE;  // 128 queries x 128 keys bf16, MN-major (2 x 16 KB)
constexpr int SM_STAT = SM_DS + 2 * TILE;  // per stage: L2 stats [128] then D stats [128] (fp32)
constexpr int STAT_BYTES = 2 * BQ * 4;
constexpr int SM_DQ = SM_STAT + Q_STAGES * STAT_BYTES;  // dQ staging: 2 boxes of 128 rows x 32 fp32 (SW128)
constexpr int DQ_BOX = 128 * 128;
constexpr int SM_BAR = SM_DQ + 2 * DQ_BOX;
constexpr int SMEM_BYTES = SM_BAR + 512 + 1024;

constexpr uint32_t T_ST = 0, T_DPT = 128, T_DV = 256, T_DK = 320, T_DQ = 384;  // T_DQ: 2 x 64
constexpr uint32_t TMEM_COLS = 512;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}


struct BwdBars {
  uint64_t kv_full[2], kv_empty[2], q_full[Q_STAGES], q_empty[Q_STAGES], do_full[DO_STAGES], do_empty[DO_STAGES];
  uint64_t s_full[2], dp_full[2], turn[2], p_ready[4], ds_ready[4], dq_full[2], dq_empty[2], acc_done, ds_free;
  uint32_t tmem_slot;
  int abort;
};

__global__ void __launch_bounds__(NUM_THREADS, 1)
    flash_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO,
                     const __grid_constant__ CUtensorMap tmdQacc, FlashBwdArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  BwdBars* bars = reinterpret_cast<BwdBars*>(smem + SM_BAR);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  WaitCtx wc{&bars->abort, args.err};

  // Persistent: this CTA walks work items w = blockIdx.x, +gridDim.x, ...;
  // item w is key tile j = w / BH of head bh = w % BH (heaviest first under
  // causal). Barrier phases run on across items: `ic` counts this CTA's
  // items, `gt` its Q tiles. (The alternating order of snake_item balances
  // the CTAs' work better on paper, 0.99 against 0.94 of the mean at config
  // 2, but measured 7 % slower here: 379 against 352 us.)
  const int nq = (args.S + BQ - 1) / BQ;
  const int nitems = ((args.S + BKV - 1) / BKV) * args.BH;
  struct Item {
    int j, bh, i0, n;
    int b, h;  // bh = b*H + h
  };
  auto item = [&](int w) {
    Item it;
    it.j = w / args.BH;
    it.bh = w % args.BH;
    it.b = it.bh / args.H;
    it.h = it.bh - it.b * args.H;
    it.i0 = args.causal ? (it.j * BKV) / BQ : 0;
    it.n = nq - it.i0;
    return it;
  };

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->kv_full[b], 1);
      mbar_init(&bars->kv_empty[b], 1);
    }
    for (int s = 0; s < DO_STAGES; ++s) {
      mbar_init(&bars->do_full[s], 1);
      mbar_init(&bars->do_empty[s], 1);
    }
    for (int s = 0; s < Q_STAGES; ++s) {
      mbar_init(&bars->q_full[s], 1);
      mbar_init(&bars->q_empty[s], 1);
    }
    for (int x = 0; x < 2; ++x) {  // per query half (groups 0-1, 2-3)
      mbar_init(&bars->s_full[x], 1);
      mbar_init(&bars->dp_full[x], 1);
      mbar_init(&bars->turn[x], 8);
    }
    for (int g = 0; g < 4; ++g) {  // one per query group (4 warps each)
      mbar_init(&bars->p_ready[g], 4);
      mbar_init(&bars->ds_ready[g], 4);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->dq_full[b], 1);
      mbar_init(&bars->dq_empty[b], 4);
    }
    mbar_init(&bars->acc_done, 1);
    mbar_init(&bars->ds_free, 1);
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == W_MMA) {
    tmem_alloc(&bars->tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_slot;
  // Launched as a programmatic dependent of the row pre-pass: its statistics
  // and the zeroed dQ accumulator are visible after this wait. The dQ
  // conversion kernel may be scheduled from here on (it waits for this grid).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // Each role's setmaxnreg sits inside its branch so that it dominates (and
  // sets the register limit for) exactly that role's code.
  if (warp >= W_TMA) {
   regs_dec<REG_CTRL>();
   if (warp == W_TMA) {
    // ---------------------------------------------------------------- TMA
    if (elect_one_lane()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmdO);
      int gt = 0, ic = 0, gdo = 0;  // gt: Q tiles issued, gdo: dO tiles issued
      bool ok = true;
      uint32_t kv_filled = 0;  // items whose K/V load was issued
      for (int w = blockIdx.x; ok && w < nitems; w += gridDim.x, ++ic) {
        const Item I = item(w);
        const int kb = ic & 1;
        if (!(ok = mbar_wait(&bars->kv_empty[kb], ((ic >> 1) & 1) ^ 1, wc))) break;
        mbar_arrive_expect_tx(&bars->kv_full[kb], 2 * TILE);
        if (args.dense3d) {
          tma_load_3d(smem + SM_K + kb * TILE, &tmK, &bars->kv_full[kb], 0, I.j * BKV, I.bh);
          tma_load_3d(smem + SM_V + kb * TILE, &tmV, &bars->kv_full[kb], 0, I.j * BKV, I.bh);
        } else {
          tma_load_4d(smem + SM_K + kb * TILE, &tmK, &bars->kv_full[kb], 0, I.h, I.j * BKV, I.b);
          tma_load_4d(smem + SM_V + kb * TILE, &tmV, &bars->kv_full[kb], 0, I.h, I.j * BKV, I.b);
        }
        ++kv_filled;
        const float* Dstat = args.rowstat + (size_t)I.bh * args.Spad;
        const float* L2stat = args.rowstat + (size_t)args.BH * args.Spad + (size_t)I.bh * args.Spad;
        for (int it = 0; it < I.n; ++it, ++gt) {
          const int s = gt % Q_STAGES, d = gt % DO_STAGES;
          if (!(ok = mbar_wait(&bars->q_empty[s], ((gt / Q_STAGES) & 1) ^ 1, wc))) break;
          mbar_arrive_expect_tx(&bars->q_full[s], TILE + STAT_BYTES);
          if (args.dense3d)
            tma_load_3d(smem + SM_Q + s * TILE, &tmQ, &bars->q_full[s], 0, (I.i0 + it) * BQ, I.bh);
          else
            tma_load_4d(smem + SM_Q + s * TILE, &tmQ, &bars->q_full[s], 0, I.h, (I.i0 + it) * BQ, I.b);
          uint8_t* st = smem + SM_STAT + s * STAT_BYTES;
          bulk_load(st, L2stat + (I.i0 + it) * BQ, BQ * 4, &bars->q_full[s]);
          bulk_load(st + BQ * 4, Dstat + (I.i0 + it) * BQ, BQ * 4, &bars->q_full[s]);
          if (!(ok = mbar_wait(&bars->do_empty[d], ((gt / DO_STAGES) & 1) ^ 1, wc))) {
            ++gt;  // the Q copy was issued: the teardown drains it
            break;
          }
          mbar_arrive_expect_tx(&bars->do_full[d], TILE);
          if (args.dense3d)
            tma_load_3d(smem + SM_DO + d * TILE, &tmdO, &bars->do_full[d], 0, (I.i0 + it) * BQ, I.bh);
          else
            tma_load_4d(smem + SM_DO + d * TILE, &tmdO, &bars->do_full[d], 0, I.h, (I.i0 + it) * BQ, I.b);
          ++gdo;
        }
      }
      // Teardown: every copy issued must have landed before the CTA leaves.
      for (uint32_t f = kv_filled > 2 ? kv_filled - 2 : 0; f < kv_filled; ++f) mbar_drain(&bars->kv_full[f & 1], (f >> 1) & 1);
      for (int f = max(0, gt - Q_STAGES); f < gt; ++f) mbar_drain(&bars->q_full[f % Q_STAGES], (f / Q_STAGES) & 1);
      for (int f = max(0, gdo - DO_STAGES); f < gdo; ++f)
        mbar_drain(&bars->do_full[f % DO_STAGES], (f / DO_STAGES) & 1);
    }
  } else if (warp == W_MMA) {
    // ---------------------------------------------------------------- MMA
    if (elect_one_lane()) {
      constexpr uint32_t id_acc = make_idesc(1, 0, 1, 128, DP);  // TMEM A x MN-major B, N = D
      constexpr uint32_t id_dq = make_idesc(1, 1, 1, 128, DP);   // MN-major dS x MN-major K
      const uint32_t sQ = smem_u32(smem + SM_Q), sdO = smem_u32(smem + SM_DO), sdS = smem_u32(smem + SM_DS);
      // Descriptors advance by adding (byte offset >> 4) to the start field.
      // d[:, 64h : 64h+64] = a . b[64h : 64h+64]^T over D: one query half
      // (b's rows 64h.. are 8 KB into the SW128 tile), N = 64.
      constexpr uint32_t id_h = make_idesc(1, 0, 0, 128, 64);
      auto half_pair = [&](uint32_t d, uint32_t a, uint32_t b, int h) {
        const uint64_t da = sw128_desc(a, 16, 1024), db = sw128_desc(b + h * 8192, 16, 1024);
#pragma unroll 1
        for (int kk = 0; kk < DP / 16; ++kk) mma_f16_ss(d + 64 * h, da + 2 * kk, db + 2 * kk, id_h, kk > 0);
      };
      // d += A(tmem) . B over the 32 queries of group g (K steps 2g, 2g+1)
      auto tmem_a_acc_g = [&](uint32_t d, uint32_t a_tmem, uint32_t b, bool first, int g) {
        const uint64_t db = sw128_desc(b, DP * 128, 1024);
#pragma unroll
        for (int kk = 2 * g; kk < 2 * g + 2; ++kk)
          mma_f16_ts(d, a_tmem + 32 * (kk >> 1) + 8 * (kk & 1), db + 128 * kk, id_acc, (!first || kk > 0) ? 1u : 0u);
      };
      int gt = 0, ic = 0;
      bool ok = true;
      for (int w = blockIdx.x; ok && w < nitems; w += gridDim.x, ++ic) {
        const Item I = item(w);
        const int kb = ic & 1;
        const uint32_t sK = smem_u32(smem + SM_K + kb * TILE), sV = smem_u32(smem + SM_V + kb * TILE);
        // S^T and dP^T of the item's first tile: their TMEM was last read by
        // the previous item's final dV / dK MMAs, issued before them.
        if (!(ok = mbar_wait(&bars->kv_full[kb], (ic >> 1) & 1, wc) &&
                   mbar_wait(&bars->q_full[gt % Q_STAGES], (gt / Q_STAGES) & 1, wc)))
          break;
        tc_fence_after();
        for (int h = 0; h < 2; ++h) {
          half_pair(tmem + T_ST, sK, sQ + (gt % Q_STAGES) * TILE, h);
          tc_commit(&bars->s_full[h]);
        }
        if (!(ok = mbar_wait(&bars->do_full[gt % DO_STAGES], (gt / DO_STAGES) & 1, wc))) break;
        tc_fence_after();
        for (int h = 0; h < 2; ++h) {
          half_pair(tmem + T_DPT, sV, sdO + (gt % DO_STAGES) * TILE, h);
          tc_commit(&bars->dp_full[h]);
        }
        for (int it = 0; it < I.n; ++it, ++gt) {
          const int s = gt % Q_STAGES, d = gt % DO_STAGES;
          const uint32_t q_s = sQ + s * TILE, do_s = sdO + d * TILE;
          const bool next = it + 1 < I.n;
          const int s1 = (gt + 1) % Q_STAGES, d1 = (gt + 1) % DO_STAGES;
          // dV += P^T dO, each query group's 32 queries as soon as its P^T is
          // in TMEM (the groups finish their exponentials at different
          // times). p_ready of an item's first tile also means a group has
          // read out its part of the previous item's dV / dK: the first dV,
          // which overwrites all of it, waits for all four groups.
          if (it == 0)
            for (int g = 0; ok && g < 4; ++g) ok = mbar_wait(&bars->p_ready[g], gt & 1, wc);
          // Each query half runs its own S -> P -> dV -> S(next) and
          // dP -> dS -> dK -> dP(next) chains; the halves take turns on the
          // exponentials, so this issue order follows the order their
          // hand-offs arrive in: P of half 0, P of half 1, dS of half 0, dS
          // of half 1.
          for (int h = 0; ok && h < 2; ++h) {
            for (int g = 2 * h; ok && g < 2 * h + 2; ++g) {  // dV += P^T dO
              if (!(ok = mbar_wait(&bars->p_ready[g], gt & 1, wc))) break;
              tc_fence_after();
              tmem_a_acc_g(tmem + T_DV, tmem + T_ST, do_s, it == 0, g);
            }
            if (!ok) break;
            if (h == 1) tc_commit(&bars->do_empty[d]);  // dV(i) is the last MMA that reads dO(i)
            if (next) {  // S^T(i+1) of this half, over its P^T(i) that dV has read
              if (!(ok = mbar_wait(&bars->q_full[s1], ((gt + 1) / Q_STAGES) & 1, wc))) break;
              tc_fence_after();
              half_pair(tmem + T_ST, sK, sQ + s1 * TILE, h);
              tc_commit(&bars->s_full[h]);
            }
          }
          if (!ok) break;
          for (int h = 0; ok && h < 2; ++h) {
            for (int g = 2 * h; ok && g < 2 * h + 2; ++g) {  // dK += dS^T Q
              if (!(ok = mbar_wait(&bars->ds_ready[g], gt & 1, wc))) break;
              tc_fence_after();
              tmem_a_acc_g(tmem + T_DK, tmem + T_DPT, q_s, it == 0, g);
            }
            if (!ok) break;
            if (h == 1) {
              tc_commit(&bars->q_empty[s]);  // dK(i) is the last MMA that reads Q(i)
              // dQ_part = dS K, as soon as both halves' dS(i) are in shared
              // memory; ds_free tells the compute warps the tile has been read.
              const int b = gt & 1;
              if (!(ok = mbar_wait(&bars->dq_empty[b], ((gt >> 1) & 1) ^ 1, wc))) break;
              tc_fence_after();
              const uint64_t da = sw128_desc(sdS, BKV * 128, 1024), dk = sw128_desc(sK, DP * 128, 1024);
#pragma unroll 1
              for (int kk = 0; kk < BKV / 16; ++kk)
                mma_f16_ss(tmem + T_DQ + 64 * b, da + 128 * kk, dk + 128 * kk, id_dq, kk > 0);
              tc_commit(&bars->dq_full[b]);
              tc_commit(&bars->ds_free);
            }
            if (next) {  // dP^T(i+1) of this half, over its dS^T(i) that dK has read
              if (!(ok = mbar_wait(&bars->do_full[d1], ((gt + 1) / DO_STAGES) & 1, wc))) break;
              tc_fence_after();
              half_pair(tmem + T_DPT, sV, sdO + d1 * TILE, h);
              tc_commit(&bars->dp_full[h]);
            }
          }
          if (!ok) break;
        }
        if (!ok) break;
        tc_commit(&bars->acc_done);    // dV, dK of this item complete
        tc_commit(&bars->kv_empty[kb]);  // K and V no longer read
      }
    }
    __syncwarp();
   }
  } else if (warp >= W_DRAIN) {
    regs_dec<REG_DRAIN>();
    // ---------------------------------------------------------------- dQ drain
    const int qw = warp & 3;
    const int row = qw * 32 + lane;
    const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
    const bool issuer = warp == W_DRAIN && lane == 0;
    uint8_t* stage = smem + SM_DQ;
    if (issuer) tma_prefetch_desc(&tmdQacc);
    int gt = 0;
    bool ok = true;
    for (int w = blockIdx.x; ok && w < nitems; w += gridDim.x) {
      const Item I = item(w);
      for (int it = 0; it < I.n; ++it, ++gt) {
        const int b = gt & 1;
        if (!(ok = mbar_wait(&bars->dq_full[b], (gt >> 1) & 1, wc))) break;
        // The previous tile's bulk reduce must have read the staging tile.
        if (issuer) bulk_wait_read0();
        named_bar_sync(1, 128);
        tc_fence_after();
        // Row `row`, columns [32c, 32c+32) -> box c; 16-byte unit u at u ^ (row & 7).
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_off + T_DQ + 64 * b + 32 * c, v);
          tmem_ld_wait();
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<uint4*>(stage + c * DQ_BOX + row * 128 + ((u ^ (row & 7)) << 4)) =
                make_uint4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->dq_empty[b]);
        fence_proxy_async_smem();
        named_bar_sync(1, 128);
        if (issuer) {
          const int q0 = (I.i0 + it) * BQ;
          tma_reduce_add_3d(&tmdQacc, stage, 0, q0, I.bh);
          if (args.D > 32) tma_reduce_add_3d(&tmdQacc, stage + DQ_BOX, 32, q0, I.bh);
          bulk_commit();
        }
      }
    }
    if (issuer) bulk_wait0();
  } else {
    regs_inc<REG_COMPUTE>();
    // ---------------------------------------------------------------- compute (P, dS)
    // Warp quarter qw holds keys (TMEM lanes) 32qw..; group g the queries
    // [32g, 32g+32) of the Q tile. Each group writes its packed bf16 P^T and
    // dS^T (16 columns) over the first half of the 32 columns it read.
    const int qw = warp & 3, g = warp >> 2;
    const int kr = qw * 32 + lane;
    const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
    const float sl2 = args.scale * 1.4426950408889634f;
    uint8_t* ds_tile = smem + SM_DS + (g >> 1) * TILE;  // queries [64(g/2), 64(g/2)+64)
    const int unit0 = 4 * (g & 1);                      // this group's 16-byte units in a 128-byte row
    int gt = 0, ic = 0;
    bool ok = true;
    for (int w = blockIdx.x; ok && w < nitems; w += gridDim.x, ++ic) {
      const Item I = item(w);
      const int key = I.j * BKV + kr;
      const bool kvalid = key < args.S;
      for (int it = 0; it < I.n; ++it, ++gt) {
        const int q0 = (I.i0 + it) * BQ + 32 * g;  // first query of this group
        // Causal mask only where a query of the group precedes this key;
        // rows past S carry L2 = +inf (P = 0) in the padded statistics.
        const bool diag = args.causal && q0 < I.j * BKV + BKV - 1;
        const float* st = reinterpret_cast<const float*>(smem + SM_STAT + (gt % Q_STAGES) * STAT_BYTES);
        const float* Ls = st + 32 * g;
        const float* Ds = st + BQ + 32 * g;
        if (!(ok = mbar_wait(&bars->s_full[g >> 1], gt & 1, wc))) break;
        tc_fence_after();
        // The two query halves take turns on the exponentials (MUFU): half 0
        // of tile i after half 1 of tile i-1, half 1 after half 0, so one
        // half's dS work and hand-offs run while the other's exponentials do.
        if (g < 2 ? gt > 0 : true) {
          if (!(ok = mbar_wait(&bars->turn[g >> 1], (g < 2 ? gt - 1 : gt) & 1, wc))) break;
        }
        float p[32];
#pragma unroll
        for (int cc = 0; cc < 32; cc += 16) {
          uint32_t sv[16];
          tmem_ld16(tmem + lane_off + T_ST + 32 * g + cc, sv);
          float lv[16];
#pragma unroll
          for (int t = 0; t < 16; t += 4) *reinterpret_cast<float4*>(&lv[t]) = *reinterpret_cast<const float4*>(Ls + cc + t);
          tmem_ld_wait();
          static_for<0, 16, 2>([&](auto tt) {  // column pairs: one packed fp32 FMA per two scores
            constexpr int t = decltype(tt)::value;
            const float2 a = ffma2(__uint_as_float(sv[t]), __uint_as_float(sv[t + 1]), sl2, -lv[t], -lv[t + 1]);
            p[cc + t] = ex2(a.x);
            p[cc + t + 1] = ex2(a.y);
          });
          if (cc == TURN_CC) {  // hand the exponentials over to the other half
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->turn[(g >> 1) ^ 1]);
          }
        }
        if (diag) {
#pragma unroll
          for (int t = 0; t < 32; ++t) p[t] = q0 + t < key ? 0.f : p[t];
        }
        if (!kvalid) {
#pragma unroll
          for (int t = 0; t < 32; ++t) p[t] = 0.f;
        }
        {
          uint32_t pk[16];
#pragma unroll
          for (int t = 0; t < 16; ++t) pk[t] = pack_bf16x2(p[2 * t], p[2 * t + 1]);
          tmem_st16(tmem + lane_off + T_ST + 32 * g, pk);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->p_ready[g]);
        if (!(ok = mbar_wait(&bars->dp_full[g >> 1], gt & 1, wc))) break;
        tc_fence_after();
        uint32_t pk[16];
#pragma unroll
        for (int cc = 0; cc < 32; cc += 16) {
          uint32_t dv[16];
          tmem_ld16(tmem + lane_off + T_DPT + 32 * g + cc, dv);
          float dd[16];
#pragma unroll
          for (int t = 0; t < 16; t += 4) *reinterpret_cast<float4*>(&dd[t]) = *reinterpret_cast<const float4*>(Ds + cc + t);
          tmem_ld_wait();
#pragma unroll
          for (int t = 0; t < 16; t += 2) {  // dS = P o (dP - D), two columns per packed op
            const float2 ds = fsubmul2(__uint_as_float(dv[t]), __uint_as_float(dv[t + 1]), dd[t], dd[t + 1], p[cc + t],
                                       p[cc + t + 1]);
            pk[(cc + t) / 2] = pack_bf16x2(ds.x, ds.y);
          }
        }
        tmem_st16(tmem + lane_off + T_DPT + 32 * g, pk);
        // dS tile for the dQ MMA: row = key kr, 128-byte row holds queries
        // [64(g/2), 64(g/2)+64), 16-byte units XOR-swizzled by (kr & 7). The
        // previous dQ must have read it (the other half may still be on the
        // previous tile's dS when this half reaches here).
        if (!(ok = mbar_wait(&bars->ds_free, (gt & 1) ^ 1, wc))) break;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int unit = unit0 + u;
          uint4* dst = reinterpret_cast<uint4*>(ds_tile + kr * 128 + ((unit ^ (kr & 7)) << 4));
          *dst = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        }
        tmem_st_wait();
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->ds_ready[g]);
      }
      if (!ok) break;
      // ---------------------------------------------------------- item epilogue
      // groups 0, 1: dV columns [32g, 32g+32); groups 2, 3: dK columns [32(g-2), ...)
      if (!(ok = mbar_wait(&bars->acc_done, ic & 1, wc))) break;
      tc_fence_after();
      const bool is_k = g >= 2;
      const int c0 = 32 * (g & 1);
      uint32_t v[32];
      tmem_ld32(tmem + lane_off + (is_k ? T_DK : T_DV) + c0, v);
      tmem_ld_wait();
      tc_fence_before();  // the next item's first dV / dK MMAs follow this warp's next p_ready
      if (kvalid) {
        const float mul = is_k ? args.scale : 1.f;
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(is_k ? args.dK : args.dV) +
                             ((size_t)I.b * args.S + key) * (is_k ? args.lddk : args.lddv) + (size_t)I.h * args.D;
        if (c0 + 32 <= args.D) {
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            uint4 wv;
            wv.x = pack_bf16x2(__uint_as_float(v[c + 0]) * mul, __uint_as_float(v[c + 1]) * mul);
            wv.y = pack_bf16x2(__uint_as_float(v[c + 2]) * mul, __uint_as_float(v[c + 3]) * mul);
            wv.z = pack_bf16x2(__uint_as_float(v[c + 4]) * mul, __uint_as_float(v[c + 5]) * mul);
            wv.w = pack_bf16x2(__uint_as_float(v[c + 6]) * mul, __uint_as_float(v[c + 7]) * mul);
            *reinterpret_cast<uint4*>(dst + c0 + c) = wv;
          }
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if (c0 + c < args.D) dst[c0 + c] = __float2bfloat16_rn(__uint_as_float(v[c]) * mul);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == W_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// D_i = dO_i . O_i (fp32), L2_i = LSE_i * log2(e) in the padded [BH][Spad]
// layout (rows past S: D = 0, L2 = +inf so that exp2(s - L2) = 0). Eight
// lanes per row, 16-byte loads when D % 8 == 0.
//
// With zero_acc it first zeroes the fp32 dQ accumulator. In the fused
// backward with a caller-provided workspace it is launched as a programmatic
// dependent of the kernel before it (typically the forward, which lets its
// dependents start at once): the zeroing reads nothing that kernel writes,
// so it runs before the wait and overlaps that kernel's tail. No kernel of
// the library that starts its dependents early uses such a workspace (the
// int8 kernels, which do, use the library's own scratch, so a backward on
// library scratch is launched in stream order).
__global__ void flash_bwd_pre_kernel(FlashBwdArgs a) {
  // The main kernel may be scheduled now; it waits for this grid's results.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (a.zero_acc) {  // fresh fp32 dQ accumulator [BH][S][D] for the bulk reduce-adds
    const long long n = (long long)a.BH * a.S * a.D;
    const long long stride = (long long)gridDim.x * blockDim.x;
    long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (((uintptr_t)a.dq_acc & 15) == 0) {
      for (; i < n / 4; i += stride) reinterpret_cast<float4*>(a.dq_acc)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      i = n / 4 * 4 + blockIdx.x * (long long)blockDim.x + threadIdx.x;
    }
    for (; i < n; i += stride) a.dq_acc[i] = 0.f;
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");  // O, dO and LSE come from the kernels before
  const long long rows = (long long)a.BH * a.Spad;
  const int sub = threadIdx.x & 7;
  const long long groups = (long long)gridDim.x * (blockDim.x >> 3);
  const bool vec = (a.D % 8) == 0;
  for (long long r = blockIdx.x * (long long)(blockDim.x >> 3) + (threadIdx.x >> 3); r < rows; r += groups) {
    const int bh = (int)(r / a.Spad), q = (int)(r % a.Spad);
    float s = 0.f;
    if (q < a.S) {
      const int b = bh / a.H, h = bh - b * a.H;
      const long long row = (long long)b * a.S + q;
      const __nv_bfloat16* o = reinterpret_cast<const __nv_bfloat16*>(a.O) + row * a.ldo + (long long)h * a.D;
      const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(a.dO) + row * a.lddo + (long long)h * a.D;
      if (vec) {
        for (int c = sub * 8; c < a.D; c += 64) {
          const uint4 ov = *reinterpret_cast<const uint4*>(o + c), gv = *reinterpret_cast<const uint4*>(g + c);
          const __nv_bfloat162* op = reinterpret_cast<const __nv_bfloat162*>(&ov);
          const __nv_bfloat162* gp = reinterpret_cast<const __nv_bfloat162*>(&gv);
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const float2 x = __bfloat1622float2(op[h]), y = __bfloat1622float2(gp[h]);
            s = fmaf(x.x, y.x, fmaf(x.y, y.y, s));
          }
        }
      } else {
        for (int c = sub; c < a.D; c += 8) s = fmaf(__bfloat162float(o[c]), __bfloat162float(g[c]), s);
      }
    }
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    if (sub == 0) {
      a.rowstat[r] = q < a.S ? s : 0.f;
      a.rowstat[rows + r] = q < a.S ? a.lse[(long long)bh * a.S + q] * 1.4426950408889634f : INFINITY;
    }
  }
}

// dQ = bf16(scale * dQ_acc), four elements per thread step. Launched as a
// programmatic dependent of the main kernel: it starts on SMs the main
// kernel has left and waits here for that grid to finish.
// It does not let its own dependents start early: the next backward's row
// pre-pass zeroes the accumulator this kernel reads before that pre-pass
// waits for it.
__global__ void flash_bwd_post_kernel(FlashBwdArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const long long total = (long long)a.BH * a.S * a.D;
  const long long quads = total / 4;
  __nv_bfloat16* dq = reinterpret_cast<__nv_bfloat16*>(a.dQ);
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < quads; i += stride) {
    const float4 v = reinterpret_cast<const float4*>(a.dq_acc)[i];
    uint2 w;
    w.x = pack_bf16x2(v.x * a.scale, v.y * a.scale);
    w.y = pack_bf16x2(v.z * a.scale, v.w * a.scale);
    reinterpret_cast<uint2*>(dq)[i] = w;
  }
  for (long long i = quads * 4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += stride)
    dq[i] = __float2bfloat16_rn(a.dq_acc[i] * a.scale);
}

// The same for dQ in a head layout other than [BH][S][D]: quad c4 of row
// (bh, s) goes to dQ + (b*S + s)*lddq + h*D + 4*c4 (D % 4 == 0 and
// BH*S*D < 2^31, both checked by the caller).
__global__ void flash_bwd_post_rows_kernel(FlashBwdArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int qpr = a.D >> 2;
  const int quads = a.BH * a.S * qpr;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < quads; i += gridDim.x * blockDim.x) {
    const int row = i / qpr, c = (i - row * qpr) << 2;
    const int bh = row / a.S, s = row - bh * a.S;
    const int b = bh / a.H, h = bh - b * a.H;
    const float4 v = reinterpret_cast<const float4*>(a.dq_acc)[i];
    uint2 w;
    w.x = pack_bf16x2(v.x * a.scale, v.y * a.scale);
    w.y = pack_bf16x2(v.z * a.scale, v.w * a.scale);
    *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(a.dQ) + ((size_t)b * a.S + s) * a.lddq +
                              (size_t)h * a.D + c) = w;
  }
}


// The dense [BH][S][D] view through a 3-D map (box 64 x 128 x 1).
bool make_map3(CUtensorMap* map, const void* base, int BH, int S, int D) {
  auto enc = get_tensor_map_encoder();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)BH};
  cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)S * D * 2};
  cuuint32_t box[3] = {DP, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

size_t flash_bwd_scratch_bytes(int BH, int S, int D) {
  return ((size_t)BH * S * D + 2 * (size_t)BH * flash_spad(S)) * sizeof(float);
}

cudaError_t flash_bwd_rowstats(const FlashBwdArgs& a, cudaStream_t s) {
  FlashBwdArgs pa = a;
  pa.zero_acc = 0;
  flash_bwd_pre_kernel<<<8 * num_sms(), 256, 0, s>>>(pa);
  return cudaGetLastError();
}

static std::atomic<int> g_flash_deterministic{0};
void flash_set_deterministic(bool on) { g_flash_deterministic.store(on ? 1 : 0); }
bool flash_deterministic() { return g_flash_deterministic.load() != 0; }

cudaError_t flash_bwd_tc(const FlashBwdArgs& a, cudaStream_t s) {
  if (a.D > DP || flash_deterministic()) return flash_bwd_split_tc(a, s);
  CUtensorMap mq{}, mk{}, mv{}, mdo{};
  FlashBwdArgs la = a;
  la.dense3d = a.H == 1 && a.ldq == a.D && a.ldk == a.D && a.ldv == a.D && a.lddo == a.D;
  if (la.dense3d) {
    if (!make_map3(&mq, a.Q, a.BH, a.S, a.D) || !make_map3(&mk, a.K, a.BH, a.S, a.D) ||
        !make_map3(&mv, a.V, a.BH, a.S, a.D) || !make_map3(&mdo, a.dO, a.BH, a.S, a.D))
      return cudaErrorInvalidValue;
  } else if (!make_head_map(&mq, a.Q, a.BH, a.H, a.S, a.D, a.ldq) ||
             !make_head_map(&mk, a.K, a.BH, a.H, a.S, a.D, a.ldk) ||
             !make_head_map(&mv, a.V, a.BH, a.H, a.S, a.D, a.ldv) ||
             !make_head_map(&mdo, a.dO, a.BH, a.H, a.S, a.D, a.lddo)) {
    return cudaErrorInvalidValue;
  }
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(flash_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  CUtensorMap mdq{};
  {
    // fp32 dQ accumulator [BH][S][D] for the bulk reduce: boxes of 128 rows x
    // 32 columns (128 bytes, 128B swizzle); rows past S and columns past D clip.
    auto enc = get_tensor_map_encoder();
    cuuint64_t dims[3] = {(cuuint64_t)a.D, (cuuint64_t)a.S, (cuuint64_t)a.BH};
    cuuint64_t strides[2] = {(cuuint64_t)a.D * 4, (cuuint64_t)a.S * a.D * 4};
    cuuint32_t box[3] = {32, 128, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    if (!enc || enc(&mdq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, a.dq_acc, dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  const int sms = num_sms();
  // Three launches chained by programmatic dependent launch: the row
  // pre-pass (which also zeroes the dQ accumulator), the main kernel, the
  // dQ conversion. Each dependent waits (griddepcontrol.wait) for its
  // predecessor's results; only its launch overlaps the predecessor's tail.
  FlashBwdArgs pa = a;
  pa.zero_acc = 1;
  cudaLaunchAttribute pdl[1];
  pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  pdl[0].val.programmaticStreamSerializationAllowed = 1;
  {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(8 * sms);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cfg.attrs = pdl;
    cfg.numAttrs = a.own_ws ? 1 : 0;
    const cudaError_t e0 = cudaLaunchKernelEx(&cfg, flash_bwd_pre_kernel, pa);
    if (e0 != cudaSuccess) return e0;
  }
  const int nkv = (a.S + BKV - 1) / BKV;
  cudaError_t e;
  {
    const int items = nkv * a.BH;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(items < sms ? items : sms);
    cfg.blockDim = dim3(NUM_THREADS);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cfg.stream = s;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    TimerScope timer(s);
    e = cudaLaunchKernelEx(&cfg, flash_bwd_kernel, mq, mk, mv, mdo, mdq, la);
    if (e != cudaSuccess) return e;
  }
  {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(4 * sms);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    const bool dense_dq = a.H == 1 && a.lddq == a.D;
    e = dense_dq ? cudaLaunchKernelEx(&cfg, flash_bwd_post_kernel, a)
                 : cudaLaunchKernelEx(&cfg, flash_bwd_post_rows_kernel, a);
    if (e != cudaSuccess) return e;
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// SIMT kernels (any D <= 256): the reference's recurrences in fp32, one
// thread per query row (forward, dQ) or key row (dK, dV).
// ---------------------------------------------------------------------------
namespace {
constexpr int SIMT_DMAX = 256;

__device__ __forceinline__ float bf(const void* p, size_t i) {
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

__global__ void flash_fwd_simt_kernel(FlashFwdArgs a) {
  const int bh = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.S) return;
  const size_t base = (size_t)bh * a.S * a.D;
  float acc[SIMT_DMAX];
  for (int d = 0; d < a.D; ++d) acc[d] = 0.f;
  float m = -INFINITY, l = 0.f;
  const int jend = a.causal ? i : a.S - 1;
  for (int jj = 0; jj <= jend; ++jj) {
    float s = 0.f;
    for (int d = 0; d < a.D; ++d) s = fmaf(bf(a.Q, base + (size_t)i * a.D + d), bf(a.K, base + (size_t)jj * a.D + d), s);
    s *= a.scale;
    const float mn = fmaxf(m, s), corr = __expf(m - mn), p = __expf(s - mn);
    l = l * corr + p;
    for (int d = 0; d < a.D; ++d) acc[d] = acc[d] * corr + p * bf(a.V, base + (size_t)jj * a.D + d);
    m = mn;
  }
  const float inv = 1.f / l;
  __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(a.O) + base + (size_t)i * a.D;
  for (int d = 0; d < a.D; ++d) o[d] = __float2bfloat16_rn(acc[d] * inv);
  if (a.lse) a.lse[(size_t)bh * a.S + i] = m + __logf(l);
}

// dQ_i = scale * sum_j dS_ij K_j  (thread per query row)
__global__ void flash_bwd_simt_dq_kernel(FlashBwdArgs a) {
  const int bh = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= a.S) return;
  const size_t base = (size_t)bh * a.S * a.D, r = (size_t)bh * a.S + i;
  const float lse = a.lse[r], Di = a.rowstat[(size_t)bh * a.Spad + i];
  float acc[SIMT_DMAX];
  for (int d = 0; d < a.D; ++d) acc[d] = 0.f;
  const int jend = a.causal ? i : a.S - 1;
  for (int jj = 0; jj <= jend; ++jj) {
    float s = 0.f, dp = 0.f;
    for (int d = 0; d < a.D; ++d) {
      s = fmaf(bf(a.Q, base + (size_t)i * a.D + d), bf(a.K, base + (size_t)jj * a.D + d), s);
      dp = fmaf(bf(a.dO, base + (size_t)i * a.D + d), bf(a.V, base + (size_t)jj * a.D + d), dp);
    }
    const float p = __expf(s * a.scale - lse), ds = p * (dp - Di);
    for (int d = 0; d < a.D; ++d) acc[d] = fmaf(ds, bf(a.K, base + (size_t)jj * a.D + d), acc[d]);
  }
  __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(a.dQ) + base + (size_t)i * a.D;
  for (int d = 0; d < a.D; ++d) o[d] = __float2bfloat16_rn(acc[d] * a.scale);
}

// dV_j = sum_i P_ij dO_i, dK_j = scale * sum_i dS_ij Q_i  (thread per key row)
__global__ void flash_bwd_simt_dkdv_kernel(FlashBwdArgs a) {
  const int bh = blockIdx.y;
  const int jj = blockIdx.x * blockDim.x + threadIdx.x;
  if (jj >= a.S) return;
  const size_t base = (size_t)bh * a.S * a.D;
  float dk[SIMT_DMAX], dv[SIMT_DMAX];
  for (int d = 0; d < a.D; ++d) dk[d] = dv[d] = 0.f;
  for (int i = a.causal ? jj : 0; i < a.S; ++i) {
    const size_t r = (size_t)bh * a.S + i;
    float s = 0.f, dp = 0.f;
    for (int d = 0; d < a.D; ++d) {
      s = fmaf(bf(a.Q, base + (size_t)i * a.D + d), bf(a.K, base + (size_t)jj * a.D + d), s);
      dp = fmaf(bf(a.dO, base + (size_t)i * a.D + d), bf(a.V, base + (size_t)jj * a.D + d), dp);
    }
    const float p = __expf(s * a.scale - a.lse[r]), ds = p * (dp - a.rowstat[(size_t)bh * a.Spad + i]);
    for (int d = 0; d < a.D; ++d) {
      dv[d] = fmaf(p, bf(a.dO, base + (size_t)i * a.D + d), dv[d]);
      dk[d] = fmaf(ds, bf(a.Q, base + (size_t)i * a.D + d), dk[d]);
    }
  }
  __nv_bfloat16* ok = reinterpret_cast<__nv_bfloat16*>(a.dK) + base + (size_t)jj * a.D;
  __nv_bfloat16* ov = reinterpret_cast<__nv_bfloat16*>(a.dV) + base + (size_t)jj * a.D;
  for (int d = 0; d < a.D; ++d) {
    ok[d] = __float2bfloat16_rn(dk[d] * a.scale);
    ov[d] = __float2bfloat16_rn(dv[d]);
  }
}
}  // namespace

cudaError_t flash_fwd_simt(const FlashFwdArgs& a, cudaStream_t s) {
  if (a.D > SIMT_DMAX) return cudaErrorInvalidValue;
  dim3 grid((a.S + 63) / 64, a.BH);
  flash_fwd_simt_kernel<<<grid, 64, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t flash_bwd_simt(const FlashBwdArgs& a, cudaStream_t s) {
  if (a.D > SIMT_DMAX) return cudaErrorInvalidValue;
  flash_bwd_pre_kernel<<<4 * num_sms(), 256, 0, s>>>(a);
  dim3 grid((a.S + 63) / 64, a.BH);
  flash_bwd_simt_dq_kernel<<<grid, 64, 0, s>>>(a);
  flash_bwd_simt_dkdv_kernel<<<grid, 64, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace dgx
