// Causal / full FlashAttention forward on sm_100a (tcgen05 + TMEM + TMA).
//
// Replaces dream_flash_attention (runtime/nn/training.inc:284-401): the same
// online-softmax recurrence (running max m, normaliser l, rescaled
// accumulator), restated for tensor cores. Layout [BH][S][D] bf16, heads
// folded into the batch as in the reference's `(B, S*dk)` tensors.
//
// A persistent grid (one CTA per SM) walks work items of 256 query rows,
// the heaviest (latest causal) blocks first; Q of the next item loads into a
// second buffer while the current one runs. An item is two 128-row tiles
// (A, B) that share every K/V tile load. Warps 0-3 run tile A's softmax, warps 4-7 tile B's, warp 8
// issues TMA loads, warps 9 and 10 issue tile A's and tile B's tcgen05.mma. TMEM holds S_A, S_B (128 fp32
// columns each), O_A, O_B (D fp32 columns each) and P_A, P_B (128 bf16 = 64
// columns each, the A operand of the P.V MMA read straight from TMEM). A
// softmax warpgroup frees its S buffer as soon as S is in registers, so the
// MMA warp computes S(j+1) = Q.K(j+1)^T while tile j's exponentials run.
//
// At head dim 64 the exponentials (MUFU, 16/clk/SM) cost more than the MMAs,
// so the two warpgroups take turns on them (A_j, B_j, A_j+1, ...): each
// group's TMEM traffic and waits overlap the other's exponential phase.
//
// O is rescaled lazily: a row keeps its stale max until the new max exceeds
// it by more than 8 (log2 units), so P stays <= 256 and the TMEM read-modify-
// write of O is rare. The final O/l and LSE use the max actually applied, so
// the result is exact up to rounding.
#include <math.h>

#include "common.h"
#include "flash.h"
#include "sm100.cuh"

namespace dgx {

namespace {

constexpr int BLOCK_M = 128;   // rows per Q tile
constexpr int BLOCK_N = 128;   // keys per K/V tile
constexpr int HALF_BYTES = 128 * 128;  // one 64-column (128-byte) SW128 sub-tile of 128 rows
constexpr int NUM_THREADS = 384;  // WG0: softmax A, WG1: softmax B, WG2: TMA warp, two MMA warps, 1 idle
// setmaxnreg split (per thread): 2 x 224 + 56 = 504 <= 3 x 168 (65536 / 384 rounded down to 8).
constexpr uint32_t REG_SOFTMAX = 224, REG_CTRL = 56;
constexpr float RESCALE_LOG2 = 8.0f;
// Exponential column after which a softmax group hands the MUFU turn over.
constexpr int TURN_AT = 80;

// Layout per head-dim class: DP = 64 (D <= 64) or 128 (64 < D <= 128), the
// head dim held in shared memory and TMEM (columns past D zero-filled).
//   DP = 64: a Q/K/V tile is one 16 KB SW128 tile; Q for the next item loads
//     into a second buffer; 3 K/V stages; TMEM S_A, S_B, O_A, O_B, P_A, P_B.
//   DP = 128: a tile is two 64-column SW128 halves (32 KB); one Q buffer and
//     2 K/V stages (192 KB in all); TMEM S_A, S_B (128 columns each) and
//     O_A, O_B (128 each) fill all 512 columns, so P(j) is written over the
//     first 64 columns of its S buffer, and the MMA warp issues S(j+1) into
//     that buffer only after PV(j) has read P(j).
template <int DP_>
struct FwdCfg {
  static constexpr int DP = DP_;
  static constexpr bool ALIAS = DP_ > 64;
  static constexpr int HALVES = DP_ / 64;
  static constexpr int TILE_BYTES = BLOCK_M * DP_ * 2;
  static constexpr int Q_BUFS = ALIAS ? 1 : 2;
  static constexpr int KV_STAGES = ALIAS ? 2 : 3;
  // shared memory map (offsets from a 1024-aligned base)
  static constexpr int SM_Q = 0;                                 // Q_A, Q_B per Q buffer
  static constexpr int SM_K = SM_Q + Q_BUFS * 2 * TILE_BYTES;    // K stages
  static constexpr int SM_V = SM_K + KV_STAGES * TILE_BYTES;     // V stages
  static constexpr int SM_BAR = SM_V + KV_STAGES * TILE_BYTES;
  static constexpr int SMEM_BYTES = SM_BAR + 256 + 1024;
  // TMEM columns
  static constexpr uint32_t T_S0 = 0, T_S1 = 128, T_O0 = 256, T_O1 = 256 + DP_;
  static constexpr uint32_t T_P0 = ALIAS ? T_S0 : 384, T_P1 = ALIAS ? T_S1 : 448;
};
constexpr int MAX_KV_STAGES = 3;
constexpr uint32_t TMEM_COLS = 512;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for two softmax arguments (x <= ~8) on the FMA/ALU pipes instead of
// MUFU: x = j + f with j the nearest integer (adding 1.5 * 2^23 leaves j in
// the low mantissa bits) and f in [-1/2, 1/2]; 2^f from a degree-3
// polynomial whose coefficients were fitted for this file by iteratively
// reweighted least squares on Chebyshev nodes (maximum relative error
// 7.5e-5, far below the 3.9e-3 resolution of the bf16 P it feeds); j is added
// into the exponent field. x is clamped at -126, so a masked score (-inf)
// gives 2^-126 instead of 0: that P adds ~1e-38 to its row sum and ~1e-38 * V
// to O, below the resolution of any result.
__device__ __forceinline__ float2 ex2_poly2(float x0, float x1) {
  x0 = fmaxf(x0, -126.0f);
  x1 = fmaxf(x1, -126.0f);
  const float2 t = fadd2(make_float2(x0, x1), 12582912.0f, 12582912.0f);
  const float2 j = fadd2(t, -12582912.0f, -12582912.0f);
  const float2 f = fadd2(make_float2(x0, x1), -j.x, -j.y);
  float2 p = ffma2(f.x, f.y, 0.05517166f, 0.24261113f, 0.24261113f);
  p = make_float2(fmaf(p.x, f.x, 0.69326097f), fmaf(p.y, f.y, 0.69326097f));
  p = make_float2(fmaf(p.x, f.x, 0.99992806f), fmaf(p.y, f.y, 0.99992806f));
  return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}
// Column pairs (of every 8) whose exponentials take the polynomial at
// DP = 64, where MUFU sets the pace: measured 122.6 -> 119.5 us at config 2
// with 2 of 8 (more pairs were slower: 3 even, 4 much slower).
constexpr int POLY_PAIRS_DP64 = 2;

struct FwdBars {
  uint64_t q_full[2], q_empty[2], k_full[MAX_KV_STAGES], v_full[MAX_KV_STAGES], kv_empty[MAX_KV_STAGES];
  uint64_t s_full[2], s_free[2], p_full[2], pv_done[2], turn[2];
  uint32_t tmem_slot;
  int abort;
};

// Work item w (heavy = late query blocks first under causal): its two 128-row
// Q tiles, head, and how many K/V tiles each tile sees.
struct FwdItem {
  int q0, bh, nA, nB;
  int b, h;  // bh = b*H + h
};
__device__ __forceinline__ FwdItem fwd_item(const FlashFwdArgs& a, int w) {
  FwdItem I;
  const int nqb = (a.S + 2 * BLOCK_M - 1) / (2 * BLOCK_M);
  const int qb = a.causal ? (nqb - 1 - w / a.BH) : (w / a.BH);
  I.bh = w % a.BH;
  I.b = I.bh / a.H;
  I.h = I.bh - I.b * a.H;
  I.q0 = qb * 2 * BLOCK_M;
  const int nkv = (a.S + BLOCK_N - 1) / BLOCK_N;
  int nt[2];
  for (int x = 0; x < 2; ++x) {
    const int qs = I.q0 + x * BLOCK_M;
    const int qe = min(qs + BLOCK_M, a.S);  // exclusive
    nt[x] = a.causal ? min((qe + BLOCK_N - 1) / BLOCK_N, nkv) : nkv;
  }
  if (I.q0 + BLOCK_M >= a.S) nt[1] = nt[0];  // tile B has no valid rows: shadow A
  I.nA = nt[0];
  I.nB = nt[1];
  return I;
}

template <int DP>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, FlashFwdArgs args) {
  using Cfg = FwdCfg<DP>;
  constexpr int TILE_BYTES = Cfg::TILE_BYTES, KV_STAGES = Cfg::KV_STAGES, Q_BUFS = Cfg::Q_BUFS;
  constexpr int SM_Q = Cfg::SM_Q, SM_K = Cfg::SM_K, SM_V = Cfg::SM_V, SM_BAR = Cfg::SM_BAR;
  constexpr uint32_t T_S0 = Cfg::T_S0, T_S1 = Cfg::T_S1, T_O0 = Cfg::T_O0, T_O1 = Cfg::T_O1, T_P0 = Cfg::T_P0,
                     T_P1 = Cfg::T_P1;
  // A programmatic dependent launched after this grid (the backward's row
  // pre-pass, which zeroes its accumulator before it waits for this grid's
  // results) may be scheduled now.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  FwdBars* bars = reinterpret_cast<FwdBars*>(smem + SM_BAR);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  WaitCtx wc{&bars->abort, args.err};
  // Persistent: this CTA walks the items snake_item(0), snake_item(1), ...;
  // every barrier phase counts on across items.
  const int nitems = ((args.S + 2 * BLOCK_M - 1) / (2 * BLOCK_M)) * args.BH;

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->q_full[b], 1);
      mbar_init(&bars->q_empty[b], 2);
    }
    for (int s = 0; s < KV_STAGES; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->kv_empty[s], 2);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&bars->s_full[x], 1);
      mbar_init(&bars->s_free[x], 4);
      mbar_init(&bars->p_full[x], 4);
      mbar_init(&bars->pv_done[x], 1);
      mbar_init(&bars->turn[x], 4);
    }
    bars->abort = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(&bars->tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_slot;

  // Each role's setmaxnreg sits inside its branch so that it dominates (and
  // sets the register limit for) exactly that role's code.
  if (warp >= 8) {
   regs_dec<REG_CTRL>();
   if (warp == 8) {
    // ---------------------------------------------------------------- TMA
    if (elect_one_lane()) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      uint32_t gkv = 0, ic = 0;
      bool ok = true;
      // A tile is HALVES boxes of 64 columns, one per SW128 half.
      auto load_tile = [&](uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int row, const FwdItem& I) {
#pragma unroll
        for (int hf = 0; hf < Cfg::HALVES; ++hf) tma_load_4d(dst + hf * HALF_BYTES, map, bar, hf * 64, I.h, row, I.b);
      };
      for (int rnd = 0, w = snake_item(0); ok && w < nitems; w = snake_item(++rnd)) {
        const FwdItem I = fwd_item(args, w);
        const int qb = ic % Q_BUFS;
        if (!(ok = mbar_wait(&bars->q_empty[qb], ((ic / Q_BUFS) & 1) ^ 1, wc))) break;
        mbar_arrive_expect_tx(&bars->q_full[qb], 2 * TILE_BYTES);
        uint8_t* sq = smem + SM_Q + qb * 2 * TILE_BYTES;
        load_tile(sq, &tmQ, &bars->q_full[qb], I.q0, I);
        load_tile(sq + TILE_BYTES, &tmQ, &bars->q_full[qb], I.q0 + BLOCK_M, I);
        ++ic;  // counted as issued before any later wait can fail
        for (int j = 0; j < I.nB; ++j, ++gkv) {
          const int s = gkv % KV_STAGES;
          if (!(ok = mbar_wait(&bars->kv_empty[s], ((gkv / KV_STAGES) & 1) ^ 1, wc))) break;
          mbar_arrive_expect_tx(&bars->k_full[s], TILE_BYTES);
          load_tile(smem + SM_K + s * TILE_BYTES, &tmK, &bars->k_full[s], j * BLOCK_N, I);
          mbar_arrive_expect_tx(&bars->v_full[s], TILE_BYTES);
          load_tile(smem + SM_V + s * TILE_BYTES, &tmV, &bars->v_full[s], j * BLOCK_N, I);
        }
      }
      // Teardown: every copy issued must have landed before the CTA leaves.
      for (uint32_t f = ic > (uint32_t)Q_BUFS ? ic - Q_BUFS : 0; f < ic; ++f)
        mbar_drain(&bars->q_full[f % Q_BUFS], (f / Q_BUFS) & 1);
      for (uint32_t f = gkv > KV_STAGES ? gkv - KV_STAGES : 0; f < gkv; ++f) {
        mbar_drain(&bars->k_full[f % KV_STAGES], (f / KV_STAGES) & 1);
        mbar_drain(&bars->v_full[f % KV_STAGES], (f / KV_STAGES) & 1);
      }
    }
  } else if (warp == 9 || warp == 10) {
    // ---------------------------------------------------------------- MMA
    // One issuing warp per Q tile (warp 9: A, warp 10: B), so each tile's
    // S -> softmax -> P -> PV chain runs at its own pace and neither waits
    // behind the other's MMAs in one issue order. Each warp's commits cover
    // its own MMAs: a K/V stage and a Q buffer are free once both warps
    // have committed (barriers of count 2).
    if (elect_one_lane()) {
      const int x = warp - 9;
      constexpr uint32_t idesc_s = make_idesc(1, 0, 0, BLOCK_M, BLOCK_N);  // Q.K^T, both K-major
      constexpr uint32_t idesc_o = make_idesc(1, 0, 1, BLOCK_M, DP);       // P (TMEM) . V (MN-major)
      const uint32_t sk = smem_u32(smem + SM_K), sv = smem_u32(smem + SM_V);
      const uint32_t t_sx = tmem + (x ? T_S1 : T_S0), t_ox = tmem + (x ? T_O1 : T_O0), t_px = tmem + (x ? T_P1 : T_P0);
      uint32_t ns = 0, np = 0;  // S and PV tiles issued by this warp
      uint32_t gkv = 0, ic = 0;  // K/V tiles and items walked
      bool ok = true;
      // Descriptors advance by adding (byte offset >> 4) to the start field;
      // at DP = 128 the contraction over D crosses into the second SW128 half
      // after four K steps, and V's two 64-column halves are the B operand's
      // two 128-byte atoms along N (leading byte offset = one half).
      auto issue_s = [&](uint32_t sq, uint32_t kvi) {
        const uint64_t dq = sw128_desc(sq + x * TILE_BYTES, 16, 1024);
        const uint64_t dk = sw128_desc(sk + (kvi % KV_STAGES) * TILE_BYTES, 16, 1024);
#pragma unroll 1
        for (int kk = 0; kk < DP / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (HALF_BYTES >> 4) + (kk & 3) * 2;
          mma_f16_ss(t_sx, dq + off, dk + off, idesc_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(&bars->s_full[x]);
        ++ns;
      };
      auto issue_pv = [&](uint32_t kvi, bool first) {
        const uint64_t dv = sw128_desc(sv + (kvi % KV_STAGES) * TILE_BYTES, HALF_BYTES, 1024);
#pragma unroll 1
        for (int kk = 0; kk < BLOCK_N / 16; ++kk)  // 16 keys = 8 packed bf16 columns per step
          mma_f16_ts(t_ox, t_px + kk * 8, dv + 128 * kk, idesc_o, (!first || kk > 0) ? 1u : 0u);
        tc_commit(&bars->pv_done[x]);
        ++np;
      };
      // The S buffer is free once the softmax has read the previous S
      // (DP = 64) or once the previous PV has read the P written over it
      // (DP = 128).
      auto s_ready = [&]() {
        if constexpr (Cfg::ALIAS) return np == 0 || mbar_wait(&bars->pv_done[x], (np - 1) & 1, wc);
        return ns == 0 || mbar_wait(&bars->s_free[x], (ns - 1) & 1, wc);
      };
      for (int rnd = 0, w = snake_item(0); ok && w < nitems; w = snake_item(++rnd), ++ic) {
        const FwdItem I = fwd_item(args, w);
        const int qb = ic % Q_BUFS;
        const int n = x ? I.nB : I.nA;
        const uint32_t sq = smem_u32(smem + SM_Q + qb * 2 * TILE_BYTES);
        if (!(ok = mbar_wait(&bars->q_full[qb], (ic / Q_BUFS) & 1, wc))) break;
        if (n > 0) {
          if (!(ok = mbar_wait(&bars->k_full[gkv % KV_STAGES], (gkv / KV_STAGES) & 1, wc) && s_ready())) break;
          tc_fence_after();
          issue_s(sq, gkv);
        }
        for (int j = 0; ok && j < n; ++j) {
          const uint32_t kvi = gkv + j;
          const bool more = j + 1 < n;
          // DP = 64: S(j+1) goes ahead of PV(j), into the other half of the
          // overlap; DP = 128: after PV(j), which must read P(j) first.
          if (!Cfg::ALIAS && more) {
            if (!(ok = mbar_wait(&bars->k_full[(kvi + 1) % KV_STAGES], ((kvi + 1) / KV_STAGES) & 1, wc) &&
                       s_ready()))
              break;
            tc_fence_after();
            issue_s(sq, kvi + 1);
          }
          if (!(ok = mbar_wait(&bars->v_full[kvi % KV_STAGES], (kvi / KV_STAGES) & 1, wc) &&
                     mbar_wait(&bars->p_full[x], np & 1, wc)))
            break;
          tc_fence_after();
          issue_pv(kvi, j == 0);
          tc_commit(&bars->kv_empty[kvi % KV_STAGES]);
          if (Cfg::ALIAS && more) {
            if (!(ok = mbar_wait(&bars->k_full[(kvi + 1) % KV_STAGES], ((kvi + 1) / KV_STAGES) & 1, wc) &&
                       s_ready()))
              break;
            tc_fence_after();
            issue_s(sq, kvi + 1);
          }
        }
        if (!ok) break;
        // K/V tiles this tile does not see (tile A under causal: the last one)
        // still need this warp's arrival; their load having landed means the
        // stage's previous use is released, so the arrival counts for this use.
        for (int j = n; ok && j < I.nB; ++j) {
          const uint32_t kvi = gkv + j;
          if (!(ok = mbar_wait(&bars->k_full[kvi % KV_STAGES], (kvi / KV_STAGES) & 1, wc))) break;
          tc_commit(&bars->kv_empty[kvi % KV_STAGES]);
        }
        tc_commit(&bars->q_empty[qb]);  // every S of this item has read Q
        gkv += I.nB;
      }
    }
    __syncwarp();
   }
  } else {
    regs_inc<REG_SOFTMAX>();
    // ---------------------------------------------------------------- softmax (warps 0-3: A, 4-7: B)
    const int x = warp >> 2;
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    const uint32_t t_s = tmem + lane_off + (x ? T_S1 : T_S0);
    const uint32_t t_o = tmem + lane_off + (x ? T_O1 : T_O0);
    const float sl2 = args.scale * 1.4426950408889634f;  // scores -> log2 units
    const uint32_t t_p = tmem + lane_off + (x ? T_P1 : T_P0);
    // Phases consumed so far across items: S / PV tiles of this group, and
    // completions of the turn barrier this group waits on (A: turn[0], which
    // completes nA-1 times per item; B: turn[1], nA times per item).
    uint32_t kbase = 0, tbase = 0;
    bool ok = true;
    for (int rnd = 0, w = snake_item(0); ok && w < nitems; w = snake_item(++rnd)) {
      const FwdItem I = fwd_item(args, w);
      const int n = x ? I.nB : I.nA;
      const int qrow = I.q0 + x * BLOCK_M + r;
      const int row_base = I.bh * args.S;  // row of the [BH*S] LSE view
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; j < n; ++j) {
        const uint32_t k = kbase + j;
        if (!(ok = mbar_wait(&bars->s_full[x], k & 1, wc))) break;
        tc_fence_after();
        float s[BLOCK_N];
#pragma unroll
        for (int c = 0; c < BLOCK_N; c += 32) tmem_ld32(t_s + c, *reinterpret_cast<uint32_t(*)[32]>(&s[c]));
        tmem_ld_wait();
        // S is in registers: let the MMA warp compute the next S into this buffer.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->s_free[x]);
        const int k0 = j * BLOCK_N;
        const bool need_mask = (args.causal && k0 + BLOCK_N - 1 > I.q0 + x * BLOCK_M) || (k0 + BLOCK_N > args.S);
        if (need_mask) {
          const int lim = (args.causal ? min(qrow, args.S - 1) : args.S - 1) - k0;  // last visible column
#pragma unroll
          for (int c = 0; c < BLOCK_N; ++c) s[c] = (c <= lim) ? s[c] : -INFINITY;
        }
        // Row max of the raw scores with 8 independent partial maxima (short
        // dependency chains, two new columns per three-input max); scale > 0,
        // so max(s)*sl2 = max(s*sl2).
        float pm[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) pm[i] = s[i];
#pragma unroll
        for (int c = 8; c < BLOCK_N; c += 2) pm[(c >> 1) & 7] = max3f(pm[(c >> 1) & 7], s[c], s[c + 1]);
        const float mt = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                               fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7]))) * sl2;
        // lazy rescale
        float factor = 1.f;
        if (mt > m_run + RESCALE_LOG2 || m_run == -INFINITY) {
          factor = (m_run == -INFINITY) ? 0.f : ex2(m_run - mt);
          m_run = mt;
        }
        const float nmb = (m_run == -INFINITY) ? 0.f : -m_run;
        // Exponential phase turn: A_j waits for B_(j-1), B_j waits for A_j.
        if (x == 0 ? j > 0 : j < I.nA) {
          if (!(ok = mbar_wait(&bars->turn[x], (x == 0 ? tbase + j - 1 : tbase + j) & 1, wc))) break;
        }
        // Column pairs go through the packed fp32 forms: one FMA-pipe
        // instruction scales two scores, one adds two exponentials into the
        // row sum's four partial pairs.
        float2 ps[4] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};
        uint32_t p[BLOCK_N / 2];
        auto step = [&](auto cc) {
          constexpr int c = decltype(cc)::value;
          const float2 a = ffma2(s[c], s[c + 1], sl2, nmb);
          float e0, e1;
          if constexpr (DP == 64 && ((c >> 1) & 7) < POLY_PAIRS_DP64) {
            const float2 e = ex2_poly2(a.x, a.y);
            e0 = e.x;
            e1 = e.y;
          } else {
            e0 = ex2(a.x);
            e1 = ex2(a.y);
          }
          ps[(c >> 1) & 3] = fadd2(ps[(c >> 1) & 3], e0, e1);
          p[c / 2] = pack_bf16x2(e0, e1);
        };
        // Hand the turn to the other group (B only while A has tiles left)
        // before the last columns: the other group's wait ends while these
        // exponentials still keep MUFU busy, so the barrier's hand-off
        // latency does not leave it idle.
        static_for<0, TURN_AT, 2>(step);
        __syncwarp();
        if (lane == 0 && (x == 0 || j + 1 < I.nA)) mbar_arrive(&bars->turn[x ^ 1]);
        static_for<TURN_AT, BLOCK_N, 2>(step);
        const float rs = ((ps[0].x + ps[0].y) + (ps[1].x + ps[1].y)) + ((ps[2].x + ps[2].y) + (ps[3].x + ps[3].y));
        l_run = l_run * factor + rs;
        if (j > 0) {
          // PV(j-1) must be done: it reads the P buffer and accumulates O.
          if (!(ok = mbar_wait(&bars->pv_done[x], (k - 1) & 1, wc))) break;
          tc_fence_after();
          if (__any_sync(0xffffffffu, factor != 1.f)) {
            uint32_t o[32];
#pragma unroll
            for (int c = 0; c < DP; c += 32) {
              tmem_ld32(t_o + c, o);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
              tmem_st16(t_o + c, *reinterpret_cast<uint32_t(*)[16]>(&o[0]));
              tmem_st16(t_o + c + 16, *reinterpret_cast<uint32_t(*)[16]>(&o[16]));
            }
            tmem_st_wait();
          }
        }
        // P(j) overwrites P(j-1), which PV(j-1) (waited for above, or of the
        // previous item, which the epilogue waited for) has read.
#pragma unroll
        for (int c = 0; c < BLOCK_N / 2; c += 16) tmem_st16(t_p + c, *reinterpret_cast<uint32_t(*)[16]>(&p[c]));
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->p_full[x]);
      }
      if (!ok) break;
      // ------------------------------------------------------------ item epilogue
      // The next item's first PV overwrites O: it follows this warp's next
      // p_full arrival, which comes after these loads.
      if (n > 0) {
        if (!(ok = mbar_wait(&bars->pv_done[x], (kbase + n - 1) & 1, wc))) break;
        tc_fence_after();
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(args.O) +
                              ((size_t)I.b * args.S + qrow) * args.ldo + (size_t)I.h * args.D;
        // 64 columns of O at a time (all the rows of the tile load together;
        // rows past S only skip the stores).
#pragma unroll
        for (int c0 = 0; c0 < DP; c0 += 64) {
          uint32_t o[64];
          tmem_ld32(t_o + c0, *reinterpret_cast<uint32_t(*)[32]>(&o[0]));
          tmem_ld32(t_o + c0 + 32, *reinterpret_cast<uint32_t(*)[32]>(&o[32]));
          tmem_ld_wait();
          if (qrow < args.S) {
            if (c0 + 64 <= args.D) {
#pragma unroll
              for (int c = 0; c < 64; c += 8) {
                uint4 wv;
                wv.x = pack_bf16x2(__uint_as_float(o[c + 0]) * inv, __uint_as_float(o[c + 1]) * inv);
                wv.y = pack_bf16x2(__uint_as_float(o[c + 2]) * inv, __uint_as_float(o[c + 3]) * inv);
                wv.z = pack_bf16x2(__uint_as_float(o[c + 4]) * inv, __uint_as_float(o[c + 5]) * inv);
                wv.w = pack_bf16x2(__uint_as_float(o[c + 6]) * inv, __uint_as_float(o[c + 7]) * inv);
                *reinterpret_cast<uint4*>(orow + c0 + c) = wv;
              }
            } else {
#pragma unroll
              for (int c = 0; c < 64; ++c)
                if (c0 + c < args.D) orow[c0 + c] = __float2bfloat16_rn(__uint_as_float(o[c]) * inv);
            }
          }
        }
        tc_fence_before();
        if (qrow < args.S && args.lse)
          args.lse[(size_t)row_base + qrow] = (m_run + __log2f(l_run)) * 0.6931471805599453f;
      }
      kbase += n;
      tbase += x == 0 ? (I.nA - 1) : I.nA;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace

// 4-D view [B][S][H][D] of a bf16 head tensor (row pitch ld elements; H = 1,
// ld = D is the dense [BH][S][D] layout): a box of 64 columns x 1 head x 128
// rows never crosses a head; rows past S and columns past D read as zero.
bool make_head_map(CUtensorMap* map, const void* base, int BH, int H, int S, int D, int ld) {
  auto enc = get_tensor_map_encoder();
  if (!enc || H <= 0 || BH % H) return false;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)S, (cuuint64_t)(BH / H)};
  cuuint64_t strides[3] = {(cuuint64_t)D * 2, (cuuint64_t)ld * 2, (cuuint64_t)S * ld * 2};
  cuuint32_t box[4] = {64, 1, 128, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool flash_tc_supported(int D, int max_d, const void* const* ptrs, int n) {
  if (D < 8 || D > max_d || D % 8) return false;
  for (int i = 0; i < n; ++i)
    if (reinterpret_cast<uintptr_t>(ptrs[i]) & 15) return false;
  return true;
}

namespace {
template <int DP>
cudaError_t launch_fwd(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const FlashFwdArgs& a,
                       cudaStream_t s) {
  constexpr int smem = FwdCfg<DP>::SMEM_BYTES;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(flash_fwd_kernel<DP>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const int nqb = (a.S + 2 * BLOCK_M - 1) / (2 * BLOCK_M);
  const int items = nqb * a.BH;
  {
    TimerScope timer(s);
    flash_fwd_kernel<DP><<<items < num_sms() ? items : num_sms(), NUM_THREADS, smem, s>>>(mq, mk, mv, a);
  }
  return cudaGetLastError();
}
}  // namespace

cudaError_t flash_fwd_tc(const FlashFwdArgs& a, cudaStream_t s) {
  CUtensorMap mq{}, mk{}, mv{};
  if (!make_head_map(&mq, a.Q, a.BH, a.H, a.S, a.D, a.ldq) || !make_head_map(&mk, a.K, a.BH, a.H, a.S, a.D, a.ldk) ||
      !make_head_map(&mv, a.V, a.BH, a.H, a.S, a.D, a.ldv))
    return cudaErrorInvalidValue;
  if (a.D <= 64) return launch_fwd<64>(mq, mk, mv, a, s);
  if (a.D <= 128) return launch_fwd<128>(mq, mk, mv, a, s);
  return cudaErrorInvalidValue;
}

}  // namespace dgx
