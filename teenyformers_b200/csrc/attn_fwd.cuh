// attn_fwd.cuh -- flash-attention-2 forward for sm_100a (bf16 in, fp32 acc).
//
// Computes, per (batch, query head), O = softmax(mask(Q K^T * scale)) V and
// LSE = m + ln(l) (natural log of the scaled scores), the same quantities as
// teenyformers' flash_attn2_causal_fwd (src/kernels/flash_attn2.rs:77-125):
// top-left causal mask (key k is hidden from query q when k > q), and the
// non-causal variant without the mask.  GQA: query head h reads KV head
// h / (Hq / Hkv).
//
// Layout in HBM: Q, O [B*Hq, Sq, D]; K, V [B*Hkv, Sk, D]; LSE [B*Hq, Sq] fp32.
//
// Persistent (one CTA per SM); each work item is two 128-row query tiles of
// one head (rows q0..q0+255), walked over 128-row key/value tiles:
//   warp 9     TMA producer: Q once, then K_j / V_j into 2-stage rings
//   warp 8     MMA issuer (one thread): S_t = Q_t K_j^T  (SS, M=128 N=128),
//              O_t += P_t V_j (A = P from TMEM, B = V from SMEM, N = D)
//   warps 0-3  softmax for query tile 0, warps 4-7 for query tile 1: each
//              thread owns one query row = one TMEM lane
// The two tiles ping-pong: while one tile's softmax runs on the SFU/FMA
// pipes, the tensor core works on the other tile.  TMEM (512 columns):
//   S0 [0,128)  S1 [128,256)  O0 [256,256+D)  O1 [256+D, 256+2D)
// P_t (bf16 pairs) overwrites the first 64 columns of S_t; the next S_t MMA
// is issued after the P_t V_j MMA, and tcgen05 MMAs of one thread execute in
// issue order.  P_t is handed to the MMA issuer once, whole: handing it over
// in two 64-key halves (the first half of P_t V_j under the second half of
// the softmax) measured ~1.5 % slower, the extra hand-off costing the single
// issuing warp more than the overlap gained.  The issuing thread blocks
// while the tensor pipe's queue is full, so its bookkeeping (slot-release
// commits) is deferred until the next batch of MMAs is queued.  The running
// max is rescaled lazily: O and l are only rescaled when the row max grows
// by more than 2^8 (P stays <= 256).
// Every mbarrier wait is bounded (sm100.cuh); a timeout unwinds the CTA.
#pragma once

#include "sm100.cuh"

namespace tfb {

struct FwdParams {
  __nv_bfloat16* o;
  float* lse;
  int Sq, Sk;
  int Hq, Hkv;
  int BHq;
  int n_pairs;
  float scale_log2;  // softmax_scale * log2(e)
  int causal;
  int heavy_first;  // item order: all heads' heaviest pairs first (K/V fit in L2)
};

template <int D>
struct FwdCfg {
  static constexpr int kThreads = 320;
  static constexpr int BM = 128, BN = 128, KSTAGES = 2;
  static constexpr int HALVES = D / 64;                  // 128-byte swizzle atoms per row
  static constexpr int HALF_BYTES = 128 * 128;           // 128 rows x 128 bytes
  static constexpr int TILE_BYTES = 128 * D * 2;         // one 128-row bf16 tile
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + 2 * TILE_BYTES;
  static constexpr int OFF_V = OFF_K + KSTAGES * TILE_BYTES;
  // epilogue staging: per query tile one 128-row x 64-column bf16 half of O
  // (128-byte swizzle, the O map's box), written out by TMA stores
  static constexpr int OFF_STG = OFF_V + KSTAGES * TILE_BYTES;
  static constexpr int OFF_BAR = OFF_STG + 2 * HALF_BYTES;
  static constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;  // barriers + 1 KB align slack
  __device__ static constexpr uint32_t tm_s(int t) { return uint32_t(t) * 128u; }
  __device__ static constexpr uint32_t tm_o(int t) { return 256u + uint32_t(t) * D; }
  static constexpr uint32_t TM_COLS = 512;
};

enum FwdBar {
  FB_QFULL = 0,
  FB_KFULL = 1,   // 2
  FB_KEMPTY = 3,  // 2
  FB_VFULL = 5,   // 2
  FB_VEMPTY = 7,  // 2
  FB_SFULL = 9,   // 2
  FB_PFULL = 11,  // 2: P_t ready in TMEM
  FB_ODONE = 13,  // 2
  FB_DRAIN = 15,
  FB_QEMPTY = 16,  // every S MMA of the item is done: Q may be replaced
  FB_OFREE = 17,   // 2: the epilogue has read O_t out of TMEM
  FB_COUNT = 19
};

// Waits without looking at the abort flag (used to drain in-flight async
// work before the CTA exits); bounded by kWaitTimeoutNs.
__device__ __forceinline__ void mbar_drain_wait(uint32_t bar, uint32_t parity, int site) {
  (void)mbar_wait(bar, parity, nullptr, site);
}

// Work item w = query-tile pair of one head.  Default order: head-major (the
// CTAs running at any time share a few heads' K/V in L2), heavy (late) pairs
// first within a head when causal.  With heavy_first (causal, and all K/V
// small enough to stay in L2): pair-major from the heaviest pair down, so the
// boustrophedon rounds approximate longest-first scheduling.  Each role
// derives the same values from w.
struct FwdItem {
  int bh, bh_kv, q0, nkv0, nkv1, n_iter;
};
__device__ __forceinline__ FwdItem fwd_item(const FwdParams& p, int w) {
  FwdItem it;
  int pair;
  if (p.heavy_first) {
    pair = p.n_pairs - 1 - w / p.BHq;
    it.bh = w % p.BHq;
  } else {
    it.bh = w / p.n_pairs;
    pair = w % p.n_pairs;
    if (p.causal) pair = p.n_pairs - 1 - pair;
  }
  const int b = it.bh / p.Hq, h = it.bh % p.Hq;
  it.bh_kv = b * p.Hkv + h / (p.Hq / p.Hkv);
  it.q0 = pair * 256;
  const int n_kv_all = (p.Sk + 127) / 128;
  auto tile_kv = [&](int t) {  // key tiles query tile t needs (0 if it is past Sq)
    const int qs = it.q0 + 128 * t;
    if (qs >= p.Sq) return 0;
    if (!p.causal) return n_kv_all;
    return min(n_kv_all, (min(p.Sq, qs + 128) - 1) / 128 + 1);
  };
  it.nkv0 = tile_kv(0);
  it.nkv1 = tile_kv(1);
  it.n_iter = max(it.nkv0, it.nkv1);
  return it;
}

// Item of round k for this CTA: rounds alternate direction (boustrophedon), so
// heavy and light items spread over the CTAs; only the last round is partial.
__device__ __forceinline__ int fwd_sched(int k) {
  const int G = gridDim.x, c = blockIdx.x;
  return k * G + ((k & 1) ? G - 1 - c : c);
}

// Persistent: one CTA per SM walks work items (fwd_sched).  Per-step barriers
// (S/P per tile, K/V ring) run on counts that continue across items; per item,
// the next item's Q load starts once the last S MMA of the current item has
// run, and its first O_t = P_t V MMA waits until the epilogue has read O_t.
template <int D>
__global__ void __launch_bounds__(320, 1)
    fa_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                        const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v,
                        const __grid_constant__ CUtensorMap tm_o, const FwdParams p) {
  using C = FwdCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + FB_COUNT);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto bar = [&](int i) { return smem_u32(bars + i); };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = p.BHq * p.n_pairs;

  // ---- setup ----
  if (threadIdx.x == 0) {
    mbar_init(bar(FB_QFULL), 1);
    mbar_init(bar(FB_QEMPTY), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(FB_KFULL + s), 1);
      mbar_init(bar(FB_KEMPTY + s), 1);
      mbar_init(bar(FB_VFULL + s), 1);
      mbar_init(bar(FB_VEMPTY + s), 1);
      mbar_init(bar(FB_SFULL + s), 1);
      mbar_init(bar(FB_PFULL + s), 4);  // one arrival per softmax warp
      mbar_init(bar(FB_ODONE + s), 1);
      mbar_init(bar(FB_OFREE + s), 4);
    }
    mbar_init(bar(FB_DRAIN), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), C::TM_COLS);
    tmem_relinquish();
  }
  if (warp == 9 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 9) {
    // =================== TMA producer (whole warp, one elected lane issues) =====
    int issued_q = 0, issued_k[2] = {0, 0}, issued_v[2] = {0, 0}, gj = 0;
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int w = fwd_sched(k);
      if (w >= n_items) break;
      const FwdItem it = fwd_item(p, w);
      if (it.n_iter == 0) continue;
      if (issued_q > 0) ok = mbar_wait_warp(bar(FB_QEMPTY), (issued_q - 1) & 1, abort_flag, 104);
      if (!ok) break;
      if (elect_one()) {
        mbar_arrive_expect_tx(bar(FB_QFULL), 2 * C::TILE_BYTES);
        for (int t = 0; t < 2; ++t)
          for (int hh = 0; hh < C::HALVES; ++hh)
            tma_load_3d(sbase + C::OFF_Q + t * C::TILE_BYTES + hh * C::HALF_BYTES, &tm_q,
                        bar(FB_QFULL), hh * 64, it.q0 + 128 * t, it.bh);
      }
      __syncwarp();
      ++issued_q;
      for (int j = 0; j < it.n_iter && ok; ++j, ++gj) {
        const int s = gj & 1, u = gj >> 1;
        if (u > 0) ok = mbar_wait_warp(bar(FB_KEMPTY + s), (u - 1) & 1, abort_flag, 101);
        if (!ok) break;
        if (elect_one()) {
          mbar_arrive_expect_tx(bar(FB_KFULL + s), C::TILE_BYTES);
          for (int hh = 0; hh < C::HALVES; ++hh)
            tma_load_3d(sbase + C::OFF_K + s * C::TILE_BYTES + hh * C::HALF_BYTES, &tm_k,
                        bar(FB_KFULL + s), hh * 64, j * 128, it.bh_kv);
        }
        __syncwarp();
        issued_k[s] += 1;
        if (u > 0) ok = mbar_wait_warp(bar(FB_VEMPTY + s), (u - 1) & 1, abort_flag, 102);
        if (!ok) break;
        if (elect_one()) {
          mbar_arrive_expect_tx(bar(FB_VFULL + s), C::TILE_BYTES);
          for (int hh = 0; hh < C::HALVES; ++hh)
            tma_load_3d(sbase + C::OFF_V + s * C::TILE_BYTES + hh * C::HALF_BYTES, &tm_v,
                        bar(FB_VFULL + s), hh * 64, j * 128, it.bh_kv);
        }
        __syncwarp();
        issued_v[s] += 1;
      }
    }
    if (!ok) {
      // Abort: let every issued copy land before the CTA's smem goes away.
      if (issued_q) mbar_drain_wait(bar(FB_QFULL), (issued_q - 1) & 1, 103);
      for (int s = 0; s < 2; ++s) {
        if (issued_k[s]) mbar_drain_wait(bar(FB_KFULL + s), (issued_k[s] - 1) & 1, 103);
        if (issued_v[s]) mbar_drain_wait(bar(FB_VFULL + s), (issued_v[s] - 1) & 1, 103);
      }
    }
  } else if (warp == 8) {
    // =================== MMA issuer (whole warp, one elected lane issues) =======
    constexpr uint32_t idesc_qk = make_idesc_bf16(128, 128, 0, 0);
    constexpr uint32_t idesc_pv = make_idesc_bf16(128, D, 0, 1);
    // Descriptors are built once; each K step only advances the start
    // address by a compile-time constant.
    const uint64_t dq0 = make_sdesc_sw128(sbase + C::OFF_Q, 16, 1024);
    const uint64_t dq1 = desc_adv(dq0, C::TILE_BYTES);
    const uint64_t dk0 = make_sdesc_sw128(sbase + C::OFF_K, 16, 1024);
    const uint64_t dk1 = desc_adv(dk0, C::TILE_BYTES);
    const uint64_t dv0 = make_sdesc_sw128(sbase + C::OFF_V, C::HALF_BYTES, 1024);
    const uint64_t dv1 = desc_adv(dv0, C::TILE_BYTES);
    // S_t = Q_t K_slot^T, then signal s_full[t]
    auto issue_qk = [&](int t, int slot) {
      if (elect_one()) {
        const uint64_t a = t ? dq1 : dq0;
        const uint64_t bk = slot ? dk1 : dk0;
        const uint32_t d = tmem + C::tm_s(t);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          mma_ss(d, desc_adv(a, kstep_off(kk, C::HALF_BYTES)),
                 desc_adv(bk, kstep_off(kk, C::HALF_BYTES)), idesc_qk, kk > 0);
        tc_commit(bar(FB_SFULL + t));
      }
      __syncwarp();
    };
    // O_t += P_t V_j over keys [64*half, 64*half + 64) of the tile; then the
    // optional commits (a commit covers every MMA issued before it).
    auto issue_pv_half = [&](int t, int slot, int half, bool acc, int commit0, int commit1) {
      if (elect_one()) {
        const uint64_t bv = slot ? dv1 : dv0;
        const uint32_t d = tmem + C::tm_o(t);
        const uint32_t a = tmem + C::tm_s(t);
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          const int kk = 4 * half + k4;
          mma_ts(d, a + kk * 8, desc_adv(bv, kk * 16 * 128), idesc_pv,
                 (acc || kk > 0) ? 1u : 0u);
        }
        if (commit0 >= 0) tc_commit(bar(commit0));
        if (commit1 >= 0) tc_commit(bar(commit1));
      }
      __syncwarp();
    };
    auto commit = [&](int b0) {
      if (elect_one()) tc_commit(bar(b0));
      __syncwarp();
    };
    bool ok = true;
    // n_q: items with work so far (QFULL/QEMPTY phases); gj: K/V steps so far;
    // st_[t]: steps of query tile t so far (S/P phases); no_[t]: items in which
    // tile t had work (ODONE/OFREE phases)
    int n_q = 0, gj = 0, st_[2] = {0, 0}, no_[2] = {0, 0};
    for (int k = 0; ok; ++k) {
      const int w = fwd_sched(k);
      if (w >= n_items) break;
      const FwdItem it = fwd_item(p, w);
      if (it.n_iter == 0) continue;
      auto nkv = [&](int t) { return t ? it.nkv1 : it.nkv0; };
      ok = mbar_wait_warp(bar(FB_QFULL), n_q & 1, abort_flag, 201);
      if (ok) ok = mbar_wait_warp(bar(FB_KFULL + (gj & 1)), (gj >> 1) & 1, abort_flag, 202);
      if (!ok) break;
      tc_fence_after();
      for (int t = 0; t < 2; ++t)
        if (nkv(t) > 0) issue_qk(t, gj & 1);
      if (it.n_iter == 1) commit(FB_QEMPTY);  // that was the item's last S MMA
      commit(FB_KEMPTY + (gj & 1));
      // Slot-release commits of a step are issued once the next batch of MMAs
      // is queued.
      int pend_v = -1, pend_k = -1;
      for (int j = 0; j < it.n_iter && ok; ++j) {
        const int s = (gj + j) & 1;
        const int sn = (gj + j + 1) & 1;
        bool v_ready = false, k_next_ready = false;
        for (int t = 0; t < 2 && ok; ++t) {
          if (j >= nkv(t)) continue;
          if (!v_ready) {
            ok = mbar_wait_warp(bar(FB_VFULL + s), ((gj + j) >> 1) & 1, abort_flag, 203);
            if (!ok) break;
            v_ready = true;
          }
          if (j == 0 && no_[t] > 0) {  // the previous item's epilogue has read O_t
            ok = mbar_wait_warp(bar(FB_OFREE + t), (no_[t] - 1) & 1, abort_flag, 208);
            if (!ok) break;
          }
          const uint32_t ph = uint32_t(st_[t] + j) & 1u;
          ok = mbar_wait_warp(bar(FB_PFULL + t), ph, abort_flag, 204);
          if (!ok) break;
          tc_fence_after();
          issue_pv_half(t, s, 0, j > 0, pend_v >= 0 ? FB_VEMPTY + pend_v : -1,
                        pend_k >= 0 ? FB_KEMPTY + pend_k : -1);
          pend_v = pend_k = -1;
          const bool more = j + 1 < nkv(t);
          issue_pv_half(t, s, 1, true, more ? -1 : FB_ODONE + t, -1);
          if (more) {
            if (!k_next_ready) {
              ok = mbar_wait_warp(bar(FB_KFULL + sn), ((gj + j + 1) >> 1) & 1, abort_flag, 205);
              if (!ok) break;
              tc_fence_after();
              k_next_ready = true;
            }
            issue_qk(t, sn);
          }
        }
        if (!ok) break;
        pend_v = s;
        pend_k = (j + 1 < it.n_iter) ? sn : -1;
        if (j + 2 == it.n_iter) commit(FB_QEMPTY);  // the item's last S MMAs are queued
      }
      if (!ok) break;
      // release the item's last V slot before moving on
      if (pend_v >= 0) commit(FB_VEMPTY + pend_v);
      if (pend_k >= 0) commit(FB_KEMPTY + pend_k);
      gj += it.n_iter;
      ++n_q;
      for (int t = 0; t < 2; ++t) {
        st_[t] += nkv(t);
        if (nkv(t) > 0) ++no_[t];
      }
    }
    // Drain: every MMA issued above completes before TMEM is released.
    if (elect_one()) tc_commit(bar(FB_DRAIN));
    __syncwarp();
    mbar_drain_wait(bar(FB_DRAIN), 0, 206);
  } else {
    // =================== softmax: warps 0-3 tile 0, 4-7 tile 1 ===================
    const int t = warp >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_base = uint32_t(wq * 32) << 16;
    const uint32_t tS = tmem + lane_base + C::tm_s(t);
    const uint32_t tO = tmem + lane_base + C::tm_o(t);
    const float sl2 = p.scale_log2;
    const uint32_t stage = sbase + C::OFF_STG + t * C::HALF_BYTES;
    const uint32_t stage_row = stage + row * 128;
    const bool epi_issuer = wq == 0 && lane == 0;  // first thread of the tile's warpgroup
    bool ok = true;
    int st_t = 0, no_t = 0;  // this tile's steps / items with work so far
    for (int k = 0; ok; ++k) {
      const int w = fwd_sched(k);
      if (w >= n_items) break;
      const FwdItem it = fwd_item(p, w);
      const int nk = t ? it.nkv1 : it.nkv0;
      if (nk == 0) continue;
      const int qs = it.q0 + 128 * t;
      const int q_idx = qs + row;
      float m = -INFINITY, l = 0.0f;
      for (int j = 0; j < nk; ++j) {
        ok = mbar_wait(bar(FB_SFULL + t), uint32_t(st_t + j) & 1u, abort_flag, 300 + t);
        ok = __all_sync(0xffffffffu, ok);  // keep .sync.aligned TMEM ops convergent
        if (!ok) break;
        tc_fence_after();
        uint32_t sr[4][32];
  #pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, sr[c]);
        tmem_wait_ld();
        const int kbase = j * 128;
        const bool need_mask = (p.causal && kbase + 127 > qs) || (kbase + 128 > p.Sk);
        if (need_mask) {
          int lim = p.Sk - 1 - kbase;  // keys with index > lim are hidden
          if (p.causal) lim = min(lim, q_idx - kbase);
  #pragma unroll
          for (int c = 0; c < 4; ++c)
  #pragma unroll
            for (int i = 0; i < 32; ++i)
              if (c * 32 + i > lim) sr[c][i] = __float_as_uint(-INFINITY);
        }
        // row max: 3-input max, four independent chains
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  #pragma unroll
        for (int c = 0; c < 4; ++c)
  #pragma unroll
          for (int i = 0; i < 32; i += 2)
            mx[(i >> 1) & 3] = fmax3(mx[(i >> 1) & 3], __uint_as_float(sr[c][i]),
                                     __uint_as_float(sr[c][i + 1]));
        const float rmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
        const float m_new = fmaxf(m, rmax * sl2);
        const bool resc = m_new > m + 8.0f;
        const float m_use = resc ? m_new : m;
        const float alpha = resc ? ex2_approx(m - m_use) : 1.0f;
        const float base = (m_use == -INFINITY) ? 0.0f : m_use;
        const uint64_t sl2x2 = f2_make(sl2, sl2);
        const uint64_t nbx2 = f2_make(-base, -base);
        uint64_t acc2[2] = {f2_make(0.0f, 0.0f), f2_make(0.0f, 0.0f)};
        // P = 2^(s*scale*log2e - m) in bf16, written over the S columns already
        // read, 32 keys per store; handed to the MMA warp once complete.
  #pragma unroll
        for (int half = 0; half < 2; ++half) {
  #pragma unroll
          for (int c = 2 * half; c < 2 * half + 2; ++c) {
            uint32_t pk[16];
  #pragma unroll
            for (int i = 0; i < 16; ++i) {
              const uint64_t x2 = f2_fma(
                  f2_make(__uint_as_float(sr[c][2 * i]), __uint_as_float(sr[c][2 * i + 1])), sl2x2,
                  nbx2);
              float x0, x1;
              f2_split(x2, x0, x1);
              const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
              acc2[i & 1] = f2_add(acc2[i & 1], f2_make(p0, p1));
              pk[i] = pack_bf16x2(p0, p1);
            }
            tmem_st16(tS + c * 16, pk);
          }
          if (half == 0 && j > 0 && __any_sync(0xffffffffu, resc)) {
            // PV(j-1) of this tile completed before S(j) was signalled.
  #pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
              uint32_t orow[32];
              tmem_ld32(tO + c * 32, orow);
              tmem_wait_ld();
  #pragma unroll
              for (int i = 0; i < 32; ++i)
                orow[i] = __float_as_uint(__uint_as_float(orow[i]) * alpha);
              tmem_st32(tO + c * 32, orow);
            }
          }
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive_warp(bar(FB_PFULL + t));
        float a0, a1, a2, a3;
        f2_split(acc2[0], a0, a1);
        f2_split(acc2[1], a2, a3);
        l = l * alpha + ((a0 + a1) + (a2 + a3));
        m = m_use;
      }
      if (!ok) break;
      // ---- epilogue: O / l (bf16) and LSE.  Each 64-column half of O_t is
      // staged in this tile's 16 KB buffer (128-byte swizzle) and leaves in one
      // TMA tensor store (rows past Sq are clipped by the map); O_t is released
      // to the next item's first P V MMA once read out of TMEM.
      ok = __all_sync(0xffffffffu, mbar_wait(bar(FB_ODONE + t), uint32_t(no_t) & 1u, abort_flag,
                                             310 + t));
      if (!ok) break;
      tc_fence_after();
      const float inv_l = 1.0f / l;
      for (int hh = 0; hh < C::HALVES; ++hh) {
        // the previous store out of this buffer (of this item or the last one)
        // has read it
        if (epi_issuer) bulk_wait_group_read0();
        named_bar_sync(1 + t, 128);
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t orow[32];
          tmem_ld32(tO + hh * 64 + c * 32, orow);
          tmem_wait_ld();
          if (hh == C::HALVES - 1 && c == 1) {
            tc_fence_before();
            mbar_arrive_warp(bar(FB_OFREE + t));
          }
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            w[i] = pack_bf16x2(__uint_as_float(orow[2 * i]) * inv_l,
                               __uint_as_float(orow[2 * i + 1]) * inv_l);
#pragma unroll
          for (int v = 0; v < 4; ++v)
            st_shared_v4(stage_row + ((uint32_t(c * 4 + v) ^ uint32_t(row & 7)) << 4), w[4 * v],
                         w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
        }
        fence_proxy_async_smem();
        named_bar_sync(1 + t, 128);
        if (epi_issuer) {
          tma_store_3d(&tm_o, stage, hh * 64, qs, it.bh);
          bulk_commit_group();
        }
      }
      if (q_idx < p.Sq) p.lse[(size_t)it.bh * p.Sq + q_idx] = (m + lg2_approx(l)) * 0.6931471805599453f;
      st_t += nk;
      ++no_t;
    }
    if (epi_issuer) bulk_wait_group0();  // O stores complete before the CTA exits
  }

  // ---- teardown ----
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TM_COLS);
  }
}

}  // namespace tfb
