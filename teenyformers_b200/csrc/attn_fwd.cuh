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
// One CTA owns two 128-row query tiles of one head (rows q0..q0+255) and
// walks 128-row key/value tiles:
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
// issue order.  The running max is rescaled lazily: O and l are only
// rescaled when the row max grows by more than 2^8 (P stays <= 256).
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
  static constexpr int OFF_BAR = OFF_V + KSTAGES * TILE_BYTES;
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
  FB_PFULL = 11,  // 2
  FB_ODONE = 13,  // 2
  FB_DRAIN = 15,
  FB_COUNT = 16
};

// Waits without looking at the abort flag (used to drain in-flight async
// work before the CTA exits); bounded by kWaitTimeoutNs.
__device__ __forceinline__ void mbar_drain_wait(uint32_t bar, uint32_t parity, int site) {
  int dummy = 0;
  (void)mbar_wait(bar, parity, (volatile int*)&dummy, site);
}

template <int D>
__global__ void __launch_bounds__(320, 1)
    fa_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                        const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const FwdParams p) {
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

  // ---- work decode: heavy (late) query-tile pairs first for causal ----
  int pair = blockIdx.x / p.BHq;
  const int bh = blockIdx.x % p.BHq;
  if (p.causal) pair = p.n_pairs - 1 - pair;
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int bh_kv = b * p.Hkv + h / (p.Hq / p.Hkv);
  const int q0 = pair * 256;
  const int n_kv_all = (p.Sk + 127) / 128;
  int nkv[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int qs = q0 + 128 * t;
    if (qs >= p.Sq) {
      nkv[t] = 0;
    } else if (p.causal) {
      const int last_q = min(p.Sq, qs + 128) - 1;
      nkv[t] = min(n_kv_all, last_q / 128 + 1);
    } else {
      nkv[t] = n_kv_all;
    }
  }
  const int n_iter = max(nkv[0], nkv[1]);

  // ---- setup ----
  if (threadIdx.x == 0) {
    mbar_init(bar(FB_QFULL), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(FB_KFULL + s), 1);
      mbar_init(bar(FB_KEMPTY + s), 1);
      mbar_init(bar(FB_VFULL + s), 1);
      mbar_init(bar(FB_VEMPTY + s), 1);
      mbar_init(bar(FB_SFULL + s), 1);
      mbar_init(bar(FB_PFULL + s), 128);
      mbar_init(bar(FB_ODONE + s), 1);
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
    // =================== TMA producer ===================
    if (lane == 0) {
      int issued_k[2] = {0, 0}, issued_v[2] = {0, 0};
      bool ok = true;
      mbar_arrive_expect_tx(bar(FB_QFULL), 2 * C::TILE_BYTES);
      for (int t = 0; t < 2; ++t)
        for (int hh = 0; hh < C::HALVES; ++hh)
          tma_load_3d(sbase + C::OFF_Q + t * C::TILE_BYTES + hh * C::HALF_BYTES, &tm_q,
                      bar(FB_QFULL), hh * 64, q0 + 128 * t, bh);
      for (int j = 0; j < n_iter && ok; ++j) {
        const int s = j & 1, u = j >> 1;
        if (u > 0) ok = mbar_wait(bar(FB_KEMPTY + s), (u - 1) & 1, abort_flag, 101);
        if (!ok) break;
        mbar_arrive_expect_tx(bar(FB_KFULL + s), C::TILE_BYTES);
        for (int hh = 0; hh < C::HALVES; ++hh)
          tma_load_3d(sbase + C::OFF_K + s * C::TILE_BYTES + hh * C::HALF_BYTES, &tm_k,
                      bar(FB_KFULL + s), hh * 64, j * 128, bh_kv);
        ++issued_k[s];
        if (u > 0) ok = mbar_wait(bar(FB_VEMPTY + s), (u - 1) & 1, abort_flag, 102);
        if (!ok) break;
        mbar_arrive_expect_tx(bar(FB_VFULL + s), C::TILE_BYTES);
        for (int hh = 0; hh < C::HALVES; ++hh)
          tma_load_3d(sbase + C::OFF_V + s * C::TILE_BYTES + hh * C::HALF_BYTES, &tm_v,
                      bar(FB_VFULL + s), hh * 64, j * 128, bh_kv);
        ++issued_v[s];
      }
      if (!ok) {
        // Abort: let every issued copy land before the CTA's smem goes away.
        mbar_drain_wait(bar(FB_QFULL), 0, 103);
        for (int s = 0; s < 2; ++s) {
          if (issued_k[s]) mbar_drain_wait(bar(FB_KFULL + s), (issued_k[s] - 1) & 1, 103);
          if (issued_v[s]) mbar_drain_wait(bar(FB_VFULL + s), (issued_v[s] - 1) & 1, 103);
        }
      }
    }
  } else if (warp == 8) {
    // =================== MMA issuer ===================
    if (lane == 0) {
      constexpr uint32_t idesc_qk = make_idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t idesc_pv = make_idesc_bf16(128, D, 0, 1);
      auto issue_qk = [&](int t, int slot) {
        const uint32_t a0 = sbase + C::OFF_Q + t * C::TILE_BYTES;
        const uint32_t b0 = sbase + C::OFF_K + slot * C::TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * C::HALF_BYTES + (kk & 3) * 32;
          mma_ss(tmem + C::tm_s(t), make_sdesc_sw128(a0 + off, 16, 1024),
                 make_sdesc_sw128(b0 + off, 16, 1024), idesc_qk, kk > 0);
        }
      };
      auto issue_pv = [&](int t, int slot, bool acc) {
        const uint32_t b0 = sbase + C::OFF_V + slot * C::TILE_BYTES;
#pragma unroll
        for (int kk = 0; kk < 128 / 16; ++kk) {
          mma_ts(tmem + C::tm_o(t), tmem + C::tm_s(t) + kk * 8,
                 make_sdesc_sw128(b0 + kk * 16 * 128, C::HALF_BYTES, 1024), idesc_pv,
                 (acc || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(bar(FB_QFULL), 0, abort_flag, 201);
      if (ok && n_iter > 0) ok = mbar_wait(bar(FB_KFULL + 0), 0, abort_flag, 202);
      if (ok && n_iter > 0) {
        tc_fence_after();
        for (int t = 0; t < 2; ++t)
          if (nkv[t] > 0) {
            issue_qk(t, 0);
            tc_commit(bar(FB_SFULL + t));
          }
        tc_commit(bar(FB_KEMPTY + 0));
      }
      for (int j = 0; j < n_iter && ok; ++j) {
        const int s = j & 1;
        const int sn = (j + 1) & 1;
        ok = mbar_wait(bar(FB_VFULL + s), (j >> 1) & 1, abort_flag, 203);
        if (!ok) break;
        bool k_next_ready = false;
        for (int t = 0; t < 2 && ok; ++t) {
          if (j >= nkv[t]) continue;
          ok = mbar_wait(bar(FB_PFULL + t), j & 1, abort_flag, 204);
          if (!ok) break;
          tc_fence_after();
          issue_pv(t, s, j > 0);
          if (j + 1 < nkv[t]) {
            if (!k_next_ready) {
              ok = mbar_wait(bar(FB_KFULL + sn), ((j + 1) >> 1) & 1, abort_flag, 205);
              if (!ok) break;
              tc_fence_after();
              k_next_ready = true;
            }
            issue_qk(t, sn);
            tc_commit(bar(FB_SFULL + t));
          } else {
            tc_commit(bar(FB_ODONE + t));
          }
        }
        if (!ok) break;
        tc_commit(bar(FB_VEMPTY + s));
        if (j + 1 < n_iter) tc_commit(bar(FB_KEMPTY + sn));
      }
      // Drain: every MMA issued above completes before TMEM is released.
      tc_commit(bar(FB_DRAIN));
      mbar_drain_wait(bar(FB_DRAIN), 0, 206);
    }
  } else {
    // =================== softmax: warps 0-3 tile 0, 4-7 tile 1 ===================
    const int t = warp >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_base = uint32_t(wq * 32) << 16;
    const uint32_t tS = tmem + lane_base + C::tm_s(t);
    const uint32_t tO = tmem + lane_base + C::tm_o(t);
    const int qs = q0 + 128 * t;
    const int q_idx = qs + row;
    const float sl2 = p.scale_log2;
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < nkv[t]; ++j) {
      ok = mbar_wait(bar(FB_SFULL + t), j & 1, abort_flag, 300 + t);
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
      float rmax = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 32; ++i) rmax = fmaxf(rmax, __uint_as_float(sr[c][i]));
      const float m_new = fmaxf(m, rmax * sl2);
      const bool resc = m_new > m + 8.0f;
      const float m_use = resc ? m_new : m;
      const float alpha = resc ? ex2_approx(m - m_use) : 1.0f;
      const float base = (m_use == -INFINITY) ? 0.0f : m_use;
      float rsum = 0.0f;
      uint32_t pk[2][32];
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float p0 = ex2_approx(fmaf(__uint_as_float(sr[c][2 * i]), sl2, -base));
          const float p1 = ex2_approx(fmaf(__uint_as_float(sr[c][2 * i + 1]), sl2, -base));
          rsum += p0 + p1;
          pk[c >> 1][(c & 1) * 16 + i] = pack_bf16x2(p0, p1);
        }
      l = l * alpha + rsum;
      tmem_st32(tS + 0, pk[0]);
      tmem_st32(tS + 32, pk[1]);
      if (j > 0 && __any_sync(0xffffffffu, resc)) {
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
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar(FB_PFULL + t));
      m = m_use;
    }
    if (ok && nkv[t] > 0) {
      ok = mbar_wait(bar(FB_ODONE + t), 0, abort_flag, 310 + t);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
        const float inv_l = 1.0f / l;
        const bool valid = q_idx < p.Sq;
        __nv_bfloat16* orow_g = p.o + ((size_t)bh * p.Sq + (valid ? q_idx : 0)) * D;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t orow[32];
          tmem_ld32(tO + c * 32, orow);
          tmem_wait_ld();
          uint32_t w[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            w[i] = pack_bf16x2(__uint_as_float(orow[2 * i]) * inv_l,
                               __uint_as_float(orow[2 * i + 1]) * inv_l);
          if (valid) {
            uint4* dst = reinterpret_cast<uint4*>(orow_g + c * 32);
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4)
              dst[v4] = make_uint4(w[4 * v4], w[4 * v4 + 1], w[4 * v4 + 2], w[4 * v4 + 3]);
          }
        }
        if (valid) p.lse[(size_t)bh * p.Sq + q_idx] = (m + lg2_approx(l)) * 0.6931471805599453f;
      }
    }
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
