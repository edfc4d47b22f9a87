// attn_bwd.cuh -- flash-attention-2 backward for sm_100a (bf16 in/out, fp32 acc).
//
// Gradients of teenyformers' flash_attn2_causal_bwd / flash_attn2_backward
// (src/kernels/flash_attn2.rs:135-279):
//   D_q  = rowsum(O_q * dO_q)                       (:171)
//   P    = exp(Q K^T * scale - LSE), future keys 0  (:186-189, top-left k > q)
//   dS   = P * (dO V^T - D_q)                       (:191-192)
//   dQ   = dS K * scale,  dK = dS^T Q * scale,  dV = P^T dO   (:194-197)
// The reference adds dK/dV with per-(q,k) fp32 atomics; here they are
// accumulated on chip, so the result is deterministic and dK/dV need no
// zero-initialisation.
//
// Three kernels, all single-CTA tcgen05 (no clusters, no multicast):
//  1. fa_bwd_prep_kernel: -D_q and -LSE*log2(e) per query row into the
//     workspace ([BHq, Sq_pad] each; stored negated so the elementwise
//     passes are one packed FMA / ADD; padded rows get 0 and -inf so their
//     P is exactly 0).
//  2. fa_bwd_dkdv_sm100_kernel: one CTA per 128-key tile of one KV head,
//     looping over the 128-row query tiles of every query head of the GQA
//     group.  Each query tile is processed as two 64-query halves h so the
//     elementwise work on one half overlaps the MMAs of the other:
//       S^T_h = K Q_h^T, dP^T_h = V dO_h^T        (M=128 keys, N=64)
//       P^T_h, dS^T_h in bf16 over the first 32 columns of S^T_h / dP^T_h
//       dV += P^T_h dO_h, dK += dS^T_h Q_h         (A from TMEM, K=64)
//     TMEM: S^T_0 [0,64) S^T_1 [64,128) dP^T_0 [128,192) dP^T_1 [192,256)
//           dV [256,256+D) dK [256+D,256+2D).
//     S^T_0/dP^T_0 of the next query tile are issued as soon as the dV/dK
//     MMAs of half 0 are queued (tcgen05 MMAs of one thread run in order).
//  3. fa_bwd_dq_sm100_kernel: one CTA per 128-row query tile, looping over
//     key tiles in two 64-key halves: S_h = Q K_h^T, dP_h = dO V_h^T,
//     dS_h (bf16) over S_h, dQ += dS_h K_h.  Q and dO are copied into TMEM
//     once, so S_h and dP_h are TS MMAs (A from TMEM; only K/V are read
//     from shared memory, which keeps N=64 MMAs at full rate).  TMEM:
//     S_0 S_1 dP_0 dP_1 as above, dQ [256,256+D), Q [384,384+D/2),
//     dO [384+D/2, 384+D).  K/V stream through a 3-stage ring.
// Roles (both kernels): warps 0-15 elementwise, four warpgroups, one per
// 32-column chunk c of half h (warpgroup 2h + c; one TMEM lane = one row per
// thread), so each SM sub-partition runs four elementwise warps; warp 16
// MMA issuer, warp 17 TMA producer.  The issuer and producer loops run on
// the whole warp and one elected lane issues.
#pragma once

#include <type_traits>

#include "sm100.cuh"

namespace tfb {

inline long long bwd_sq_pad(int Sq) { return ((long long)Sq + 127) / 128 * 128; }
// -LSE*log2e and -D rows ([BHq, Sq_pad] fp32 each), as the two-kernel path uses
inline size_t bwd_workspace_bytes(long long bhq, int Sq) {
  return (size_t)(2 * bhq * bwd_sq_pad(Sq) * 4);
}
// ... plus the fused path's fp32 dQ accumulator [BHq, Sq_pad, D] (sized for D = 128)
// and its work-item counter (256 bytes)
inline size_t bwd_fused_workspace_bytes(long long bhq, int Sq) {
  return bwd_workspace_bytes(bhq, Sq) + (size_t)bhq * bwd_sq_pad(Sq) * 128 * 4 + 256;
}

// ------------------------------------------------------------------ prep
// grid = ceil(BHq * Sq_pad / 16), block 256: 16 threads per row, 8 elements
// (16 bytes) each; requires D % 128 == 0 or D == 64.
// With dq_acc non-null it also zeroes that row of the [rows, D] fp32 dQ
// accumulator of the fused backward, and with counter non-null resets the
// fused kernel's work-item counter.
template <int D>
__global__ void __launch_bounds__(256)
    fa_bwd_prep_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dO,
                       const float* __restrict__ lse, float* __restrict__ ws_lse2,
                       float* __restrict__ ws_delta, float* __restrict__ dq_acc,
                       int* __restrict__ counter, int Sq, int Sq_pad, long long rows) {
  constexpr int TPR = 16;  // threads per row
  const long long row = (long long)blockIdx.x * (256 / TPR) + threadIdx.x / TPR;
  const int sub = threadIdx.x % TPR;
  if (counter && blockIdx.x == 0 && threadIdx.x == 0) *counter = 0;
  if (row >= rows) return;
  if (dq_acc) {
    float4* z = reinterpret_cast<float4*>(dq_acc + row * D);
#pragma unroll
    for (int v = sub; v < D / 4; v += TPR) z[v] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const long long bh = row / Sq_pad;
  const int qi = (int)(row % Sq_pad);
  float acc = 0.0f;
  if (qi < Sq) {
    const uint4* po = reinterpret_cast<const uint4*>(o + ((size_t)bh * Sq + qi) * D);
    const uint4* pd = reinterpret_cast<const uint4*>(dO + ((size_t)bh * Sq + qi) * D);
#pragma unroll
    for (int v = sub; v < D / 8; v += TPR) {
      const uint4 a = po[v], g = pd[v];
      const uint32_t wa[4] = {a.x, a.y, a.z, a.w}, wg[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc += __uint_as_float(wa[i] << 16) * __uint_as_float(wg[i] << 16);
        acc += __uint_as_float(wa[i] & 0xFFFF0000u) * __uint_as_float(wg[i] & 0xFFFF0000u);
      }
    }
  }
#pragma unroll
  for (int off = TPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (sub == 0) {
    ws_delta[row] = -acc;
    ws_lse2[row] = qi < Sq ? -lse[(size_t)bh * Sq + qi] * 1.4426950408889634f : -INFINITY;
  }
}

// ------------------------------------------------------------------ shared config
struct BwdParams {
  __nv_bfloat16* dq;
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  const float* ws_lse2;   // -LSE * log2(e)
  const float* ws_delta;  // -rowsum(O * dO)
  int Sq, Sk, Sq_pad;
  int Hq, Hkv;
  int BHq, BHkv;
  int n_qt, n_kt;
  float scale;       // softmax scale (natural)
  float scale_log2;  // scale * log2(e)
  int causal;
  int* work_counter;  // fused path: next work item (zeroed by the prep kernel)
  int n_items;        // fused path: BHkv * n_kt
};

__device__ __forceinline__ void bulk_load(uint32_t smem_dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void mbar_wait_noabort(uint32_t bar, uint32_t parity, int site) {
  (void)mbar_wait(bar, parity, nullptr, site);
}

constexpr int kBwdThreads = 576;  // 16 elementwise warps + MMA warp + TMA warp
constexpr int kBwdMmaWarp = 16, kBwdTmaWarp = 17;

template <int D>
struct BwdKvCfg {
  static constexpr int kThreads = kBwdThreads;
  static constexpr int HALVES = D / 64;
  static constexpr int HALF_BYTES = 128 * 128;
  static constexpr int TILE_BYTES = 128 * D * 2;
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + TILE_BYTES;
  static constexpr int OFF_STAGE = OFF_V + TILE_BYTES;  // 2 stages of {Q, dO, lse2, delta}
  static constexpr int STAGE_Q = 0;
  static constexpr int STAGE_DO = TILE_BYTES;
  static constexpr int STAGE_LSE = 2 * TILE_BYTES;
  static constexpr int STAGE_DELTA = 2 * TILE_BYTES + 512;
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES + 1024;
  static constexpr int OFF_BAR = OFF_STAGE + 2 * STAGE_BYTES;
  static constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;
  static constexpr uint32_t TM_DV = 256, TM_DK = 256 + D;
  static constexpr uint32_t TM_COLS = 512;
  __device__ static constexpr uint32_t tm_st(int h) { return uint32_t(h) * 64u; }
  __device__ static constexpr uint32_t tm_dpt(int h) { return 128u + uint32_t(h) * 64u; }
};

template <int D>
struct BwdQCfg {
  static constexpr int kThreads = kBwdThreads;
  static constexpr int HALVES = D / 64;
  static constexpr int HALF_BYTES = 128 * 128;
  static constexpr int TILE_BYTES = 128 * D * 2;
  static constexpr int KV_STAGES = 3;
  static constexpr int OFF_STAGE = 0;  // KV_STAGES stages of {K, V}
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
  static constexpr int OFF_BAR = OFF_STAGE + KV_STAGES * STAGE_BYTES;
  static constexpr int SMEM_BYTES = OFF_BAR + 256 + 1024;
  static constexpr uint32_t TM_DQ = 256, TM_Q = 384, TM_DO = 384 + D / 2;
  static constexpr uint32_t TM_COLS = 512;
  __device__ static constexpr uint32_t tm_s(int h) { return uint32_t(h) * 64u; }
  __device__ static constexpr uint32_t tm_dp(int h) { return 128u + uint32_t(h) * 64u; }
};

enum BwdKvBar { KB_KV = 0, KB_QFULL = 1, KB_QEMPTY = 3, KB_SFULL = 5, KB_PFULL = 7,
                KB_ACC = 9, KB_DRAIN = 10, KB_COUNT = 11 };
enum BwdQBar { QB_Q = 0, QB_KVFULL = 1, QB_KVEMPTY = 4, QB_SFULL = 7, QB_PFULL = 9,
               QB_ACC = 11, QB_DRAIN = 12, QB_QFREE = 13, QB_DQFREE = 14, QB_COUNT = 15 };

// TMEM column (relative to a half's base) of the bf16-packed operand for
// the 16-row K step kk of that half: the 64 rows are written as two 32-row
// chunks, each packed into the first 16 columns of its own 32-column slot.
__device__ __forceinline__ constexpr uint32_t packed_col(int kk) {
  return uint32_t((kk >> 1) * 32 + (kk & 1) * 8);
}

// Stores one 32-column fp32 TMEM chunk (scaled) as 32 bf16 to global.
__device__ __forceinline__ void store_row_chunk_bf16(__nv_bfloat16* dst, const uint32_t (&r)[32],
                                                     float mul) {
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 16; ++i)
    w[i] = pack_bf16x2(__uint_as_float(r[2 * i]) * mul, __uint_as_float(r[2 * i + 1]) * mul);
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int v = 0; v < 4; ++v) d4[v] = make_uint4(w[4 * v], w[4 * v + 1], w[4 * v + 2], w[4 * v + 3]);
}

// Operand descriptors are built once per buffer and advanced per step by a
// compile-time constant (desc_adv).  A 128-row tile is stored as D/64
// column halves of 128 rows x 128 bytes (SW128):
//  - read K-major (rows = M or N, 64-element atoms along K):  base LBO 16,
//    step kk at kstep_off(kk), 64-row sub-tile row0 at + row0 * 128;
//  - read MN-major as K x N with N = D (rows = K): base LBO = HALF_BYTES,
//    K rows row0 + 16 kk at + (row0 + 16 kk) * 128.
template <int HALF_BYTES>
__device__ __forceinline__ uint64_t kmajor_base(uint32_t tile) {
  return make_sdesc_sw128(tile, 16, 1024);
}
template <int HALF_BYTES>
__device__ __forceinline__ uint64_t mnmajor_base(uint32_t tile) {
  return make_sdesc_sw128(tile, HALF_BYTES, 1024);
}

// ------------------------------------------------------------------ dK / dV
template <int D>
__global__ void __launch_bounds__(kBwdThreads, 1)
    fa_bwd_dkdv_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                             const __grid_constant__ CUtensorMap tm_do,
                             const __grid_constant__ CUtensorMap tm_k,
                             const __grid_constant__ CUtensorMap tm_v, const BwdParams p) {
  using C = BwdKvCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + KB_COUNT);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto bar = [&](int i) { return smem_u32(bars + i); };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // Head-major (a head's Q/dO stay hot in L2 while its key tiles run), and
  // within a head key tile 0 first: it has the most query tiles when causal.
  const int bh_kv = blockIdx.x / p.n_kt;
  const int kt = blockIdx.x % p.n_kt;
  const int b = bh_kv / p.Hkv, hk = bh_kv % p.Hkv;
  const int G = p.Hq / p.Hkv;
  const int k0 = kt * 128;
  const int qt_first = p.causal ? min(kt, p.n_qt) : 0;  // query tile i sees keys iff i >= kt
  const int qt_per_head = p.n_qt - qt_first;
  const int n_tiles = G * qt_per_head;

  if (threadIdx.x == 0) {
    mbar_init(bar(KB_KV), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(KB_QFULL + s), 1);
      mbar_init(bar(KB_QEMPTY + s), 1);
      mbar_init(bar(KB_SFULL + s), 1);
      mbar_init(bar(KB_PFULL + s), 8);  // one arrival per elementwise warp
    }
    mbar_init(bar(KB_ACC), 1);
    mbar_init(bar(KB_DRAIN), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), C::TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kBwdTmaWarp) {
    // ---------------- TMA producer (whole warp, one elected lane issues) --------
    if (n_tiles > 0) {
      int issued0 = 0, issued1 = 0;
      bool ok = true;
      if (elect_one()) {
        mbar_arrive_expect_tx(bar(KB_KV), 2 * C::TILE_BYTES);
        for (int hh = 0; hh < C::HALVES; ++hh) {
          tma_load_3d(sbase + C::OFF_K + hh * C::HALF_BYTES, &tm_k, bar(KB_KV), hh * 64, k0,
                      bh_kv);
          tma_load_3d(sbase + C::OFF_V + hh * C::HALF_BYTES, &tm_v, bar(KB_KV), hh * 64, k0,
                      bh_kv);
        }
      }
      __syncwarp();
      for (int it = 0; it < n_tiles && ok; ++it) {
        const int st = it & 1, u = it >> 1;
        if (u > 0) ok = mbar_wait_warp(bar(KB_QEMPTY + st), (u - 1) & 1, abort_flag, 401);
        if (!ok) break;
        const int g = it / qt_per_head;
        const int qi = qt_first + it % qt_per_head;
        const int bh_q = b * p.Hq + hk * G + g;
        const uint32_t sb = sbase + C::OFF_STAGE + st * C::STAGE_BYTES;
        if (elect_one()) {
          mbar_arrive_expect_tx(bar(KB_QFULL + st), 2 * C::TILE_BYTES + 1024);
          for (int hh = 0; hh < C::HALVES; ++hh) {
            tma_load_3d(sb + C::STAGE_Q + hh * C::HALF_BYTES, &tm_q, bar(KB_QFULL + st),
                        hh * 64, qi * 128, bh_q);
            tma_load_3d(sb + C::STAGE_DO + hh * C::HALF_BYTES, &tm_do, bar(KB_QFULL + st),
                        hh * 64, qi * 128, bh_q);
          }
          const size_t ws_off = (size_t)bh_q * p.Sq_pad + (size_t)qi * 128;
          bulk_load(sb + C::STAGE_LSE, p.ws_lse2 + ws_off, 512, bar(KB_QFULL + st));
          bulk_load(sb + C::STAGE_DELTA, p.ws_delta + ws_off, 512, bar(KB_QFULL + st));
        }
        __syncwarp();
        (st ? issued1 : issued0) += 1;
      }
      if (!ok) {
        mbar_wait_noabort(bar(KB_KV), 0, 402);
        if (issued0) mbar_wait_noabort(bar(KB_QFULL + 0), (issued0 - 1) & 1, 402);
        if (issued1) mbar_wait_noabort(bar(KB_QFULL + 1), (issued1 - 1) & 1, 402);
      }
    }
  } else if (warp == kBwdMmaWarp) {
    // ---------------- MMA issuer (whole warp, one elected lane issues) ----------
    if (n_tiles > 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16(128, 64, 0, 0);
      constexpr uint32_t idesc_acc = make_idesc_bf16(128, D, 0, 1);
      const uint64_t d_k = kmajor_base<C::HALF_BYTES>(sbase + C::OFF_K);
      const uint64_t d_v = kmajor_base<C::HALF_BYTES>(sbase + C::OFF_V);
      const uint64_t d_q0 = kmajor_base<C::HALF_BYTES>(sbase + C::OFF_STAGE + C::STAGE_Q);
      const uint64_t d_do0 = kmajor_base<C::HALF_BYTES>(sbase + C::OFF_STAGE + C::STAGE_DO);
      const uint64_t m_q0 = mnmajor_base<C::HALF_BYTES>(sbase + C::OFF_STAGE + C::STAGE_Q);
      const uint64_t m_do0 = mnmajor_base<C::HALF_BYTES>(sbase + C::OFF_STAGE + C::STAGE_DO);
      // S^T_h = K Q_h^T and dP^T_h = V dO_h^T for stage st, then signal s_full[h]
      auto issue_s = [&](int h, int st) {
        if (elect_one()) {
          const uint32_t so = st * C::STAGE_BYTES + h * 64 * 128;
          const uint64_t bq = desc_adv(d_q0, so), bdo = desc_adv(d_do0, so);
          const uint32_t dst = tmem + C::tm_st(h), ddp = tmem + C::tm_dpt(h);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            mma_ss(dst, desc_adv(d_k, kstep_off(kk, C::HALF_BYTES)),
                   desc_adv(bq, kstep_off(kk, C::HALF_BYTES)), idesc_s, kk > 0);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            mma_ss(ddp, desc_adv(d_v, kstep_off(kk, C::HALF_BYTES)),
                   desc_adv(bdo, kstep_off(kk, C::HALF_BYTES)), idesc_s, kk > 0);
          tc_commit(bar(KB_SFULL + h));
        }
        __syncwarp();
      };
      // dV += P^T_h dO_h, dK += dS^T_h Q_h; then an optional commit
      auto issue_acc = [&](int h, int st, bool acc, int commit) {
        if (elect_one()) {
          const uint32_t so = st * C::STAGE_BYTES + h * 64 * 128;
          const uint64_t bdo = desc_adv(m_do0, so), bq = desc_adv(m_q0, so);
          const uint32_t ap = tmem + C::tm_st(h), ads = tmem + C::tm_dpt(h);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_ts(tmem + C::TM_DV, ap + packed_col(kk), desc_adv(bdo, kk * 16 * 128), idesc_acc,
                   (acc || kk > 0) ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_ts(tmem + C::TM_DK, ads + packed_col(kk), desc_adv(bq, kk * 16 * 128), idesc_acc,
                   (acc || kk > 0) ? 1u : 0u);
          if (commit >= 0) tc_commit(bar(commit));
        }
        __syncwarp();
      };
      bool ok = mbar_wait_warp(bar(KB_KV), 0, abort_flag, 411);
      if (ok) ok = mbar_wait_warp(bar(KB_QFULL + 0), 0, abort_flag, 412);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
      }
      for (int it = 0; it < n_tiles && ok; ++it) {
        const int st = it & 1;
        const bool more = it + 1 < n_tiles;
        ok = mbar_wait_warp(bar(KB_PFULL + 0), it & 1, abort_flag, 413);
        if (!ok) break;
        tc_fence_after();
        issue_acc(0, st, it > 0, -1);
        if (more) {
          ok = mbar_wait_warp(bar(KB_QFULL + (st ^ 1)), ((it + 1) >> 1) & 1, abort_flag, 414);
          if (!ok) break;
          tc_fence_after();
          issue_s(0, st ^ 1);
        }
        ok = mbar_wait_warp(bar(KB_PFULL + 1), it & 1, abort_flag, 415);
        if (!ok) break;
        tc_fence_after();
        issue_acc(1, st, true, more ? KB_QEMPTY + st : KB_ACC);
        if (more) issue_s(1, st ^ 1);
      }
      if (elect_one()) tc_commit(bar(KB_DRAIN));
      __syncwarp();
      mbar_wait_noabort(bar(KB_DRAIN), 0, 416);
    }
  } else {
    // ------------- elementwise: warpgroup 2h + c owns query columns
    // [64h + 32c, 64h + 32c + 32) of every tile; thread = key row
    const int wg = warp >> 2;
    const int h = wg >> 1, cq = wg & 1;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_base = uint32_t(wq * 32) << 16;
    const int key = k0 + row;
    const float sl2 = p.scale_log2;
    const int col0 = h * 64 + cq * 32;  // first query column of this warpgroup's chunk
    bool ok = true;
    for (int it = 0; it < n_tiles && ok; ++it) {
      const int st = it & 1;
      const int qi = qt_first + it % qt_per_head;
      const uint8_t* sb = smem + C::OFF_STAGE + st * C::STAGE_BYTES;
      const float4* s_lse = reinterpret_cast<const float4*>(sb + C::STAGE_LSE);
      const float4* s_delta = reinterpret_cast<const float4*>(sb + C::STAGE_DELTA);
      const bool diag = p.causal && qi * 128 < k0 + 127;
      const int qlim = key - qi * 128;  // query columns with index < qlim are hidden (k > q)
      ok = mbar_wait(bar(KB_SFULL + h), it & 1, abort_flag, 421);
      if (ok) ok = mbar_wait(bar(KB_QFULL + st), (it >> 1) & 1, abort_flag, 422);
      ok = __all_sync(0xffffffffu, ok);  // keep .sync.aligned TMEM ops convergent
      if (!ok) break;
      tc_fence_after();
      // P^T = 2^(s*scale*log2e - lse), dS^T = P^T * (dP^T - D), both packed to
      // bf16 over the columns already read; 16 query columns per step.
      auto step = [&](auto mask_tag, int sub) {
        constexpr bool kMask = decltype(mask_tag)::value;
        const int c0 = col0 + sub * 16;
        uint32_t sr[16], dr[16];
        tmem_ld16(tmem + lane_base + C::tm_st(h) + cq * 32 + sub * 16, sr);
        tmem_ld16(tmem + lane_base + C::tm_dpt(h) + cq * 32 + sub * 16, dr);
        tmem_wait_ld();
        uint32_t pk[8], dk[8];
#pragma unroll
        for (int v4 = 0; v4 < 4; ++v4) {
          const float4 l4 = s_lse[c0 / 4 + v4];    // -lse2
          const float4 d4 = s_delta[c0 / 4 + v4];  // -D
          const float nl[4] = {l4.x, l4.y, l4.z, l4.w};
          const float nd[4] = {d4.x, d4.y, d4.z, d4.w};
          float pv[4], dsv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int i = v4 * 4 + e;
            float pe = ex2_approx(fmaf(__uint_as_float(sr[i]), sl2, nl[e]));
            if (kMask && c0 + i < qlim) pe = 0.0f;
            pv[e] = pe;
            dsv[e] = pe * (__uint_as_float(dr[i]) + nd[e]);
          }
          pk[2 * v4] = pack_bf16x2(pv[0], pv[1]);
          pk[2 * v4 + 1] = pack_bf16x2(pv[2], pv[3]);
          dk[2 * v4] = pack_bf16x2(dsv[0], dsv[1]);
          dk[2 * v4 + 1] = pack_bf16x2(dsv[2], dsv[3]);
        }
        // Packed output stays inside this warpgroup's own 32 read columns
        // (the other warpgroup of the half may still be reading its own):
        // chunk cq, step sub -> columns 32*cq + 8*sub of the half.
        tmem_st8(tmem + lane_base + C::tm_st(h) + cq * 32 + sub * 8, pk);
        tmem_st8(tmem + lane_base + C::tm_dpt(h) + cq * 32 + sub * 8, dk);
      };
      if (diag) {
        step(std::true_type{}, 0);
        step(std::true_type{}, 1);
      } else {
        step(std::false_type{}, 0);
        step(std::false_type{}, 1);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive_warp(bar(KB_PFULL + h));
    }
    // ---- epilogue: warpgroups 0,1 write dV, 2,3 dK (= acc * scale), 64 columns each
    const bool valid = key < p.Sk;
    __nv_bfloat16* out_row = (h == 0 ? p.dv : p.dk) +
                             ((size_t)bh_kv * p.Sk + (valid ? key : 0)) * D + cq * (D / 2);
    if (n_tiles == 0) {
      if (valid) {
        uint4* a4 = reinterpret_cast<uint4*>(out_row);
        for (int v4 = 0; v4 < D / 16; ++v4) a4[v4] = make_uint4(0, 0, 0, 0);
      }
    } else if (__all_sync(0xffffffffu, ok && mbar_wait(bar(KB_ACC), 0, abort_flag, 423))) {
      tc_fence_after();
      const uint32_t acc_col = (h == 0 ? C::TM_DV : C::TM_DK) + cq * (D / 2);
      const float mul = h == 0 ? 1.0f : p.scale;
#pragma unroll 1
      for (int c = 0; c < D / 64; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + acc_col + c * 32, r);
        tmem_wait_ld();
        if (valid) store_row_chunk_bf16(out_row + c * 32, r, mul);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TM_COLS);
  }
}

// ------------------------------------------------------------------ dQ
// Persistent: gridDim.x CTAs (one per SM) walk the work items in rounds of
// gridDim.x, boustrophedon order (sched_item), so every CTA gets a mix of
// heavy and light items; item w is query tile qi of head bh, head-major
// (a few heads' K/V hot in L2 at a time) with heavy (late) query tiles first
// under the causal mask.  The K/V ring, the per-half S / P barriers and TMEM carry over from
// item to item; the next item's Q / dO rows are prefetched into registers
// while the current item runs, staged into TMEM as soon as its last S MMA
// has drained (QB_QFREE), and the MMA warp starts the next item's S MMAs
// while the elementwise warps run the current item's epilogue.
struct DqItem {
  int bh, qi, q0, n_kv, bh_kv;
};

// Item of round k for this CTA: rounds alternate direction so the heavy
// items at the start of each head spread evenly over the CTAs.  Only the
// last round can be partial, so an out-of-range item means "no more".
__device__ __forceinline__ int sched_item(int k) {
  const int G = gridDim.x, c = blockIdx.x;
  return k * G + ((k & 1) ? G - 1 - c : c);
}

__device__ __forceinline__ DqItem dq_item(const BwdParams& p, int w) {
  DqItem it;
  it.bh = w / p.n_qt;
  it.qi = w % p.n_qt;
  if (p.causal) it.qi = p.n_qt - 1 - it.qi;
  it.q0 = it.qi * 128;
  it.n_kv = p.n_kt;
  if (p.causal) it.n_kv = min(p.n_kt, (min(p.Sq, it.q0 + 128) - 1) / 128 + 1);
  const int b = it.bh / p.Hq, h_q = it.bh % p.Hq;
  it.bh_kv = b * p.Hkv + h_q / (p.Hq / p.Hkv);
  return it;
}

template <int D>
__global__ void __launch_bounds__(kBwdThreads, 1)
    fa_bwd_dq_sm100_kernel(const __grid_constant__ CUtensorMap tm_k,
                           const __grid_constant__ CUtensorMap tm_v, const BwdParams p,
                           const __nv_bfloat16* __restrict__ q,
                           const __nv_bfloat16* __restrict__ dO) {
  using C = BwdQCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + QB_COUNT);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto bar = [&](int i) { return smem_u32(bars + i); };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = p.BHq * p.n_qt;

  if (threadIdx.x == 0) {
    mbar_init(bar(QB_Q), 16);  // one arrival per elementwise warp
    mbar_init(bar(QB_QFREE), 1);
    mbar_init(bar(QB_DQFREE), 16);
    for (int s = 0; s < C::KV_STAGES; ++s) {
      mbar_init(bar(QB_KVFULL + s), 1);
      mbar_init(bar(QB_KVEMPTY + s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(QB_SFULL + s), 1);
      mbar_init(bar(QB_PFULL + s), 8);
    }
    mbar_init(bar(QB_ACC), 1);
    mbar_init(bar(QB_DRAIN), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), C::TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kBwdTmaWarp) {
    // ---------------- TMA producer (whole warp, one elected lane issues) --------
    int issued[C::KV_STAGES] = {};
    bool ok = true;
    int g = 0;  // K/V tiles this CTA has loaded so far (ring position)
    for (int k = 0; ok; ++k) {
      const int w = sched_item(k);
      if (w >= n_items) break;
      const DqItem it = dq_item(p, w);
      for (int j = 0; j < it.n_kv && ok; ++j, ++g) {
        const int st = g % C::KV_STAGES, u = g / C::KV_STAGES;
        if (u > 0) ok = mbar_wait_warp(bar(QB_KVEMPTY + st), (u - 1) & 1, abort_flag, 501);
        if (!ok) break;
        const uint32_t sb = sbase + C::OFF_STAGE + st * C::STAGE_BYTES;
        if (elect_one()) {
          mbar_arrive_expect_tx(bar(QB_KVFULL + st), 2 * C::TILE_BYTES);
          for (int hh = 0; hh < C::HALVES; ++hh) {
            tma_load_3d(sb + hh * C::HALF_BYTES, &tm_k, bar(QB_KVFULL + st), hh * 64, j * 128,
                        it.bh_kv);
            tma_load_3d(sb + C::TILE_BYTES + hh * C::HALF_BYTES, &tm_v, bar(QB_KVFULL + st),
                        hh * 64, j * 128, it.bh_kv);
          }
        }
        __syncwarp();
#pragma unroll
        for (int s2 = 0; s2 < C::KV_STAGES; ++s2) issued[s2] += (s2 == st);
      }
    }
    if (!ok) {
#pragma unroll
      for (int s2 = 0; s2 < C::KV_STAGES; ++s2)
        if (issued[s2]) mbar_wait_noabort(bar(QB_KVFULL + s2), (issued[s2] - 1) & 1, 502);
    }
  } else if (warp == kBwdMmaWarp) {
    // ---------------- MMA issuer (whole warp, one elected lane issues) ----------
    constexpr uint32_t idesc_s = make_idesc_bf16(128, 64, 0, 0);
    constexpr uint32_t idesc_dq = make_idesc_bf16(128, D, 0, 1);
    const uint64_t d_k0 = kmajor_base<C::HALF_BYTES>(sbase + C::OFF_STAGE);
    const uint64_t d_v0 = kmajor_base<C::HALF_BYTES>(sbase + C::OFF_STAGE + C::TILE_BYTES);
    const uint64_t m_k0 = mnmajor_base<C::HALF_BYTES>(sbase + C::OFF_STAGE);
    // S_h = Q K_h^T, dP_h = dO V_h^T for key stage st (A = Q / dO in TMEM),
    // then signal s_full[h] (and, for the item's last tile, QB_QFREE)
    auto issue_s = [&](int h, int st, bool last_of_item) {
      if (elect_one()) {
        const uint32_t so = st * C::STAGE_BYTES + h * 64 * 128;
        const uint64_t bk = desc_adv(d_k0, so), bv = desc_adv(d_v0, so);
        const uint32_t ds = tmem + C::tm_s(h), ddp = tmem + C::tm_dp(h);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          mma_ts(ds, tmem + C::TM_Q + kk * 8, desc_adv(bk, kstep_off(kk, C::HALF_BYTES)), idesc_s,
                 kk > 0);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          mma_ts(ddp, tmem + C::TM_DO + kk * 8, desc_adv(bv, kstep_off(kk, C::HALF_BYTES)),
                 idesc_s, kk > 0);
        tc_commit(bar(QB_SFULL + h));
        if (last_of_item && h == 1) tc_commit(bar(QB_QFREE));
      }
      __syncwarp();
    };
    // dQ += dS_h K_h; then commits
    auto issue_dq = [&](int h, int st, bool acc, int commit0, int commit1) {
      if (elect_one()) {
        const uint64_t bk = desc_adv(m_k0, st * C::STAGE_BYTES + h * 64 * 128);
        const uint32_t a = tmem + C::tm_s(h);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_ts(tmem + C::TM_DQ, a + packed_col(kk), desc_adv(bk, kk * 16 * 128), idesc_dq,
                 (acc || kk > 0) ? 1u : 0u);
        if (commit0 >= 0) tc_commit(bar(commit0));
        if (commit1 >= 0) tc_commit(bar(commit1));
      }
      __syncwarp();
    };
    bool ok = true;
    int g = 0;
    for (int li = 0; ok; ++li) {
      const int w = sched_item(li);
      if (w >= n_items) break;
      const DqItem it = dq_item(p, w);
      ok = mbar_wait_warp(bar(QB_Q), li & 1, abort_flag, 511);  // Q, dO of this item in TMEM
      if (ok) ok = mbar_wait_warp(bar(QB_KVFULL + g % C::KV_STAGES), (g / C::KV_STAGES) & 1,
                                  abort_flag, 512);
      if (!ok) break;
      tc_fence_after();
      issue_s(0, g % C::KV_STAGES, it.n_kv == 1);
      issue_s(1, g % C::KV_STAGES, it.n_kv == 1);
      for (int j = 0; j < it.n_kv && ok; ++j) {
        const int gj = g + j;
        const int st = gj % C::KV_STAGES;
        const int stn = (gj + 1) % C::KV_STAGES;
        const bool more = j + 1 < it.n_kv;
        ok = mbar_wait_warp(bar(QB_PFULL + 0), gj & 1, abort_flag, 513);
        // the previous item's epilogue has read its dQ before this item's
        // first dQ MMA overwrites the accumulator
        if (ok && j == 0 && li > 0)
          ok = mbar_wait_warp(bar(QB_DQFREE), (li - 1) & 1, abort_flag, 517);
        if (!ok) break;
        tc_fence_after();
        issue_dq(0, st, j > 0, -1, -1);
        if (more) {
          ok = mbar_wait_warp(bar(QB_KVFULL + stn), ((gj + 1) / C::KV_STAGES) & 1, abort_flag, 514);
          if (!ok) break;
          tc_fence_after();
          issue_s(0, stn, j + 2 == it.n_kv);
        }
        ok = mbar_wait_warp(bar(QB_PFULL + 1), gj & 1, abort_flag, 515);
        if (!ok) break;
        tc_fence_after();
        issue_dq(1, st, true, QB_KVEMPTY + st, more ? -1 : QB_ACC);
        if (more) issue_s(1, stn, j + 2 == it.n_kv);
      }
      g += it.n_kv;
    }
    if (elect_one()) tc_commit(bar(QB_DRAIN));
    __syncwarp();
    mbar_wait_noabort(bar(QB_DRAIN), 0, 516);
  } else {
    // ------------- elementwise: warpgroup 2h + c owns key columns
    // [64h + 32c, 64h + 32c + 32) of every tile; thread = query row
    const int wg = warp >> 2;
    const int h = wg >> 1, cq = wg & 1;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_base = uint32_t(wq * 32) << 16;
    const float sl2 = p.scale_log2;
    const int col0 = h * 64 + cq * 32;
    const __nv_bfloat16* qsrc = h == 0 ? q : dO;
    // This warpgroup's quarter of the item's Q (h = 0) or dO (h = 1) row:
    // D/2 elements = D/4 words, prefetched one item ahead.
    uint32_t pre[D / 4];
    float pre_nlse2 = 0.0f, pre_ndelta = 0.0f;
    auto prefetch = [&](int w) {
      const DqItem it = dq_item(p, w);
      const int qrow = it.q0 + row;
      const size_t ws_idx = (size_t)it.bh * p.Sq_pad + qrow;  // qrow < Sq_pad always
      pre_nlse2 = p.ws_lse2[ws_idx];    // -LSE * log2(e)
      pre_ndelta = p.ws_delta[ws_idx];  // -D
      const uint4* src =
          reinterpret_cast<const uint4*>(qsrc + ((size_t)it.bh * p.Sq + qrow) * D + cq * (D / 2));
      const bool in = qrow < p.Sq;
#pragma unroll
      for (int v4 = 0; v4 < D / 16; ++v4) {
        const uint4 x = in ? src[v4] : make_uint4(0, 0, 0, 0);
        pre[4 * v4] = x.x;
        pre[4 * v4 + 1] = x.y;
        pre[4 * v4 + 2] = x.z;
        pre[4 * v4 + 3] = x.w;
      }
    };
    if (sched_item(0) < n_items) prefetch(sched_item(0));
    bool ok = true;
    int g = 0, li = 0;
    int prev_w = -1;  // item whose epilogue is still owed
    auto epilogue = [&](int w, int lj) {
      // dQ = acc * scale; warpgroup wg writes columns [wg*D/4, (wg+1)*D/4)
      const DqItem it = dq_item(p, w);
      const int qrow = it.q0 + row;
      if (!__all_sync(0xffffffffu, mbar_wait(bar(QB_ACC), lj & 1, abort_flag, 522))) return false;
      tc_fence_after();
      const bool valid = qrow < p.Sq;
      __nv_bfloat16* dq_row = p.dq + ((size_t)it.bh * p.Sq + (valid ? qrow : 0)) * D + wg * (D / 4);
      if (D / 4 == 32) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + C::TM_DQ + wg * (D / 4), r);
        tmem_wait_ld();
        if (valid) store_row_chunk_bf16(dq_row, r, p.scale);
      } else {  // D = 64: 16 columns per warpgroup
        uint32_t r[16];
        tmem_ld16(tmem + lane_base + C::TM_DQ + wg * (D / 4), r);
        tmem_wait_ld();
        if (valid) {
          uint32_t wv[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            wv[i] = pack_bf16x2(__uint_as_float(r[2 * i]) * p.scale,
                                __uint_as_float(r[2 * i + 1]) * p.scale);
          uint4* d4 = reinterpret_cast<uint4*>(dq_row);
          d4[0] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
          d4[1] = make_uint4(wv[4], wv[5], wv[6], wv[7]);
        }
      }
      tc_fence_before();
      mbar_arrive_warp(bar(QB_DQFREE));
      return true;
    };
    for (; ok; ++li) {
      const int w = sched_item(li);
      if (w >= n_items) break;
      const DqItem it = dq_item(p, w);
      const int qrow = it.q0 + row;
      // Stage this item's Q / dO into TMEM once the previous item's S MMAs
      // have drained, then prefetch the next item's rows.
      if (li > 0) ok = __all_sync(0xffffffffu, mbar_wait(bar(QB_QFREE), (li - 1) & 1, abort_flag, 523));
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        uint32_t wv[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) wv[i] = pre[c * 16 + i];
        tmem_st16(tmem + lane_base + (h == 0 ? C::TM_Q : C::TM_DO) + cq * (D / 4) + c * 16, wv);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive_warp(bar(QB_Q));
      const float nlse2 = pre_nlse2, ndelta = pre_ndelta;
      if (sched_item(li + 1) < n_items) prefetch(sched_item(li + 1));
      // the previous item's dQ, overlapping this item's first S MMAs
      if (prev_w >= 0) {
        ok = epilogue(prev_w, li - 1);
        if (!ok) break;
      }
      for (int j = 0; j < it.n_kv && ok; ++j) {
        const int gj = g + j;
        const int kb = j * 128;
        const bool need_mask = (p.causal && kb + 127 > it.q0) || (kb + 128 > p.Sk);
        int lim = p.Sk - 1 - kb;  // key columns with index > lim are hidden
        if (p.causal) lim = min(lim, qrow - kb);
        ok = mbar_wait(bar(QB_SFULL + h), gj & 1, abort_flag, 521);
        ok = __all_sync(0xffffffffu, ok);  // keep .sync.aligned TMEM ops convergent
        if (!ok) break;
        tc_fence_after();
        // dS = 2^(s*scale*log2e - lse) * (dP - D), packed to bf16 inside this
        // warpgroup's own columns (see packed_col), 16 keys per step.
        auto step = [&](auto mask_tag, int sub) {
          constexpr bool kMask = decltype(mask_tag)::value;
          const int c0 = col0 + sub * 16;
          uint32_t sr[16], dr[16];
          tmem_ld16(tmem + lane_base + C::tm_s(h) + cq * 32 + sub * 16, sr);
          tmem_ld16(tmem + lane_base + C::tm_dp(h) + cq * 32 + sub * 16, dr);
          tmem_wait_ld();
          uint32_t dsk[8];
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            float p0 = ex2_approx(fmaf(__uint_as_float(sr[i]), sl2, nlse2));
            float p1 = ex2_approx(fmaf(__uint_as_float(sr[i + 1]), sl2, nlse2));
            if (kMask) {
              if (c0 + i > lim) p0 = 0.0f;
              if (c0 + i + 1 > lim) p1 = 0.0f;
            }
            dsk[i / 2] = pack_bf16x2(p0 * (__uint_as_float(dr[i]) + ndelta),
                                     p1 * (__uint_as_float(dr[i + 1]) + ndelta));
          }
          tmem_st8(tmem + lane_base + C::tm_s(h) + cq * 32 + sub * 8, dsk);
        };
        if (need_mask) {
          step(std::true_type{}, 0);
          step(std::true_type{}, 1);
        } else {
          step(std::false_type{}, 0);
          step(std::false_type{}, 1);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive_warp(bar(QB_PFULL + h));
      }
      g += it.n_kv;
      prev_w = w;
    }
    if (ok && prev_w >= 0) epilogue(prev_w, li - 1);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TM_COLS);
  }
}

}  // namespace tfb
