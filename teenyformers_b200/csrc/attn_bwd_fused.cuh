// attn_bwd_fused.cuh -- one-kernel flash-attention backward for sm_100a
// (bf16 in/out, fp32 accumulation), the main backward path.
//
// Same gradients as attn_bwd.cuh (flash_attn2.rs:135-279).  One CTA per
// 128-key tile of one KV head loops over the 128-row query tiles of every
// query head of its GQA group and, per query tile j, issues five MMAs:
//   S^T_j  = K Q_j^T                 (SS, M=128 keys, N=128 queries)
//   dP^T_j = V dO_j^T                (SS)
//   dV    += P^T_j dO_j              (A = bf16 P^T packed over S^T in TMEM)
//   dQ_j   = dS_j K                  (SS, A = dS from shared memory, M=128
//                                     queries; result in the dP^T columns)
//   dK    += dS^T_j Q_j              (SS, A = the same shared tile read as
//                                     dS^T, K-major)
// dQ_j leaves through a dedicated warpgroup: TMEM -> registers (which frees
// the columns for dP^T_{j+1}) -> shared memory -> TMA tensor reduce-add
// (fp32) into a [BHq, Sq_pad, D] accumulator in the workspace.  A small
// kernel then scales it into dQ (bf16).  dK/dV stay on chip (deterministic);
// the dQ sum order across key tiles is not fixed (fp32 adds in L2).
//
// MMA issue order per iteration j (tcgen05 MMAs of one thread run in order):
//   S^T_{j+1} | [dS_j] dQ_j, dK_j | [dQ_j read out] dP^T_{j+1} | [P_{j+1}] dV_{j+1}
// so the exponentials of tile j+1 run under dQ_j, dK_j and dP^T_{j+1}.  dQ_j
// goes before dK_j because the chain dS_j -> dQ_j -> read-out -> dP^T_{j+1}
// -> dS_{j+1} sets the pace; dK_j only accumulates.
//
// TMEM (512 columns): S^T/P^T [0,128), dP^T/dQ [128,256),
//                     dV [256,256+D), dK [256+D,256+2D).
// Warps: 0-3 dQ reduction, 4-11 elementwise (two warpgroups, 64 query
// columns each; one TMEM lane = one key row per thread), 12 MMA issuer,
// 13 TMA producer, 14-15 idle.  For D = 128 registers are rebalanced with
// setmaxnreg: the reduction warpgroup holds a whole 128-column dQ row.
#pragma once

#include "attn_bwd.cuh"

namespace tfb {

__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, uint32_t smem_src,
                                                  int c0, int c1) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], "
      "[%1];" ::"l"(reinterpret_cast<uint64_t>(map)),
      "r"(smem_src), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void bulk_wait_group_read1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
// AND of `v` over the `nthreads` threads of named barrier `id` (all of them
// get the same answer, so they take the same branch afterwards).
__device__ __forceinline__ bool named_bar_and(int id, int nthreads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(v)), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}
template <int N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

constexpr int kFusedThreads = 512;
constexpr int kFusedMmaWarp = 12, kFusedTmaWarp = 13;
// setmaxnreg split for D = 128 (launch: 512 threads x 128 registers = the
// whole 64K register file): reduction 160, elementwise 128, MMA/TMA/idle
// warpgroup 96 -> 128*160 + 256*128 + 128*96 = 65536.  D = 64 keeps 128 each.
constexpr int kRegsReduce = 160, kRegsProducer = 96;

template <int D>
struct BwdFusedCfg {
  static constexpr int HALVES = D / 64;
  static constexpr int HALF_BYTES = 128 * 128;
  static constexpr int TILE_BYTES = 128 * D * 2;
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + TILE_BYTES;
  static constexpr int OFF_Q = OFF_V + TILE_BYTES;    // 2 stages
  static constexpr int OFF_DO = OFF_Q + 2 * TILE_BYTES;  // 1 stage
  static constexpr int OFF_DS = OFF_DO + TILE_BYTES;  // dS^T [128 keys][128 queries] bf16
  static constexpr int DS_BYTES = 2 * HALF_BYTES;
  static constexpr int OFF_STG = OFF_DS + DS_BYTES;  // 2 x dQ staging [128 rows][32 fp32], SW128
  static constexpr int STG_BYTES = 2 * 128 * 128;
  static constexpr int OFF_LSE = OFF_STG + STG_BYTES;  // 2 stages x 128 fp32 (-LSE*log2e)
  static constexpr int OFF_DELTA = OFF_LSE + 1024;     // 2 stages x 128 fp32 (-D)
  static constexpr int OFF_BAR = OFF_DELTA + 1024;
  // no alignment slack: the dynamic shared window must start 1024-aligned
  // (checked at kernel entry)
  static constexpr int SMEM_BYTES = OFF_BAR + 256;
  static constexpr uint32_t TM_ST = 0, TM_DPT = 128, TM_DV = 256, TM_DK = 256 + D;
  static constexpr uint32_t TM_COLS = 512;
};

enum BwdFusedBar {
  FB2_KVFULL = 0, FB2_KVEMPTY = 1, FB2_QFULL = 2, FB2_QEMPTY = 4, FB2_DOFULL = 6,
  FB2_DOEMPTY = 7, FB2_SFULL = 8, FB2_PFULL = 9, FB2_DPFULL = 10, FB2_DSSMEM = 11,
  FB2_DQFULL = 12, FB2_DQEMPTY = 13, FB2_ACC = 14, FB2_ACCFREE = 15, FB2_ITEMFULL = 16,
  FB2_ITEMEMPTY = 20, FB2_DRAIN = 24, FB2_COUNT = 25
};
constexpr int kItemRing = 4;      // work items the TMA warp may fetch ahead
constexpr int kItemConsumers = 13;  // MMA warp + 8 elementwise warps + 4 reduction warps

// TMEM column (relative to the operand's base) of the bf16-packed P^T for
// the 16-query K step kk: elementwise warpgroup e packs its 64 query
// columns [64e, 64e+64) into their first 32 columns, 8 per 16 queries.
__device__ __forceinline__ constexpr uint32_t packed_col64(int kk) {
  return uint32_t((kk >> 2) * 64 + (kk & 3) * 8);
}

// Work item w = one 128-key tile of one KV head.  Items go in groups of
// kItemHeadGroup KV heads (their Q/dO and dQ accumulator stay hot in L2 while
// the group runs); within a group key-tile-major, key tile 0 first (the most
// query tiles when causal), so the items handed out last are the lightest.
constexpr int kItemHeadGroup = 8;
struct FusedItem {
  int bh_kv, b, hk, k0, qt_first, qt_per_head, n_tiles;
};
__device__ __forceinline__ FusedItem fused_item(const BwdParams& p, int w) {
  FusedItem it;
  const int per_group = kItemHeadGroup * p.n_kt;
  const int h0 = (w / per_group) * kItemHeadGroup;
  const int gs = min(kItemHeadGroup, p.BHkv - h0);  // heads in this group
  const int local = w - h0 * p.n_kt;
  const int kt = local / gs;
  it.bh_kv = h0 + local % gs;
  it.b = it.bh_kv / p.Hkv;
  it.hk = it.bh_kv % p.Hkv;
  it.k0 = kt * 128;
  it.qt_first = p.causal ? min(kt, p.n_qt) : 0;  // query tile i sees keys iff i >= kt
  it.qt_per_head = p.n_qt - it.qt_first;
  it.n_tiles = (p.Hq / p.Hkv) * it.qt_per_head;
  return it;
}

// Persistent: one CTA per SM takes work items from a global counter (zeroed
// by the prep kernel); the TMA warp fetches them into a small shared ring the
// other roles read.  Tile-level barriers run on a CTA-wide tile count across
// items; per item, the next item's K/V load and first S^T / dP^T MMAs overlap
// the previous item's dK/dV epilogue (its first dV/dK MMA waits until the
// epilogue has read the accumulators out of TMEM).
template <int D>
__global__ void __launch_bounds__(kFusedThreads, 1)
    fa_bwd_fused_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                              const __grid_constant__ CUtensorMap tm_do,
                              const __grid_constant__ CUtensorMap tm_k,
                              const __grid_constant__ CUtensorMap tm_v,
                              const __grid_constant__ CUtensorMap tm_dqacc,
                              const __grid_constant__ CUtensorMap tm_dk,
                              const __grid_constant__ CUtensorMap tm_dv, const BwdParams p) {
  using C = BwdFusedCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw;
  const uint32_t sbase = smem_u32(smem);
  if (sbase & 1023u) {  // uniform over the CTA: nothing has been set up yet
    if (threadIdx.x == 0) atomicCAS(&g_device_status, 0, 600);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + FB2_COUNT);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* item_ring = reinterpret_cast<volatile int*>(tmem_slot + 2);
  auto bar = [&](int i) { return smem_u32(bars + i); };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.Hq / p.Hkv;

  if (threadIdx.x == 0) {
    mbar_init(bar(FB2_KVFULL), 1);
    mbar_init(bar(FB2_KVEMPTY), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(FB2_QFULL + s), 1);
      mbar_init(bar(FB2_QEMPTY + s), 1);
    }
    mbar_init(bar(FB2_DOFULL), 1);
    mbar_init(bar(FB2_DOEMPTY), 1);
    mbar_init(bar(FB2_SFULL), 1);
    mbar_init(bar(FB2_PFULL), 8);  // one arrival per elementwise warp
    mbar_init(bar(FB2_DPFULL), 1);
    mbar_init(bar(FB2_DSSMEM), 8);   // dS tile in shared memory (A of dQ and dK)
    mbar_init(bar(FB2_DQFULL), 1);
    mbar_init(bar(FB2_DQEMPTY), 4);  // one per reduction warp
    mbar_init(bar(FB2_ACC), 1);
    mbar_init(bar(FB2_ACCFREE), 8);
    for (int s = 0; s < kItemRing; ++s) {
      mbar_init(bar(FB2_ITEMFULL + s), 1);
      mbar_init(bar(FB2_ITEMEMPTY + s), kItemConsumers);
    }
    mbar_init(bar(FB2_DRAIN), 1);
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

  // Item k of this CTA, read by a consumer warp from the ring (-1: no more);
  // false when the wait gave up.
  auto take_item = [&](int k, int& w) -> bool {
    const int slot = k % kItemRing;
    if (!mbar_wait_warp(bar(FB2_ITEMFULL + slot), (k / kItemRing) & 1, abort_flag, 640))
      return false;
    w = item_ring[slot];
    __syncwarp();
    if (lane == 0) mbar_arrive(bar(FB2_ITEMEMPTY + slot));
    return true;
  };

  if (warp >= kFusedMmaWarp) {
    if constexpr (D == 128) regs_dec<kRegsProducer>();
    if (warp == kFusedTmaWarp) {
      // ---------------- TMA producer: fetches the items, loads K/V, Q, dO ------
      int kv_loads = 0, issued_q[2] = {0, 0}, issued_do = 0, g = 0;
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int slot = k % kItemRing;
        if (k >= kItemRing)
          ok = mbar_wait_warp(bar(FB2_ITEMEMPTY + slot), ((k / kItemRing) - 1) & 1, abort_flag,
                              601);
        if (!ok) break;
        int w = 0;
        if (lane == 0) {
          w = k == 0 ? (int)blockIdx.x : atomicAdd(p.work_counter, 1) + (int)gridDim.x;
          if (w >= p.n_items) w = -1;
          item_ring[slot] = w;
        }
        w = __shfl_sync(0xffffffffu, w, 0);
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(FB2_ITEMFULL + slot));
        if (w < 0) break;
        const FusedItem it = fused_item(p, w);
        if (it.n_tiles == 0) continue;
        if (kv_loads > 0)
          ok = mbar_wait_warp(bar(FB2_KVEMPTY), (kv_loads - 1) & 1, abort_flag, 602);
        if (!ok) break;
        if (elect_one()) {
          mbar_arrive_expect_tx(bar(FB2_KVFULL), 2 * C::TILE_BYTES);
          for (int hh = 0; hh < C::HALVES; ++hh) {
            tma_load_3d(sbase + C::OFF_K + hh * C::HALF_BYTES, &tm_k, bar(FB2_KVFULL), hh * 64,
                        it.k0, it.bh_kv);
            tma_load_3d(sbase + C::OFF_V + hh * C::HALF_BYTES, &tm_v, bar(FB2_KVFULL), hh * 64,
                        it.k0, it.bh_kv);
          }
        }
        __syncwarp();
        ++kv_loads;
        for (int t = 0; t < it.n_tiles && ok; ++t, ++g) {
          const int st = g & 1, u = g >> 1;
          const int qi = it.qt_first + t % it.qt_per_head;
          const int bh_q = it.b * p.Hq + it.hk * G + t / it.qt_per_head;
          // Q (+ -LSE*log2e, -D) into stage st
          if (u > 0) ok = mbar_wait_warp(bar(FB2_QEMPTY + st), (u - 1) & 1, abort_flag, 603);
          if (!ok) break;
          if (elect_one()) {
            const uint32_t sq = sbase + C::OFF_Q + st * C::TILE_BYTES;
            mbar_arrive_expect_tx(bar(FB2_QFULL + st), C::TILE_BYTES + 1024);
            for (int hh = 0; hh < C::HALVES; ++hh)
              tma_load_3d(sq + hh * C::HALF_BYTES, &tm_q, bar(FB2_QFULL + st), hh * 64,
                          qi * 128, bh_q);
            const size_t ws_off = (size_t)bh_q * p.Sq_pad + (size_t)qi * 128;
            bulk_load(sbase + C::OFF_LSE + st * 512, p.ws_lse2 + ws_off, 512,
                      bar(FB2_QFULL + st));
            bulk_load(sbase + C::OFF_DELTA + st * 512, p.ws_delta + ws_off, 512,
                      bar(FB2_QFULL + st));
          }
          __syncwarp();
          issued_q[st] += 1;
          // dO into its single stage once dV of the previous tile has read it
          if (g > 0) ok = mbar_wait_warp(bar(FB2_DOEMPTY), (g - 1) & 1, abort_flag, 604);
          if (!ok) break;
          if (elect_one()) {
            mbar_arrive_expect_tx(bar(FB2_DOFULL), C::TILE_BYTES);
            for (int hh = 0; hh < C::HALVES; ++hh)
              tma_load_3d(sbase + C::OFF_DO + hh * C::HALF_BYTES, &tm_do, bar(FB2_DOFULL),
                          hh * 64, qi * 128, bh_q);
          }
          __syncwarp();
          issued_do += 1;
        }
      }
      if (!ok) {  // let the copies in flight land before the CTA exits
        if (kv_loads) mbar_wait_noabort(bar(FB2_KVFULL), (kv_loads - 1) & 1, 605);
        for (int s = 0; s < 2; ++s)
          if (issued_q[s]) mbar_wait_noabort(bar(FB2_QFULL + s), (issued_q[s] - 1) & 1, 605);
        if (issued_do) mbar_wait_noabort(bar(FB2_DOFULL), (issued_do - 1) & 1, 605);
      }
    } else if (warp == kFusedMmaWarp) {
      // ---------------- MMA issuer (whole warp, one elected lane issues) --------
      constexpr uint32_t idesc_s = make_idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t idesc_acc = make_idesc_bf16(128, D, 0, 1);
      constexpr uint32_t idesc_dq = make_idesc_bf16(128, D, 1, 1);
      const uint64_t d_k = kmajor_base<C::HALF_BYTES>(sbase + C::OFF_K);
      const uint64_t d_v = kmajor_base<C::HALF_BYTES>(sbase + C::OFF_V);
      const uint64_t d_q0 = kmajor_base<C::HALF_BYTES>(sbase + C::OFF_Q);
      const uint64_t d_do = kmajor_base<C::HALF_BYTES>(sbase + C::OFF_DO);
      const uint64_t m_q0 = mnmajor_base<C::HALF_BYTES>(sbase + C::OFF_Q);
      const uint64_t m_do = mnmajor_base<C::HALF_BYTES>(sbase + C::OFF_DO);
      const uint64_t m_k = mnmajor_base<C::HALF_BYTES>(sbase + C::OFF_K);
      const uint64_t m_ds = mnmajor_base<C::HALF_BYTES>(sbase + C::OFF_DS);
      // D_tm = A B^T over K = D (both K-major), then commit `done`
      auto issue_t = [&](uint32_t d_tm, uint64_t a, uint64_t bq, int done) {
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            mma_ss(d_tm, desc_adv(a, kstep_off(kk, C::HALF_BYTES)),
                   desc_adv(bq, kstep_off(kk, C::HALF_BYTES)), idesc_s, kk > 0);
          tc_commit(bar(done));
        }
        __syncwarp();
      };
      // acc += packed(A_tm) B over K = 128 query rows (B MN-major), then commit
      auto issue_acc = [&](uint32_t acc_tm, uint32_t a_tm, uint64_t bb, bool acc, int done) {
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_ts(acc_tm, a_tm + packed_col64(kk), desc_adv(bb, kk * 16 * 128), idesc_acc,
                   (acc || kk > 0) ? 1u : 0u);
          tc_commit(bar(done));
        }
        __syncwarp();
      };
      // dK += dS^T Q over K = 128 query rows: A = the shared dS^T tile read
      // K-major (queries contiguous), B = Q MN-major; then commit `done`
      const uint64_t d_ds = kmajor_base<C::HALF_BYTES>(sbase + C::OFF_DS);
      auto issue_dk = [&](uint64_t bq, bool acc, int done) {
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_ss(tmem + C::TM_DK, desc_adv(d_ds, kstep_off(kk, C::HALF_BYTES)),
                   desc_adv(bq, kk * 16 * 128), idesc_acc, (acc || kk > 0) ? 1u : 0u);
          tc_commit(bar(done));
        }
        __syncwarp();
      };
      // dQ = dS K over K = 128 keys (A, B MN-major), into the dP^T columns
      auto issue_dq = [&]() {
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_ss(tmem + C::TM_DPT, desc_adv(m_ds, kk * 16 * 128), desc_adv(m_k, kk * 16 * 128),
                   idesc_dq, kk > 0);
          tc_commit(bar(FB2_DQFULL));
        }
        __syncwarp();
      };
      auto qdesc = [&](int g) { return desc_adv(d_q0, (g & 1) * C::TILE_BYTES); };
      bool ok = true;
      int kv_items = 0, g0 = 0;
      for (int k = 0; ok; ++k) {
        int w;
        ok = take_item(k, w);
        if (!ok || w < 0) break;
        const FusedItem item = fused_item(p, w);
        const int n = item.n_tiles;
        if (n == 0) continue;
        ok = mbar_wait_warp(bar(FB2_KVFULL), kv_items & 1, abort_flag, 611);
        if (ok) ok = mbar_wait_warp(bar(FB2_QFULL + (g0 & 1)), (g0 >> 1) & 1, abort_flag, 612);
        if (!ok) break;
        tc_fence_after();
        issue_t(tmem + C::TM_ST, d_k, qdesc(g0), FB2_SFULL);
        // dP^T_0 reuses the dQ columns of the previous item's last tile
        if (g0 > 0) ok = mbar_wait_warp(bar(FB2_DQEMPTY), (g0 - 1) & 1, abort_flag, 613);
        if (ok) ok = mbar_wait_warp(bar(FB2_DOFULL), g0 & 1, abort_flag, 614);
        if (!ok) break;
        tc_fence_after();
        issue_t(tmem + C::TM_DPT, d_v, d_do, FB2_DPFULL);
        // the previous item's dK/dV have left TMEM
        if (kv_items > 0)
          ok = mbar_wait_warp(bar(FB2_ACCFREE), (kv_items - 1) & 1, abort_flag, 615);
        if (ok) ok = mbar_wait_warp(bar(FB2_PFULL), g0 & 1, abort_flag, 616);
        if (!ok) break;
        tc_fence_after();
        issue_acc(tmem + C::TM_DV, tmem + C::TM_ST, m_do, false, FB2_DOEMPTY);
        for (int it = 0; it < n && ok; ++it) {
          const int g = g0 + it;
          const bool more = it + 1 < n;
          if (more) {
            ok = mbar_wait_warp(bar(FB2_QFULL + ((g + 1) & 1)), ((g + 1) >> 1) & 1, abort_flag,
                                617);
            if (!ok) break;
            tc_fence_after();
            issue_t(tmem + C::TM_ST, d_k, qdesc(g + 1), FB2_SFULL);
          }
          ok = mbar_wait_warp(bar(FB2_DSSMEM), g & 1, abort_flag, 618);
          if (!ok) break;
          tc_fence_after();
          // dQ first: it is on the dependency chain (its read-out frees the
          // columns of dP^T_{g+1}); dK only accumulates
          issue_dq();
          issue_dk(desc_adv(m_q0, (g & 1) * C::TILE_BYTES), it > 0, FB2_QEMPTY + (g & 1));
          if (!more) {
            if (elect_one()) {
              tc_commit(bar(FB2_KVEMPTY));  // S^T, dP^T, dQ of this item are all issued
              tc_commit(bar(FB2_ACC));
            }
            __syncwarp();
          } else {
            ok = mbar_wait_warp(bar(FB2_DQEMPTY), g & 1, abort_flag, 619);
            if (ok) ok = mbar_wait_warp(bar(FB2_DOFULL), (g + 1) & 1, abort_flag, 620);
            if (!ok) break;
            tc_fence_after();
            issue_t(tmem + C::TM_DPT, d_v, d_do, FB2_DPFULL);
            ok = mbar_wait_warp(bar(FB2_PFULL), (g + 1) & 1, abort_flag, 621);
            if (!ok) break;
            tc_fence_after();
            issue_acc(tmem + C::TM_DV, tmem + C::TM_ST, m_do, true, FB2_DOEMPTY);
          }
        }
        ++kv_items;
        g0 += n;
      }
      if (elect_one()) tc_commit(bar(FB2_DRAIN));
      __syncwarp();
      mbar_wait_noabort(bar(FB2_DRAIN), 0, 622);
    }
  } else if (warp >= 4) {
    // ------------- elementwise: warpgroup e owns query columns [64e, 64e+64);
    // thread = key row
    const int ewg = (warp - 4) >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_base = uint32_t(wq * 32) << 16;
    const float sl2 = p.scale_log2;
    const int col0 = ewg * 64;
    // dS^T row `row` in the SW128 tile read by the dQ MMA (MN-major) and the
    // dK MMA (K-major): half ewg, 16-byte chunk c of the row at physical chunk
    // c ^ (row & 7)
    const uint32_t ds_row = sbase + C::OFF_DS + ewg * C::HALF_BYTES + row * 128;
    const bool epi_issuer = (warp & 3) == 0 && lane == 0;  // first thread of the warpgroup
    bool ok = true;
    int kv_items = 0, g0 = 0;
    for (int k = 0; ok; ++k) {
      int w;
      ok = take_item(k, w);
      if (!ok || w < 0) break;
      const FusedItem item = fused_item(p, w);
      const int key = item.k0 + row;
      const bool valid = key < p.Sk;
      __nv_bfloat16* out_row =
          (ewg == 0 ? p.dv : p.dk) + ((size_t)item.bh_kv * p.Sk + (valid ? key : 0)) * D;
      if (item.n_tiles == 0) {  // keys no query sees: zero gradients
        if (valid) {
          uint4* a4 = reinterpret_cast<uint4*>(out_row);
          for (int v4 = 0; v4 < D / 8; ++v4) a4[v4] = make_uint4(0, 0, 0, 0);
        }
        continue;
      }
      for (int it = 0; it < item.n_tiles && ok; ++it) {
        const int g = g0 + it;
        const int st = g & 1;
        const int qi = item.qt_first + it % item.qt_per_head;
        const float4* s_lse = reinterpret_cast<const float4*>(smem + C::OFF_LSE + st * 512);
        const float4* s_delta = reinterpret_cast<const float4*>(smem + C::OFF_DELTA + st * 512);
        const bool diag = p.causal && qi * 128 < item.k0 + 127;
        const int qlim = key - qi * 128;  // query columns with index < qlim are hidden (k > q)
        ok = mbar_wait(bar(FB2_SFULL), g & 1, abort_flag, 631);
        if (ok) ok = mbar_wait(bar(FB2_QFULL + st), (g >> 1) & 1, abort_flag, 632);
        ok = __all_sync(0xffffffffu, ok);  // keep .sync.aligned TMEM ops convergent
        if (!ok) break;
        tc_fence_after();
        // Phase 1: P^T = 2^(s*scale*log2e - lse), 16 queries per step, packed to
        // bf16 over columns already read; fp32 P kept for phase 2.  The next
        // step's TMEM load is in flight while a step computes (the packed
        // store of step s, columns [8s, 8s+8), never overlaps the load of
        // step s+1, columns [16s+16, 16s+32)).
        float pf[64];
        uint32_t sr[2][16];
        auto p_step = [&](auto mask_tag, int sub) {
          constexpr bool kMask = decltype(mask_tag)::value;
          const int c0 = col0 + sub * 16;
          tmem_wait_ld();
          if (sub < 3) tmem_ld16(tmem + lane_base + C::TM_ST + c0 + 16, sr[(sub + 1) & 1]);
          const uint32_t(&cur)[16] = sr[sub & 1];
          uint32_t pk[8];
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4) {
            const float4 l4 = s_lse[c0 / 4 + v4];  // -lse2
            const float nl[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int i = v4 * 4 + e;
              float pe = ex2_approx(fmaf(__uint_as_float(cur[i]), sl2, nl[e]));
              if (kMask && c0 + i < qlim) pe = 0.0f;
              pf[sub * 16 + i] = pe;
            }
            pk[2 * v4] = pack_bf16x2(pf[sub * 16 + 4 * v4], pf[sub * 16 + 4 * v4 + 1]);
            pk[2 * v4 + 1] = pack_bf16x2(pf[sub * 16 + 4 * v4 + 2], pf[sub * 16 + 4 * v4 + 3]);
          }
          tmem_st8(tmem + lane_base + C::TM_ST + col0 + sub * 8, pk);
        };
        tmem_ld16(tmem + lane_base + C::TM_ST + col0, sr[0]);
        if (diag) {
#pragma unroll
          for (int sub = 0; sub < 4; ++sub) p_step(std::true_type{}, sub);
        } else {
#pragma unroll
          for (int sub = 0; sub < 4; ++sub) p_step(std::false_type{}, sub);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive_warp(bar(FB2_PFULL));
        // Phase 2: dS^T = P^T (dP^T - D), bf16 into the shared dS tile (A of
        // dQ and dK).
        ok = __all_sync(0xffffffffu, mbar_wait(bar(FB2_DPFULL), g & 1, abort_flag, 633));
        if (!ok) break;
        tc_fence_after();
        uint32_t dr[2][16];
        tmem_ld16(tmem + lane_base + C::TM_DPT + col0, dr[0]);
#pragma unroll
        for (int sub = 0; sub < 4; ++sub) {
          const int c0 = col0 + sub * 16;
          tmem_wait_ld();
          if (sub < 3) tmem_ld16(tmem + lane_base + C::TM_DPT + c0 + 16, dr[(sub + 1) & 1]);
          const uint32_t(&cur)[16] = dr[sub & 1];
          uint32_t dk[8];
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4) {
            const float4 d4 = s_delta[c0 / 4 + v4];  // -D
            const float nd[4] = {d4.x, d4.y, d4.z, d4.w};
            float dsv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
              dsv[e] = pf[sub * 16 + v4 * 4 + e] * (__uint_as_float(cur[v4 * 4 + e]) + nd[e]);
            dk[2 * v4] = pack_bf16x2(dsv[0], dsv[1]);
            dk[2 * v4 + 1] = pack_bf16x2(dsv[2], dsv[3]);
          }
          const uint32_t ch = uint32_t(2 * sub);
          st_shared_v4(ds_row + ((ch ^ uint32_t(row & 7)) << 4), dk[0], dk[1], dk[2], dk[3]);
          st_shared_v4(ds_row + (((ch + 1) ^ uint32_t(row & 7)) << 4), dk[4], dk[5], dk[6],
                       dk[7]);
        }
        // dQ and dK read the shared tile; dQ overwrites the dP^T columns read
        // above (tcgen05.wait::ld done), hence the tcgen05 fence as well
        tc_fence_before();
        fence_proxy_async_smem();
        mbar_arrive_warp(bar(FB2_DSSMEM));
      }
      if (!ok) break;
      // ---- epilogue: warpgroup 0 writes dV, 1 writes dK (= acc * scale).  Each
      // 64-column half goes bf16 into this warpgroup's half of the dS tile
      // (free: the item's last dQ MMA has read it), laid out as the output
      // map's 128-byte swizzle, and leaves in one TMA tensor store (rows past
      // Sk are clipped by the map).  The accumulators are released once read.
      ok = __all_sync(0xffffffffu, mbar_wait(bar(FB2_ACC), kv_items & 1, abort_flag, 634));
      if (!ok) break;
      tc_fence_after();
      const uint32_t acc_col = ewg == 0 ? C::TM_DV : C::TM_DK;
      const float mul = ewg == 0 ? 1.0f : p.scale;
      const CUtensorMap* out_map = ewg == 0 ? &tm_dv : &tm_dk;
      const uint32_t stage = sbase + C::OFF_DS + ewg * C::HALF_BYTES;
      const uint32_t stage_row = stage + row * 128;
      for (int hh = 0; hh < C::HALVES; ++hh) {
        if (hh > 0) {  // the previous half's store has read the staging tile
          if (epi_issuer) bulk_wait_group_read0();
          named_bar_sync(2 + ewg, 128);
        }
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem + lane_base + acc_col + hh * 64 + c * 32, r);
          tmem_wait_ld();
          if (hh == C::HALVES - 1 && c == 1) {
            tc_fence_before();
            mbar_arrive_warp(bar(FB2_ACCFREE));
          }
          uint32_t wv[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            wv[i] = pack_bf16x2(__uint_as_float(r[2 * i]) * mul, __uint_as_float(r[2 * i + 1]) * mul);
#pragma unroll
          for (int v = 0; v < 4; ++v)
            st_shared_v4(stage_row + ((uint32_t(c * 4 + v) ^ uint32_t(row & 7)) << 4), wv[4 * v],
                         wv[4 * v + 1], wv[4 * v + 2], wv[4 * v + 3]);
        }
        fence_proxy_async_smem();
        named_bar_sync(2 + ewg, 128);
        if (epi_issuer) {
          tma_store_3d(out_map, stage, hh * 64, item.k0, item.bh_kv);
          bulk_commit_group();
        }
      }
      // the dS tile is rewritten by the next item's first tile: its stores must
      // have read the staging first
      if (epi_issuer) bulk_wait_group_read0();
      named_bar_sync(2 + ewg, 128);
      ++kv_items;
      g0 += item.n_tiles;
    }
    if (epi_issuer) bulk_wait_group0();  // dK / dV stores complete before the CTA exits
  } else {
    // ------------- dQ reduction: thread = query row of the tile
    if constexpr (D == 128) regs_inc<kRegsReduce>();
    const int row = warp * 32 + lane;
    const uint32_t lane_base = uint32_t(warp * 32) << 16;
    const uint32_t stg_row = sbase + C::OFF_STG + row * 128;
    bool ok = true;
    int g = 0;
    for (int k = 0; ok; ++k) {
      int w;
      ok = named_bar_and(1, 128, take_item(k, w));
      if (!ok || w < 0) break;
      const FusedItem item = fused_item(p, w);
      for (int t = 0; t < item.n_tiles && ok; ++t, ++g) {
        const int qi = item.qt_first + t % item.qt_per_head;
        const int bh_q = item.b * p.Hq + item.hk * G + t / item.qt_per_head;
        const int grow0 = bh_q * p.Sq_pad + qi * 128;  // first accumulator row of the tile
        // the four warps agree before any of them reaches the named barriers below
        ok = named_bar_and(1, 128, mbar_wait(bar(FB2_DQFULL), g & 1, abort_flag, 641));
        if (!ok) break;
        tc_fence_after();
        uint32_t acc[D];
#pragma unroll
        for (int c = 0; c < D / 32; ++c)
          tmem_ld32(tmem + lane_base + C::TM_DPT + c * 32,
                    *reinterpret_cast<uint32_t(*)[32]>(&acc[c * 32]));
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive_warp(bar(FB2_DQEMPTY));
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          // chunk c of every tile uses buffer c & 1 (D / 32 chunks per tile is even)
          const uint32_t buf = uint32_t(c & 1) * (C::STG_BYTES / 2);
          // the reduction issued two chunks ago (same buffer) must have read it
          if (threadIdx.x == 0) bulk_wait_group_read1();
          named_bar_sync(1, 128);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            st_shared_v4(stg_row + buf + ((uint32_t(j) ^ uint32_t(row & 7)) << 4),
                         acc[c * 32 + 4 * j], acc[c * 32 + 4 * j + 1], acc[c * 32 + 4 * j + 2],
                         acc[c * 32 + 4 * j + 3]);
          fence_proxy_async_smem();
          named_bar_sync(1, 128);
          if (threadIdx.x == 0) {
            tma_reduce_add_2d(&tm_dqacc, sbase + C::OFF_STG + buf, c * 32, grow0);
            bulk_commit_group();
          }
        }
      }
    }
    if (threadIdx.x == 0) bulk_wait_group0();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TM_COLS);
  }
}

// dQ (bf16) = scale * accumulator rows [bh, s < Sq] of [BHq, Sq_pad, D] fp32;
// 8 elements per thread, grid-stride.
template <int D>
__global__ void __launch_bounds__(256)
    fa_bwd_dq_convert_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dq,
                             int Sq, int Sq_pad, long long rows, float scale) {
  constexpr int VPR = D / 8;
  const long long total = rows * VPR;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / VPR;
    const int c = (int)(i % VPR);
    const long long bh = r / Sq, s = r % Sq;
    const float4* src = reinterpret_cast<const float4*>(acc + ((bh * Sq_pad + s) * D + c * 8));
    const float4 a = src[0], b4 = src[1];
    uint4 w;
    w.x = pack_bf16x2(a.x * scale, a.y * scale);
    w.y = pack_bf16x2(a.z * scale, a.w * scale);
    w.z = pack_bf16x2(b4.x * scale, b4.y * scale);
    w.w = pack_bf16x2(b4.z * scale, b4.w * scale);
    reinterpret_cast<uint4*>(dq + r * D)[c] = w;
  }
}

}  // namespace tfb
