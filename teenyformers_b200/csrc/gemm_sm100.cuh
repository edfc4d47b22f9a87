// gemm_sm100.cuh -- bf16 GEMM on the 5th-generation tensor cores with the
// Llama block's elementwise work fused into its epilogue.
//
//   acc[M, N] = A[M, K] * B[N, K]^T      (bf16 in, fp32 accumulate in TMEM)
//
// A is row-major [M, K] (activations; or the attention output in its
// [B, H, S, 128] layout, read as the [B*S, H*128] matrix merge_heads would
// build -- the merge is folded into the A loads), B is row-major [N, K] (an
// nn.Linear weight [out, in]), so both operands are K-major.  In the
// reference block these GEMMs are teeny-core Linear calls
// (src/layers/attention.rs:83-148, src/layers/ffn.rs:47-56,
// src/layers/llama_block.rs:55-65); the epilogues replace the kernels that
// follow them:
//   STORE      C = acc as bf16 (+ a residual R: C = bf16(acc) + R)  (Linear)
//   SWIGLU     B's rows hold gate and up interleaved in 128-row blocks
//              (tile n = [gate rows 128n.. | up rows 128n..]);
//              C[M, N/2] = silu(gate) * up                    (swiglu.rs:56-95)
//   QKV_ROPE   B = [Wq; Wk; Wv]; each 128-column head of acc is rotated
//              (Q and K heads; rope.rs:57-96 angles, interleaved or rotate-
//              half pairs) and written to its [B, H, S, 128] place
//              (transpose_heads.rs:49-70), V heads copied
//   PUSH       tensor-parallel reduce-scatter by push: the rows of acc that
//              rank o owns (o = row / slice) go straight into rank o's
//              receive buffer, slot [this rank], over NVLink (plain peer
//              stores), so the transfer overlaps the GEMM tile by tile;
//              the all-reduce kernel then sums its own slice from local memory
//
// Structure: persistent clusters of two CTAs (cta_group::2), one CTA per SM,
// 256 x 256 output tiles in grouped order (group_m row blocks share the
// weight's column blocks in L2).  CTA r of a pair holds A rows 128r.. and B
// rows 128r.. of the tile; the even CTA's MMAs read both CTAs' shared memory
// and write both CTAs' TMEM (each CTA's 128 lanes = its 128 output rows), so
// per k-block an SM stages 32 KB for 128 x 256 x 64 of work.
//   warp 0     TMA producer (both CTAs): its A and B halves of a k-block into
//              a 6-stage ring (32 KB per stage, 128-byte swizzle); the copies
//              are counted on the even CTA's stage barrier
//   warp 1     MMA issuer (even CTA): 4 x tcgen05.mma.cta_group::2 256x256x16
//              per k-block into one of two 256-column TMEM accumulators (512
//              columns: the epilogue of tile i overlaps the main loop of
//              tile i+1); commits are multicast to both CTAs
//   warps 2-5  epilogue (both CTAs): warp w reads TMEM lanes 32*(w%4).. (its
//              32 rows), converts, applies the epilogue, stages its rows in
//              its own 8 KB swizzled shared-memory area and writes them back
//              with coalesced 16-byte stores (128-byte row segments).
// No load uses cluster multicast.  Every wait is bounded (kWaitTimeoutNs,
// then a status code 9xx and an abort that drains issued copies and MMAs
// before TMEM is freed).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "norm_act.cuh"
#include "sm100.cuh"

namespace tfb {

enum GemmEpilogue : int {
  GEMM_EPI_STORE = 0,
  GEMM_EPI_SWIGLU = 1,
  GEMM_EPI_QKV_ROPE = 2,
  GEMM_EPI_PUSH = 3,
};

constexpr int kGemmBM = 128, kGemmBN = 256, kGemmBK = 64;  // per-CTA rows, tile columns, k-block
constexpr int kGemmThreads = 192;
constexpr int kGemmMaxPeers = 8;
constexpr int kGemmHeadDim = 128;  // QKV_ROPE and the heads-layout A operand

struct GemmParams {
  int M, N, K;  // acc is [M, N]
  int n_mblk, n_nblk, n_kblk, n_tiles, group_m;
  // A in [B, H, S, 128] layout (a_heads = 1): A row m = (b, s) with
  // b = m / a_seq, column k = (h, d) with h = k / 128
  int a_heads, a_seq, a_n_heads;
  // STORE / SWIGLU output, row stride ld_out elements; STORE adds `residual`
  // ([M, N], row stride ld_out) when it is non-null
  __nv_bfloat16* out;
  long long ld_out;
  const __nv_bfloat16* residual;
  // QKV_ROPE: outputs [B, H, S, 128]; rope_cs = [seq, 64] (cos, sin) pairs or
  // null (no rotation); rope_style 0 = interleaved pairs, 1 = rotate-half
  __nv_bfloat16* q_out;
  __nv_bfloat16* k_out;
  __nv_bfloat16* v_out;
  const float4* rope_cs;
  int seq, n_q_heads, n_kv_heads, rope_style;
  // PUSH: receive buffer of every rank ([world, slice_rows, N] each)
  __nv_bfloat16* peer_out[kGemmMaxPeers];
  int rank, world, slice_rows;
  // the walk over tiles starts at tile tile_rotate (0 <= tile_rotate < n_tiles)
  // and wraps: PUSH gives each rank a different starting owner so the ranks'
  // peer stores spread over every NVLink destination instead of all ranks
  // writing into one owner at a time
  int tile_rotate;
};

__device__ __forceinline__ void gemm_sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                            uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}
__device__ __forceinline__ uint4 gemm_lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// Tile t -> (row block, column block): groups of group_m row blocks walk all
// column blocks, row block fastest, so the CTAs running at once share a few
// column blocks of B and a few row blocks of A in L2.
__device__ __forceinline__ void gemm_tile(const GemmParams& p, int t, int& mb, int& nb) {
  t += p.tile_rotate;
  if (t >= p.n_tiles) t -= p.n_tiles;
  const int per_group = p.group_m * p.n_nblk;
  const int g = t / per_group;
  const int m_first = g * p.group_m;
  const int gm = min(p.group_m, p.n_mblk - m_first);
  const int local = t - g * per_group;
  mb = m_first + local % gm;
  nb = local / gm;
}

__device__ __forceinline__ float gemm_silu(float g) { return g / (1.0f + __expf(-g)); }

// Writes this warp's 32 staged rows of 64 bf16 (128 B each, 16-byte chunks
// XOR-swizzled by row) to dst rows row0.. with row stride ld; rows at or past
// rows_valid and 8-column groups at or past cols_valid are skipped.  With
// res_row0, the same-shaped bf16 residual is added (fp32 add of the two bf16
// values, rounded once more: what the unfused GEMM + add computes).
__device__ __forceinline__ void gemm_store_rows64(uint32_t stg, __nv_bfloat16* dst_row0,
                                                  const __nv_bfloat16* res_row0, long long ld,
                                                  int lane, int rows_valid, int cols_valid) {
  const int jj = lane & 7;
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int rr = it * 4 + (lane >> 3);
    uint4 v = gemm_lds128(stg + rr * 128 + ((jj ^ (rr & 7)) << 4));
    if (rr < rows_valid && jj * 8 < cols_valid) {
      if (res_row0) {
        float a[8], r[8];
        bf16x8_to_f32(v, a);
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(res_row0 + (long long)rr * ld + jj * 8), r);
#pragma unroll
        for (int e = 0; e < 8; ++e) a[e] += r[e];
        v = f32_to_bf16x8(a);
      }
      *reinterpret_cast<uint4*>(dst_row0 + (long long)rr * ld + jj * 8) = v;
    }
  }
}

// ---- CTA pairs (cta_group::2): a 2-CTA cluster computes a 256 x 256 tile;
// each CTA holds 128 rows of the A tile and 128 rows (half) of the B tile,
// and the even CTA issues MMAs that read both CTAs' shared memory and write
// both CTAs' TMEM (each CTA's 128 lanes hold its 128 output rows).
constexpr int kPairStages = 6;

struct GemmPairCfg {
  static constexpr int A_BYTES = 128 * kGemmBK * 2;  // this CTA's 128 A rows
  static constexpr int B_BYTES = 128 * kGemmBK * 2;  // this CTA's 128 B rows
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int OFF_EPI = kPairStages * STAGE_BYTES;
  static constexpr int EPI_WARP_BYTES = 32 * 256;
  static constexpr int OFF_BAR = OFF_EPI + 4 * EPI_WARP_BYTES;
  static constexpr int SMEM_BYTES = OFF_BAR + 256;
  static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;
  static constexpr int TM_COLS = 2 * kGemmBN;
};
static_assert(GemmPairCfg::SMEM_ALLOC <= 232448, "paired GEMM shared memory exceeds the limit");

enum {
  PB_FULL = 0,
  PB_EMPTY = kPairStages,
  PB_AFULL = 2 * kPairStages,
  PB_AEMPTY = 2 * kPairStages + 2,
  PB_DRAIN = 2 * kPairStages + 4,
  PB_COUNT = 2 * kPairStages + 5
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// All threads of both CTAs (release / acquire at cluster scope).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_cta(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
// TMA loads into this CTA's shared memory whose completion is counted on the
// even CTA's mbarrier (bar_cluster, a cluster address); no multicast.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t smem_dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d_pair(uint32_t smem_dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// D (both CTAs' TMEM) (+)= A (both CTAs' smem) * B (both CTAs' smem), issued
// by the even CTA.  The disable-output-lane mask is all zero.
__device__ __forceinline__ void mma_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;"
      "\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(z)
      : "memory");
}
// Arrive on the mbarrier at this offset in every CTA of `mask` once all
// previously issued pair MMAs have completed.
__device__ __forceinline__ void tc_commit_pair_mc(uint32_t bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar),
      "h"(mask)
      : "memory");
}
__device__ __forceinline__ void tc_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

// Epilogue of one accumulator tile for one warp: `acc` addresses this warp's
// TMEM lane quarter of the tile's 256 accumulator columns, rows row0..row0+31
// of the output, column block nb; `stg` is the warp's 8 KB staging area.
// release_acc() runs right after the tile's last TMEM load, so the MMA warp
// can reuse the accumulator while the stores drain.
template <int EPI, class Release>
__device__ __forceinline__ void gemm_epilogue_warp(const GemmParams& p, uint32_t acc, int row0,
                                                   int nb, int lane, uint32_t stg,
                                                   Release&& release_acc) {
  if (row0 >= p.M) {  // a tile half past the last row (256-row tiles): nothing to write
    release_acc();
    return;
  }
  if constexpr (EPI == GEMM_EPI_STORE || EPI == GEMM_EPI_PUSH) {
    long long ld;
    __nv_bfloat16* dst_row0;
    const __nv_bfloat16* res_row0 = nullptr;
    if constexpr (EPI == GEMM_EPI_STORE) {
      ld = p.ld_out;
      dst_row0 = p.out + (long long)row0 * ld;
      if (p.residual) res_row0 = p.residual + (long long)row0 * ld;
    } else {
      // rank `owner` keeps rows [owner * slice, (owner + 1) * slice); ours go
      // to its slot [rank] (rows rank * slice.. of its receive buffer)
      ld = p.N;
      const int owner = row0 / p.slice_rows;
      dst_row0 =
          p.peer_out[owner] + ((long long)(p.rank - owner) * p.slice_rows + row0) * ld;
    }
    const int rows_valid = p.M - row0;
    for (int c = 0; c < kGemmBN / 64; ++c) {
      uint32_t r0[32], r1[32];
      tmem_ld32(acc + c * 64, r0);
      tmem_ld32(acc + c * 64 + 32, r1);
      tmem_wait_ld();
      if (c == kGemmBN / 64 - 1) release_acc();
      const uint32_t sb = stg + (c & 1) * 4096;
#pragma unroll
      for (int jc = 0; jc < 8; ++jc) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int k = 8 * jc + 2 * e;
          const float lo = __uint_as_float(k < 32 ? r0[k] : r1[k - 32]);
          const float hi = __uint_as_float(k + 1 < 32 ? r0[k + 1] : r1[k + 1 - 32]);
          w[e] = pack_bf16x2(lo, hi);
        }
        gemm_sts128(sb + lane * 128 + ((jc ^ (lane & 7)) << 4), w[0], w[1], w[2], w[3]);
      }
      __syncwarp();
      const int col0 = nb * kGemmBN + c * 64;
      gemm_store_rows64(sb, dst_row0 + col0, res_row0 ? res_row0 + col0 : nullptr, ld, lane,
                        rows_valid, p.N - col0);
      __syncwarp();
    }
  } else if constexpr (EPI == GEMM_EPI_SWIGLU) {
    // acc columns 0..127 = gate, 128..255 = up of output columns 128 nb..
    const int n_out = p.N / 2;
    const int rows_valid = p.M - row0;
    __nv_bfloat16* dst_row0 = p.out + (long long)row0 * p.ld_out;
    for (int c = 0; c < 2; ++c) {
      const uint32_t sb = stg + (c & 1) * 4096;
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t gr[32], ur[32];
        tmem_ld32(acc + c * 64 + hh * 32, gr);
        tmem_ld32(acc + 128 + c * 64 + hh * 32, ur);
        tmem_wait_ld();
        if (c == 1 && hh == 1) release_acc();
#pragma unroll
        for (int jc = 0; jc < 4; ++jc) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int k = 8 * jc + 2 * e;
            const float lo = gemm_silu(__uint_as_float(gr[k])) * __uint_as_float(ur[k]);
            const float hi =
                gemm_silu(__uint_as_float(gr[k + 1])) * __uint_as_float(ur[k + 1]);
            w[e] = pack_bf16x2(lo, hi);
          }
          const int js = hh * 4 + jc;
          gemm_sts128(sb + lane * 128 + ((js ^ (lane & 7)) << 4), w[0], w[1], w[2], w[3]);
        }
      }
      __syncwarp();
      const int col0 = nb * 128 + c * 64;
      gemm_store_rows64(sb, dst_row0 + col0, nullptr, p.ld_out, lane, rows_valid,
                        n_out - col0);
      __syncwarp();
    }
  } else {
    // QKV_ROPE: the tile's two 128-column heads; rows row0..row0+31 are
    // positions s0.. of one sequence (seq is a multiple of 128)
    const int bidx = row0 / p.seq, s0 = row0 - bidx * p.seq;
    const float4* cs_row = p.rope_cs ? p.rope_cs + (long long)(s0 + lane) * 32 : nullptr;
    const int last_hs = (nb * kGemmBN + 128 < p.N) ? 1 : 0;
    for (int hs = 0; hs <= last_hs; ++hs) {
      const int hidx = (nb * kGemmBN) / 128 + hs;
      __nv_bfloat16* base;
      int H, h;
      bool rot;
      if (hidx < p.n_q_heads) {
        base = p.q_out, H = p.n_q_heads, h = hidx, rot = true;
      } else if (hidx < p.n_q_heads + p.n_kv_heads) {
        base = p.k_out, H = p.n_kv_heads, h = hidx - p.n_q_heads, rot = true;
      } else {
        base = p.v_out, H = p.n_kv_heads, h = hidx - p.n_q_heads - p.n_kv_heads, rot = false;
      }
      rot = rot && cs_row != nullptr;
      const bool half = p.rope_style == 1;
      for (int pp = 0; pp < 2; ++pp) {
        // rotate-half: x0 = columns 32pp.., x1 = columns 64 + 32pp.. (pair i = (x0[i], x1[i]));
        // interleaved: x0 | x1 = columns 64pp..64pp+63 (pair i = elements 2i, 2i+1)
        uint32_t r0[32], r1[32];
        const uint32_t a0 = acc + hs * 128 + (half ? pp * 32 : pp * 64);
        tmem_ld32(a0, r0);
        tmem_ld32(a0 + (half ? 64 : 32), r1);
        tmem_wait_ld();
        if (hs == last_hs && pp == 1) release_acc();
        float x0[32], x1[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          x0[e] = __uint_as_float(r0[e]);
          x1[e] = __uint_as_float(r1[e]);
        }
        if (rot) {
#pragma unroll
          for (int i4 = 0; i4 < 16; ++i4) {
            const float4 cs = cs_row[pp * 16 + i4];  // pairs k = 32pp + 2 i4, +1
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int i = 2 * i4 + e;
              const float c = e ? cs.z : cs.x, sn = e ? cs.w : cs.y;
              if (half) {
                const float a = x0[i], bb = x1[i];
                x0[i] = a * c - bb * sn;
                x1[i] = a * sn + bb * c;
              } else {
                float& a = (2 * i < 32) ? x0[2 * i] : x1[2 * i - 32];
                float& bb = (2 * i + 1 < 32) ? x0[2 * i + 1] : x1[2 * i + 1 - 32];
                const float av = a, bv = bb;
                a = av * c - bv * sn;
                bb = av * sn + bv * c;
              }
            }
          }
        }
        const int ch0 = half ? pp * 4 : pp * 8, ch1 = half ? 8 + pp * 4 : pp * 8 + 4;
#pragma unroll
        for (int jc = 0; jc < 4; ++jc) {
          gemm_sts128(stg + lane * 256 + (((ch0 + jc) ^ (lane & 7)) << 4),
                      pack_bf16x2(x0[8 * jc], x0[8 * jc + 1]),
                      pack_bf16x2(x0[8 * jc + 2], x0[8 * jc + 3]),
                      pack_bf16x2(x0[8 * jc + 4], x0[8 * jc + 5]),
                      pack_bf16x2(x0[8 * jc + 6], x0[8 * jc + 7]));
          gemm_sts128(stg + lane * 256 + (((ch1 + jc) ^ (lane & 7)) << 4),
                      pack_bf16x2(x1[8 * jc], x1[8 * jc + 1]),
                      pack_bf16x2(x1[8 * jc + 2], x1[8 * jc + 3]),
                      pack_bf16x2(x1[8 * jc + 4], x1[8 * jc + 5]),
                      pack_bf16x2(x1[8 * jc + 6], x1[8 * jc + 7]));
        }
      }
      __syncwarp();
      // 32 consecutive positions of head h: one contiguous 8 KB run
      __nv_bfloat16* dst = base + (((long long)bidx * H + h) * p.seq + s0) * kGemmHeadDim;
      const int jc = lane & 15;
#pragma unroll
      for (int it = 0; it < 16; ++it) {
        const int rr = it * 2 + (lane >> 4);
        const uint4 v = gemm_lds128(stg + rr * 256 + ((jc ^ (rr & 7)) << 4));
        *reinterpret_cast<uint4*>(dst + rr * kGemmHeadDim + jc * 8) = v;
      }
      __syncwarp();
    }
  }
}

// The GEMM kernel (structure above); p.n_mblk counts 256-row blocks.
template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_sm100_pair_kernel(const __grid_constant__ CUtensorMap tm_a,
                                const __grid_constant__ CUtensorMap tm_b, const GemmParams p) {
  using C = GemmPairCfg;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;  // same offset in both CTAs
  uint8_t* sptr = smem_raw + (sbase - raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sptr + C::OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + PB_COUNT);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  auto bar = [&](int i) { return smem_u32(bars + i); };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const bool leader = crank == 0;
  const int pair = (int)cluster_id_x(), n_pairs = (int)cluster_count_x();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(bar(PB_FULL + s), 1);
      mbar_init(bar(PB_EMPTY + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(PB_AFULL + b), 1);
      mbar_init(bar(PB_AEMPTY + b), 8);  // 4 epilogue warps x 2 CTAs
    }
    mbar_init(bar(PB_DRAIN), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), C::TM_COLS);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised before any remote signal
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ===================== TMA producer (both CTAs) =====================
    const uint32_t full0 = mapa_cta(bar(PB_FULL), 0);  // the even CTA's FULL[0]
    int g = 0;
    bool ok = true;
    for (int t = pair; t < p.n_tiles && ok; t += n_pairs) {
      int mb, nb;
      gemm_tile(p, t, mb, nb);
      const int m0 = mb * 256 + (int)crank * 128;  // this CTA's A rows
      const int n0 = nb * 256 + (int)crank * 128;  // this CTA's B rows
      for (int kb = 0; kb < p.n_kblk; ++kb, ++g) {
        const int s = g % kPairStages, u = g / kPairStages;
        if (u > 0) ok = mbar_wait_warp(bar(PB_EMPTY + s), (u - 1) & 1, abort_flag, 911);
        if (!ok) break;
        if (elect_one()) {
          const uint32_t sa = sbase + s * C::STAGE_BYTES;
          const uint32_t fb = full0 + s * 8;
          if (leader) mbar_arrive_expect_tx(bar(PB_FULL + s), 2 * C::STAGE_BYTES);
          if (p.a_heads) {
            const int b = m0 / p.a_seq, s0 = m0 - b * p.a_seq;
            tma_load_3d_pair(sa, &tm_a, fb, (kb & 1) * 64, s0, b * p.a_n_heads + (kb >> 1));
          } else {
            tma_load_2d_pair(sa, &tm_a, fb, kb * kGemmBK, m0);
          }
          tma_load_2d_pair(sa + C::A_BYTES, &tm_b, fb, kb * kGemmBK, n0);
        }
        __syncwarp();
      }
    }
    if (!ok) {
      if (leader) {
        // the last copies counted on each stage (both CTAs') land first
        for (int s = 0; s < kPairStages; ++s) {
          const int n_s = g > s ? (g - s - 1) / kPairStages + 1 : 0;
          if (n_s) (void)mbar_wait(bar(PB_FULL + s), (n_s - 1) & 1, nullptr, 912);
        }
      } else {
        // the odd CTA cannot see the even CTA's barrier: give copies in flight
        // into its own shared memory time to land
        __nanosleep(200000);
      }
    }
  } else if (warp == 1) {
    // ===================== MMA issuer (even CTA only) ===================
    if (leader) {
      constexpr uint32_t idesc = make_idesc_bf16(256, kGemmBN, 0, 0);
      const uint64_t da0 = make_sdesc_sw128(sbase, 16, 1024);
      const uint64_t db0 = make_sdesc_sw128(sbase + C::A_BYTES, 16, 1024);
      int g = 0, i = 0;
      bool ok = true;
      for (int t = pair; t < p.n_tiles && ok; t += n_pairs, ++i) {
        const int b = i & 1, use = i >> 1;
        if (use > 0) ok = mbar_wait_warp(bar(PB_AEMPTY + b), (use - 1) & 1, abort_flag, 913);
        if (!ok) break;
        tc_fence_after();
        const uint32_t acc = tmem + b * kGemmBN;
        for (int kb = 0; kb < p.n_kblk; ++kb, ++g) {
          const int s = g % kPairStages;
          ok = mbar_wait_warp(bar(PB_FULL + s), (g / kPairStages) & 1, abort_flag, 914);
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
            const uint32_t off = s * C::STAGE_BYTES;
#pragma unroll
            for (int kk = 0; kk < kGemmBK / 16; ++kk)
              mma_ss_pair(acc, desc_adv(da0, off + kk * 32), desc_adv(db0, off + kk * 32), idesc,
                          (kb | kk) != 0 ? 1u : 0u);
            tc_commit_pair_mc(bar(PB_EMPTY + s), 0x3);  // the stage is free in both CTAs
          }
          __syncwarp();
        }
        if (!ok) break;
        if (elect_one()) tc_commit_pair_mc(bar(PB_AFULL + b), 0x3);
        __syncwarp();
      }
      // every pair MMA has completed before either CTA frees TMEM or exits
      if (elect_one()) tc_commit_pair(bar(PB_DRAIN));
      __syncwarp();
      (void)mbar_wait(bar(PB_DRAIN), 0, nullptr, 915);
    }
  } else {
    // ===================== epilogue (both CTAs) =========================
    const int q = warp & 3;
    const uint32_t stg = sbase + C::OFF_EPI + (warp - 2) * C::EPI_WARP_BYTES;
    const uint32_t aempty0 = mapa_cta(bar(PB_AEMPTY), 0);
    int i = 0;
    for (int t = pair; t < p.n_tiles; t += n_pairs, ++i) {
      int mb, nb;
      gemm_tile(p, t, mb, nb);
      const int b = i & 1, use = i >> 1;
      if (!mbar_wait_warp(bar(PB_AFULL + b), use & 1, abort_flag, 916)) break;
      tc_fence_after();
      const uint32_t acc = tmem + ((uint32_t)(q * 32) << 16) + b * kGemmBN;
      const int row0 = mb * 256 + (int)crank * 128 + q * 32;
      auto release_acc = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(aempty0 + b * 8);
      };
      gemm_epilogue_warp<EPI>(p, acc, row0, nb, lane, stg, release_acc);
    }
    if constexpr (EPI == GEMM_EPI_PUSH) __threadfence_system();  // peer stores before any flag
  }

  tc_fence_before();
  cluster_sync_all();  // no CTA frees TMEM or leaves while the pair still uses it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, C::TM_COLS);
  }
}

}  // namespace tfb
