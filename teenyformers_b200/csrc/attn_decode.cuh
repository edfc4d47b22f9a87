// attn_decode.cuh -- KV-cache decode attention for sm_100a (bf16 in/out,
// fp32 softmax and accumulation).
//
// The caller of the attention op that comes after prefill: each of `batch`
// sequences has cache_seqlens[b] keys/values in a [B, Hkv, S_cap, D] cache,
// the last n_q of which belong to the n_q new query tokens.  Query i of
// sequence b sits at position L_b - n_q + i and sees keys 0 .. L_b - n_q + i
// (with n_q = 1: the whole cache).  teenyformers' generation loop instead
// re-runs the full prefix through the causal kernel for every new token
// (examples/llama_generate.rs:373-400); this computes the same softmax
// attention for the new rows only (flash_attn2.rs:77-125 semantics, scale
// applied to the scores, natural-log LSE).
//
// The work is HBM-bound: one KV head serves G * n_q query rows (G = Hq/Hkv),
// a handful per key, so the kernel streams K/V once at full bandwidth and
// does the arithmetic with warp-level mma.sync m16n8k16 tiles (tcgen05's
// smallest M of 64 would be mostly padding at 4-16 rows).
//   grid (splits, Hkv * row_blocks, B), 4 warps; each CTA owns one
//   16-row block of one KV head's query rows and one contiguous split of
//   the keys, streamed as 64-key tiles through a 3-stage TMA ring (SW128,
//   so ldmatrix reads are conflict-free).  Warp w takes keys 16w..16w+15 of
//   every tile and keeps its own online-softmax state; the four states are
//   merged through shared memory at the end.  With one split the CTA writes
//   O / LSE; otherwise fp32 partials go to the workspace and
//   fa_decode_combine_kernel merges the splits.
#pragma once

#include "sm100.cuh"

namespace tfb {

constexpr int kDecTileKeys = 64;
constexpr int kDecStages = 3;
constexpr int kDecThreads = 128;

struct DecodeParams {
  const __nv_bfloat16* q;  // [B, Hq, n_q, D]
  __nv_bfloat16* o;        // [B, Hq, n_q, D]
  float* lse;              // [B, Hq, n_q]
  const int* seqlens;      // [B] keys in the cache per sequence
  float* part_o;           // [splits, B*Hq*n_q, D] fp32 (splits > 1)
  float* part_lse;         // [splits, B*Hq*n_q]
  int Hq, Hkv, n_q, cap, splits, chunk, row_blocks;
  float scale_log2;
};

template <int D>
struct DecCfg {
  static constexpr int HALVES = D / 64;
  static constexpr int TILE_BYTES = kDecTileKeys * D * 2;    // one of K, V
  static constexpr int HALF_BYTES = kDecTileKeys * 128;      // 64 keys x 128 B
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;         // K then V
  static constexpr int OFF_BAR = kDecStages * STAGE_BYTES;
  // the end-of-loop merge reuses the (then idle) K/V stages
  static constexpr int OFF_MERGE = 0;                         // 4 warps x (m, l) x 16 rows
  static constexpr int OFF_OMERGE = 512;                      // 4 warps x 16 x D fp32
  static_assert(OFF_OMERGE + 4 * 16 * D * 4 <= OFF_BAR, "merge area exceeds the stages");
  static constexpr int SMEM_BYTES = OFF_BAR + 64 + 1024;
};

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                          uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// Byte offset of (row, 16-byte chunk c of the row's D) in a SW128 tile stored
// as 64-column halves of [64 rows x 128 B].
__device__ __forceinline__ uint32_t sw128_off(int row, int c) {
  return uint32_t((c >> 3) * (kDecTileKeys * 128) + row * 128 + (((c & 7) ^ (row & 7)) << 4));
}

template <int D>
__global__ void __launch_bounds__(kDecThreads)
    fa_decode_kernel(const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const DecodeParams p) {
  using C = DecCfg<D>;
  constexpr int NT_D = D / 8;   // n-tiles of the output (8 columns each)
  constexpr int KS_D = D / 16;  // k-steps of S = Q K^T
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  auto bar = [&](int i) { return smem_u32(bars + i); };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x;
  const int hkv = blockIdx.y / p.row_blocks, rb = blockIdx.y % p.row_blocks;
  const int b = blockIdx.z;
  const int G = p.Hq / p.Hkv;
  const int R = G * p.n_q;  // query rows of this KV head
  const int L = min(max(p.seqlens[b], 0), p.cap);  // out-of-range lengths are clamped
  const int k_begin = split * p.chunk;
  const int k_end = min(L, k_begin + p.chunk);
  const int n_tiles = k_end > k_begin ? (k_end - k_begin + kDecTileKeys - 1) / kDecTileKeys : 0;
  const int bh_kv = b * p.Hkv + hkv;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kDecStages; ++s) mbar_init(bar(s), 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int t) {  // tile t of this split into stage t % kDecStages
    const int s = t % kDecStages;
    const uint32_t dst = sbase + s * C::STAGE_BYTES;
    mbar_arrive_expect_tx(bar(s), C::STAGE_BYTES);
    for (int hh = 0; hh < C::HALVES; ++hh) {
      tma_load_3d(dst + hh * C::HALF_BYTES, &tm_k, bar(s), hh * 64, k_begin + t * kDecTileKeys,
                  bh_kv);
      tma_load_3d(dst + C::TILE_BYTES + hh * C::HALF_BYTES, &tm_v, bar(s), hh * 64,
                  k_begin + t * kDecTileKeys, bh_kv);
    }
  };
  int issued = 0;  // tiles whose loads thread 0 has issued
  if (threadIdx.x == 0)
    for (; issued < min(n_tiles, kDecStages - 1); ++issued) issue(issued);

  // ---- this thread's two query rows: r0 = lane/4 and r0 + 8 of the block
  const int r_lo = rb * 16 + (lane >> 2), r_hi = r_lo + 8;
  auto row_pos = [&](int r) {  // last key index the row may see; -1 for padding rows
    if (r >= R) return -1;
    return L - p.n_q + (r % p.n_q);
  };
  const int lim_lo = row_pos(r_lo), lim_hi = row_pos(r_hi);
  // Q fragments (A operand, 16 rows x D), straight from global memory
  uint32_t qa[KS_D][4];
  {
    auto qrow = [&](int r) -> const uint32_t* {
      if (r >= R) return nullptr;
      const int g = r / p.n_q, i = r % p.n_q;
      return reinterpret_cast<const uint32_t*>(
          p.q + (((size_t)b * p.Hq + hkv * G + g) * p.n_q + i) * D);
    };
    const uint32_t* ql = qrow(r_lo);
    const uint32_t* qh = qrow(r_hi);
#pragma unroll
    for (int ks = 0; ks < KS_D; ++ks) {
      const int w0 = ks * 8 + (lane & 3);  // bf16 pair index: columns 16ks + 2(lane%4)
      qa[ks][0] = ql ? ql[w0] : 0u;
      qa[ks][1] = qh ? qh[w0] : 0u;
      qa[ks][2] = ql ? ql[w0 + 4] : 0u;
      qa[ks][3] = qh ? qh[w0 + 4] : 0u;
    }
  }
  float o[NT_D][4];
#pragma unroll
  for (int n = 0; n < NT_D; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.0f, l_hi = 0.0f;
  const float sl2 = p.scale_log2;
  bool ok = true;

  for (int t = 0; t < n_tiles && ok; ++t) {
    const int s = t % kDecStages;
    // every warp is done with tile t-1, whose stage the next load reuses
    __syncthreads();
    if (threadIdx.x == 0 && t + kDecStages - 1 < n_tiles) issue(issued++);
    ok = mbar_wait(bar(s), (t / kDecStages) & 1, nullptr, 701);
    if (!__syncthreads_and(ok)) {
      ok = false;
      // let the loads still in flight land before the shared memory goes away
      if (threadIdx.x == 0)
        for (int u = t + 1; u < issued; ++u)
          (void)mbar_wait(bar(u % kDecStages), (u / kDecStages) & 1, nullptr, 702);
      break;
    }
    const uint32_t kt = sbase + s * C::STAGE_BYTES, vt = kt + C::TILE_BYTES;
    const int key0 = k_begin + t * kDecTileKeys + warp * 16;  // this warp's 16 keys
    // S (16 rows x 16 keys) = Q K^T: two 8-key n-tiles
    float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int ks = 0; ks < KS_D; ks += 2) {
      // ldmatrix x4: matrices (keys 0-7 | 8-15) x (D chunk 2ks | 2ks+1 ... ) per lane group
      // lanes 0-7: keys 0-7 chunk c0; 8-15: keys 0-7 chunk c0+1; 16-23: keys 8-15 chunk c0;
      // 24-31: keys 8-15 chunk c0+1, where c0 = 2*ks (16-byte chunks of 8 columns)
      const int krow = warp * 16 + (lane & 7) + ((lane >> 4) << 3);
      const int c = 2 * ks + ((lane >> 3) & 1);
      uint32_t b00, b01, b10, b11;
      ldsm_x4(kt + sw128_off(krow, c), b00, b01, b10, b11);
      mma_bf16_16816(sacc[0], qa[ks], b00, b01);
      mma_bf16_16816(sacc[1], qa[ks], b10, b11);
      const int c2 = c + 2;
      ldsm_x4(kt + sw128_off(krow, c2), b00, b01, b10, b11);
      mma_bf16_16816(sacc[0], qa[ks + 1], b00, b01);
      mma_bf16_16816(sacc[1], qa[ks + 1], b10, b11);
    }
    // mask, online softmax (log2 domain)
    float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int kk = key0 + n * 8 + (lane & 3) * 2 + e;
        if (kk > lim_lo) sacc[n][e] = -INFINITY;
        if (kk > lim_hi) sacc[n][2 + e] = -INFINITY;
        mx_lo = fmaxf(mx_lo, sacc[n][e]);
        mx_hi = fmaxf(mx_hi, sacc[n][2 + e]);
      }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
      mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, off));
      mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, off));
    }
    const float mn_lo = fmaxf(m_lo, mx_lo * sl2), mn_hi = fmaxf(m_hi, mx_hi * sl2);
    const float base_lo = mn_lo == -INFINITY ? 0.0f : mn_lo;
    const float base_hi = mn_hi == -INFINITY ? 0.0f : mn_hi;
    const float al_lo = ex2_approx(m_lo - base_lo), al_hi = ex2_approx(m_hi - base_hi);
    m_lo = mn_lo;
    m_hi = mn_hi;
    float ps_lo = 0.0f, ps_hi = 0.0f;
    uint32_t pa[4];  // P as the A operand of P V (16 rows x 16 keys)
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      const float p0 = ex2_approx(fmaf(sacc[n][0], sl2, -base_lo));
      const float p1 = ex2_approx(fmaf(sacc[n][1], sl2, -base_lo));
      const float p2 = ex2_approx(fmaf(sacc[n][2], sl2, -base_hi));
      const float p3 = ex2_approx(fmaf(sacc[n][3], sl2, -base_hi));
      ps_lo += p0 + p1;
      ps_hi += p2 + p3;
      pa[2 * n] = pack_bf16x2(p0, p1);
      pa[2 * n + 1] = pack_bf16x2(p2, p3);
    }
    l_lo = l_lo * al_lo + ps_lo;
    l_hi = l_hi * al_hi + ps_hi;
#pragma unroll
    for (int n = 0; n < NT_D; ++n) {
      o[n][0] *= al_lo;
      o[n][1] *= al_lo;
      o[n][2] *= al_hi;
      o[n][3] *= al_hi;
    }
    // O += P V: B = V (16 keys x 8 columns per n-tile) via ldmatrix.trans
#pragma unroll
    for (int n = 0; n < NT_D; n += 2) {
      // lanes 0-7: keys 0-7, chunk n; 8-15: keys 8-15, chunk n; 16-23: keys 0-7,
      // chunk n+1; 24-31: keys 8-15, chunk n+1
      const int vrow = warp * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
      const int c = n + (lane >> 4);
      uint32_t v0, v1, v2, v3;
      ldsm_x4_t(vt + sw128_off(vrow, c), v0, v1, v2, v3);
      mma_bf16_16816(o[n], pa, v0, v1);
      mma_bf16_16816(o[n + 1], pa, v2, v3);
    }
  }
  // row sums over the 4 lanes that share a row
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, off);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, off);
  }
  // ---- merge the four warps' states through shared memory
  float* sm_ml = reinterpret_cast<float*>(smem + C::OFF_MERGE);     // [warp][m|l][16]
  float* sm_o = reinterpret_cast<float*>(smem + C::OFF_OMERGE);     // [warp][16][D]
  __syncthreads();
  const int rl = lane >> 2, rh = rl + 8;
  if ((lane & 3) == 0) {
    sm_ml[warp * 32 + rl] = m_lo;
    sm_ml[warp * 32 + rh] = m_hi;
    sm_ml[warp * 32 + 16 + rl] = l_lo;
    sm_ml[warp * 32 + 16 + rh] = l_hi;
  }
#pragma unroll
  for (int n = 0; n < NT_D; ++n) {
    const int col = n * 8 + (lane & 3) * 2;
    sm_o[(warp * 16 + rl) * D + col] = o[n][0];
    sm_o[(warp * 16 + rl) * D + col + 1] = o[n][1];
    sm_o[(warp * 16 + rh) * D + col] = o[n][2];
    sm_o[(warp * 16 + rh) * D + col + 1] = o[n][3];
  }
  __syncthreads();
  if (!ok) return;
  // thread t: row t / 8, columns (t % 8) * D/8 .. +D/8
  const int row = threadIdx.x >> 3, cseg = (threadIdx.x & 7) * (D / 8);
  const int r = rb * 16 + row;
  if (r >= R) return;
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < 4; ++w) M = fmaxf(M, sm_ml[w * 32 + row]);
  const float Mb = M == -INFINITY ? 0.0f : M;
  float wsc[4], Ls = 0.0f;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    wsc[w] = ex2_approx(sm_ml[w * 32 + row] - Mb);
    Ls += wsc[w] * sm_ml[w * 32 + 16 + row];
  }
  const int g = r / p.n_q, i = r % p.n_q;
  const size_t orow = ((size_t)b * p.Hq + hkv * G + g) * p.n_q + i;
  // natural-log LSE of the scaled scores; -inf for an empty split
  const float lse = Ls > 0.0f ? (Mb + lg2_approx(Ls)) * 0.6931471805599453f : -INFINITY;
  const float inv = Ls > 0.0f ? 1.0f / Ls : 0.0f;
  if (p.splits == 1) {
    uint32_t w[D / 16];
#pragma unroll
    for (int j = 0; j < D / 16; ++j) {
      float v[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int col = cseg + 2 * j + e;
        float acc = 0.0f;
#pragma unroll
        for (int ww = 0; ww < 4; ++ww) acc += wsc[ww] * sm_o[(ww * 16 + row) * D + col];
        v[e] = acc * inv;
      }
      w[j] = pack_bf16x2(v[0], v[1]);
    }
    uint4* dst = reinterpret_cast<uint4*>(p.o + orow * D + cseg);
#pragma unroll
    for (int j = 0; j < D / 64; ++j) dst[j] = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
    if ((threadIdx.x & 7) == 0) p.lse[orow] = lse;
  } else {
    const size_t rows_total = (size_t)gridDim.z * p.Hq * p.n_q;
    float* dst = p.part_o + ((size_t)split * rows_total + orow) * D + cseg;
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      float acc = 0.0f;
#pragma unroll
      for (int ww = 0; ww < 4; ++ww) acc += wsc[ww] * sm_o[(ww * 16 + row) * D + cseg + j];
      dst[j] = acc * inv;
    }
    if ((threadIdx.x & 7) == 0) p.part_lse[(size_t)split * rows_total + orow] = lse;
  }
}

// O = sum_s exp(lse_s - lse) O_s, lse = log sum_s exp(lse_s): one warp per
// query row, D/32 columns per lane.
template <int D>
__global__ void __launch_bounds__(256)
    fa_decode_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                             __nv_bfloat16* __restrict__ o, float* __restrict__ lse, long long rows,
                             int splits) {
  const long long row = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, part_lse[s * rows + row]);
  const float Mb = M == -INFINITY ? 0.0f : M;
  float acc[D / 32];
#pragma unroll
  for (int j = 0; j < D / 32; ++j) acc[j] = 0.0f;
  float wsum = 0.0f;
  for (int s = 0; s < splits; ++s) {
    const float ls = part_lse[s * rows + row];
    if (ls == -INFINITY) continue;
    const float w = __expf(ls - Mb);
    wsum += w;
    const float* src = part_o + ((size_t)s * rows + row) * D;
#pragma unroll
    for (int j = 0; j < D / 32; ++j) acc[j] += w * src[lane + 32 * j];
  }
  const float inv = wsum > 0.0f ? 1.0f / wsum : 0.0f;
#pragma unroll
  for (int j = 0; j < D / 32; ++j) o[row * D + lane + 32 * j] = __float2bfloat16_rn(acc[j] * inv);
  if (lane == 0) lse[row] = wsum > 0.0f ? Mb + logf(wsum) : -INFINITY;
}

}  // namespace tfb
