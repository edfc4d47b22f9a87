// comm_norm.cuh -- the tensor-parallel Llama layer's all-reduce, fused with the
// residual add and RMSNorm that follow it, in one kernel over NVLink peer
// memory (plain peer loads and stores; no multicast).
//
// In the layer (src/layers/llama_block.rs:55-65 split over N ranks) each rank
// holds a partial o_proj (or down_proj) output P_r [rows, cols]; the next op
// is h = x + sum_r P_r followed by y = RMSNorm(h) (fused_add_rmsnorm.rs:53-110).
// Two-shot, per call:
//   barrier A   every rank's P_r is complete (its GEMM ran before this kernel)
//   phase 1     rank r owns rows [r*rows/N, (r+1)*rows/N): h = x + sum_p P_p
//               (peer loads, fp32 sum in rank order), written as bf16 into
//               every rank's symmetric h buffer (peer stores) -- the reduce-
//               scatter and the all-gather in one pass
//   barrier B   all slices have landed everywhere
//   phase 2     y = RMSNorm(h) * weight over all rows, from the local h
// Each rank moves (N-1)/N of the tensor in and (N-1)/N out over NVLink.
// The barriers are per CTA: CTA c signals CTA c of every rank through the
// ranks' signal pads and waits, bounded (2 s, then a status code), for theirs;
// CTA c's phase-2 rows are exactly the rows the CTAs c of all ranks wrote in
// phase 1, so no wider barrier is needed.
#pragma once

#include "norm_act.cuh"

namespace tfb {

constexpr int kArCtas = 128;       // below the SM count: all resident at once
constexpr int kArThreads = 512;
constexpr int kArMaxWorld = 8;
constexpr int kArPadOffsetU32 = 256;  // our flags live past the first 1 KB of each pad
constexpr int kArPadU32 = kArPadOffsetU32 + 2 * kArCtas * kArMaxWorld;  // 9216 bytes

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// CTA-level barrier with CTA blockIdx.x of every rank; flags carry the call's
// epoch (monotonic), slot [phase][cta][source rank] in the destination's pad.
__device__ __forceinline__ bool ar_barrier(uint32_t* const* pads, int rank, int world, int phase,
                                           uint32_t epoch, int site) {
  __threadfence_system();  // this thread's peer stores before the flags
  __syncthreads();
  bool ok = true;
  if (threadIdx.x < world) {
    const int slot = kArPadOffsetU32 + (phase * kArCtas + blockIdx.x) * kArMaxWorld;
    st_release_sys(pads[threadIdx.x] + slot + rank, epoch);
    const uint32_t* mine = pads[rank] + slot + threadIdx.x;
    const unsigned long long t0 = globaltimer_ns();
    for (unsigned it = 0;; ++it) {
      if ((int)(ld_acquire_sys(mine) - epoch) >= 0) break;
      if ((it & 255u) == 255u && globaltimer_ns() - t0 > kWaitTimeoutNs) {
        atomicCAS(&g_device_status, 0, site);
        ok = false;
        break;
      }
    }
  }
  return __syncthreads_and(ok);
}

// W: peer capacity of this instantiation (2, 4 or 8; world <= W); each thread
// keeps 16 / W vectors x W peers (64 registers) of loads in flight.
template <int W>
__global__ void __launch_bounds__(kArThreads)
    allreduce_residual_rmsnorm_kernel(const __nv_bfloat16* const* __restrict__ peer_src,
                                      __nv_bfloat16* const* __restrict__ peer_h,
                                      uint32_t* const* __restrict__ pads,
                                      const __nv_bfloat16* __restrict__ residual,
                                      const __nv_bfloat16* __restrict__ weight,
                                      __nv_bfloat16* __restrict__ y, int rank, int world,
                                      int rows, int cols, float eps, uint32_t epoch) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slice = rows / world;
  const int nvec = cols / 8;
  if (!ar_barrier(pads, rank, world, 0, epoch, 801)) return;
  // ---- phase 1: this CTA's rows of this rank's slice (rows c, c + kArCtas, ...),
  // summed over the ranks, to every rank's h.  All threads walk the CTA's
  // (row, 16-byte vector) pairs, 16 / W at a time, so many peer loads are
  // in flight.
  constexpr int kArUnroll = 16 / W;
  const int my_rows = slice > (int)blockIdx.x ? (slice - 1 - (int)blockIdx.x) / kArCtas + 1 : 0;
  const long long n_items = (long long)my_rows * nvec;
  for (long long base = threadIdx.x; base < n_items; base += (long long)kArThreads * kArUnroll) {
    uint4 part[kArUnroll][W];
    size_t off[kArUnroll];
    bool live[kArUnroll];
#pragma unroll
    for (int u = 0; u < kArUnroll; ++u) {
      const long long idx = base + (long long)u * kArThreads;
      live[u] = idx < n_items;
      const int rl = live[u] ? (int)(idx / nvec) : 0, v = live[u] ? (int)(idx % nvec) : 0;
      const size_t row = (size_t)rank * slice + blockIdx.x + (size_t)rl * kArCtas;
      off[u] = row * cols + (size_t)v * 8;
#pragma unroll
      for (int p = 0; p < W; ++p)
        if (p < world && live[u]) part[u][p] = *reinterpret_cast<const uint4*>(peer_src[p] + off[u]);
    }
#pragma unroll
    for (int u = 0; u < kArUnroll; ++u) {
      if (!live[u]) continue;
      float acc[8];
      if (residual) {
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(residual + off[u]), acc);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
      }
#pragma unroll
      for (int p = 0; p < W; ++p)
        if (p < world) {
          float f[8];
          bf16x8_to_f32(part[u][p], f);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] += f[e];
        }
      const uint4 hv = f32_to_bf16x8(acc);
#pragma unroll
      for (int p = 0; p < W; ++p)
        if (p < world) *reinterpret_cast<uint4*>(peer_h[p] + off[u]) = hv;
    }
  }
  if (!ar_barrier(pads, rank, world, 1, epoch, 802)) return;
  if (!weight || !y) return;
  // ---- phase 2: RMSNorm of the rows the CTAs with this index wrote
  // (rows blockIdx.x + k * kArCtas of every rank's slice), one warp per row
  const __nv_bfloat16* h = peer_h[rank];
  const uint4* w4 = reinterpret_cast<const uint4*>(weight);
  for (int p = 0; p < world; ++p)
    for (int k = warp; k < my_rows; k += kArThreads / 32) {
      const size_t row = (size_t)p * slice + blockIdx.x + (size_t)k * kArCtas;
      const uint4* hr = reinterpret_cast<const uint4*>(h + row * cols);
      float ss = 0.0f;
      for (int v = lane; v < nvec; v += 32) {
        float f[8];
        bf16x8_to_f32(hr[v], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = fmaf(f[e], f[e], ss);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float rstd = rsqrtf(ss / (float)cols + eps);
      uint4* yr = reinterpret_cast<uint4*>(y + row * cols);
      for (int v = lane; v < nvec; v += 32) {
        float f[8], wf[8];
        bf16x8_to_f32(hr[v], f);
        bf16x8_to_f32(w4[v], wf);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = f[e] * rstd * wf[e];
        yr[v] = f32_to_bf16x8(f);
      }
    }
}

}  // namespace tfb
