// attn_f32.cuh -- fp32 flash-attention forward/backward with the reference's
// exact argument set (teenyformers src/kernels/flash_attn2.rs:61-279), for
// callers that keep the reference's fp32 tensors ([BH, S, D], any D <= 256).
//
// These are CUDA-core kernels: fp32 inputs have no dense tensor-core path
// with fp32 rounding, and this entry exists for drop-in parity (config #1
// sizes), not throughput; the bf16 tcgen05 kernels are the fast path.
//
// Forward: a warp owns one query row; keys are staged 32 at a time in shared
// memory, each lane scores one key, and the running max / sum / accumulator
// are updated once per 32 keys (same online softmax as flash_attn2.rs:95-118,
// regrouped).  Top-left causal mask k > q.  LSE = m + ln(l).
//
// Backward: the reference adds dK/dV with fp32 atomics (flash_attn2.rs:
// 196-197); here dQ comes from a query-row pass and dK/dV from a key-row pass
// over the same p / ds terms, so results are deterministic and need no
// zero-initialised outputs or scratch memory.
#pragma once

#include <math.h>
#include <stdint.h>

namespace tfb {

constexpr int kF32Rows = 8;   // warps (rows) per CTA
constexpr int kF32Tile = 32;  // staged rows of the other operand
constexpr int kF32MaxD = 256;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// grid = (ceil(Sq / 8), BH), block = 256; dyn smem = (8 + 2*32) * D floats
__global__ void __launch_bounds__(256)
    fa_fwd_f32_kernel(const float* __restrict__ q, const float* __restrict__ k,
                      const float* __restrict__ v, float* __restrict__ o, float* __restrict__ lse,
                      int Sq, int Sk, int D, float scale, float neg_inf, int causal, int Hq,
                      int Hkv) {
  extern __shared__ float fsm[];
  float* sq = fsm;                    // [8][D]
  float* sk = sq + kF32Rows * D;      // [32][D]
  float* sv = sk + kF32Tile * D;      // [32][D]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y;
  const int bkv = (bh / Hq) * Hkv + (bh % Hq) / (Hq / Hkv);
  const int qr = blockIdx.x * kF32Rows + warp;
  const bool valid = qr < Sq;
  for (int i = threadIdx.x; i < kF32Rows * D; i += blockDim.x) {
    const int r = blockIdx.x * kF32Rows + i / D;
    sq[i] = r < Sq ? q[((size_t)bh * Sq + r) * D + i % D] : 0.0f;
  }
  float acc[kF32MaxD / 32];
#pragma unroll
  for (int i = 0; i < kF32MaxD / 32; ++i) acc[i] = 0.0f;
  float m = -INFINITY, l = 0.0f;
  const int q_hi_block = min(Sq, (int)(blockIdx.x + 1) * kF32Rows) - 1;
  const int k_end = causal ? min(Sk, q_hi_block + 1) : Sk;
  for (int k0 = 0; k0 < k_end; k0 += kF32Tile) {
    __syncthreads();
    for (int i = threadIdx.x; i < kF32Tile * D; i += blockDim.x) {
      const int r = k0 + i / D;
      const size_t g = ((size_t)bkv * Sk + r) * D + i % D;
      sk[i] = r < Sk ? k[g] : 0.0f;
      sv[i] = r < Sk ? v[g] : 0.0f;
    }
    __syncthreads();
    const int kr = k0 + lane;
    float dot = 0.0f;
    for (int d = 0; d < D; ++d) dot += sq[warp * D + d] * sk[lane * D + d];
    float s = dot * scale;
    if (kr >= Sk || (causal && kr > qr)) s = neg_inf;
    const float m_new = fmaxf(m, warp_max(s));
    const float base = m_new == -INFINITY ? 0.0f : m_new;
    const float alpha = expf(m - base);
    const float pr = expf(s - base);
    l = l * alpha + warp_sum(pr);
#pragma unroll
    for (int i = 0; i < kF32MaxD / 32; ++i) acc[i] *= alpha;
    for (int kk = 0; kk < kF32Tile; ++kk) {
      const float pk = __shfl_sync(0xffffffffu, pr, kk);
#pragma unroll
      for (int i = 0; i < kF32MaxD / 32; ++i) {
        const int d = lane + 32 * i;
        if (d < D) acc[i] += pk * sv[kk * D + d];
      }
    }
    m = m_new;
  }
  if (valid) {
    float* orow = o + ((size_t)bh * Sq + qr) * D;
#pragma unroll
    for (int i = 0; i < kF32MaxD / 32; ++i) {
      const int d = lane + 32 * i;
      if (d < D) orow[d] = acc[i] / l;
    }
    if (lane == 0) lse[(size_t)bh * Sq + qr] = m + logf(l);
  }
}

// dQ pass.  grid = (ceil(Sq / 8), BH), block 256; dyn smem = (3*8 + 2*32) * D
__global__ void __launch_bounds__(256)
    fa_bwd_dq_f32_kernel(const float* __restrict__ q, const float* __restrict__ k,
                         const float* __restrict__ v, const float* __restrict__ o,
                         const float* __restrict__ dO, const float* __restrict__ lse,
                         float* __restrict__ dq, int Sq, int Sk, int D, float scale, int causal,
                         int Hq, int Hkv) {
  extern __shared__ float fsm[];
  float* sq = fsm;
  float* sdo = sq + kF32Rows * D;
  float* so = sdo + kF32Rows * D;
  float* sk = so + kF32Rows * D;
  float* sv = sk + kF32Tile * D;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y;
  const int bkv = (bh / Hq) * Hkv + (bh % Hq) / (Hq / Hkv);
  const int qr = blockIdx.x * kF32Rows + warp;
  for (int i = threadIdx.x; i < kF32Rows * D; i += blockDim.x) {
    const int r = blockIdx.x * kF32Rows + i / D;
    const size_t g = ((size_t)bh * Sq + r) * D + i % D;
    sq[i] = r < Sq ? q[g] : 0.0f;
    sdo[i] = r < Sq ? dO[g] : 0.0f;
    so[i] = r < Sq ? o[g] : 0.0f;
  }
  __syncthreads();
  // D_q = rowsum(O * dO)  (flash_attn2.rs:171)
  float part = 0.0f;
  for (int d = lane; d < D; d += 32) part += so[warp * D + d] * sdo[warp * D + d];
  const float delta = warp_sum(part);
  const float lq = qr < Sq ? lse[(size_t)bh * Sq + qr] : 0.0f;
  float acc[kF32MaxD / 32];
#pragma unroll
  for (int i = 0; i < kF32MaxD / 32; ++i) acc[i] = 0.0f;
  const int q_hi_block = min(Sq, (int)(blockIdx.x + 1) * kF32Rows) - 1;
  const int k_end = causal ? min(Sk, q_hi_block + 1) : Sk;
  for (int k0 = 0; k0 < k_end; k0 += kF32Tile) {
    __syncthreads();
    for (int i = threadIdx.x; i < kF32Tile * D; i += blockDim.x) {
      const int r = k0 + i / D;
      const size_t g = ((size_t)bkv * Sk + r) * D + i % D;
      sk[i] = r < Sk ? k[g] : 0.0f;
      sv[i] = r < Sk ? v[g] : 0.0f;
    }
    __syncthreads();
    const int kr = k0 + lane;
    float dot = 0.0f, dov = 0.0f;
    for (int d = 0; d < D; ++d) {
      dot += sq[warp * D + d] * sk[lane * D + d];
      dov += sdo[warp * D + d] * sv[lane * D + d];
    }
    float pr = expf(dot * scale - lq);
    if (kr >= Sk || (causal && kr > qr)) pr = 0.0f;
    const float ds = pr * (dov - delta);
    for (int kk = 0; kk < kF32Tile; ++kk) {
      const float dsk = __shfl_sync(0xffffffffu, ds, kk);
#pragma unroll
      for (int i = 0; i < kF32MaxD / 32; ++i) {
        const int d = lane + 32 * i;
        if (d < D) acc[i] += dsk * sk[kk * D + d] * scale;
      }
    }
  }
  if (qr < Sq) {
    float* out = dq + ((size_t)bh * Sq + qr) * D;
#pragma unroll
    for (int i = 0; i < kF32MaxD / 32; ++i) {
      const int d = lane + 32 * i;
      if (d < D) out[d] = acc[i];
    }
  }
}

// dK/dV pass over key rows; every query head of the KV head's group
// contributes.  grid = (ceil(Sk / 8), B*Hkv), block 256;
// dyn smem = (2*8 + 3*32) * D floats + 2*32 floats
__global__ void __launch_bounds__(256)
    fa_bwd_dkdv_f32_kernel(const float* __restrict__ q, const float* __restrict__ k,
                           const float* __restrict__ v, const float* __restrict__ o,
                           const float* __restrict__ dO, const float* __restrict__ lse,
                           float* __restrict__ dk, float* __restrict__ dv, int Sq, int Sk, int D,
                           float scale, int causal, int Hq, int Hkv) {
  extern __shared__ float fsm[];
  float* sk = fsm;                       // [8][D]
  float* sv = sk + kF32Rows * D;         // [8][D]
  float* sq = sv + kF32Rows * D;         // [32][D]
  float* sdo = sq + kF32Tile * D;        // [32][D]
  float* so = sdo + kF32Tile * D;        // [32][D]
  float* sl = so + kF32Tile * D;         // [32]
  float* sdelta = sl + kF32Tile;         // [32]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bkv = blockIdx.y;
  const int b = bkv / Hkv, hk = bkv % Hkv, G = Hq / Hkv;
  const int kr = blockIdx.x * kF32Rows + warp;
  for (int i = threadIdx.x; i < kF32Rows * D; i += blockDim.x) {
    const int r = blockIdx.x * kF32Rows + i / D;
    const size_t g = ((size_t)bkv * Sk + r) * D + i % D;
    sk[i] = r < Sk ? k[g] : 0.0f;
    sv[i] = r < Sk ? v[g] : 0.0f;
  }
  float gk[kF32MaxD / 32], gv[kF32MaxD / 32];
#pragma unroll
  for (int i = 0; i < kF32MaxD / 32; ++i) gk[i] = gv[i] = 0.0f;
  const int k_lo_block = blockIdx.x * kF32Rows;
  const int q_start = causal ? (k_lo_block / kF32Tile) * kF32Tile : 0;
  for (int g = 0; g < G; ++g) {
    const int bh = b * Hq + hk * G + g;
    for (int q0 = q_start; q0 < Sq; q0 += kF32Tile) {
      __syncthreads();
      for (int i = threadIdx.x; i < kF32Tile * D; i += blockDim.x) {
        const int r = q0 + i / D;
        const size_t gi = ((size_t)bh * Sq + r) * D + i % D;
        sq[i] = r < Sq ? q[gi] : 0.0f;
        sdo[i] = r < Sq ? dO[gi] : 0.0f;
        so[i] = r < Sq ? o[gi] : 0.0f;
      }
      __syncthreads();
      // lse and D_q of the 32 staged queries (one warp computes them)
      if (warp == 0) {
        const int r = q0 + lane;
        sl[lane] = r < Sq ? lse[(size_t)bh * Sq + r] : 0.0f;
      }
      if (warp < kF32Tile / 4) {
        for (int qq = warp * 4; qq < warp * 4 + 4; ++qq) {
          float part = 0.0f;
          for (int d = lane; d < D; d += 32) part += so[qq * D + d] * sdo[qq * D + d];
          part = warp_sum(part);
          if (lane == 0) sdelta[qq] = part;
        }
      }
      __syncthreads();
      const int qr = q0 + lane;
      float dot = 0.0f, dov = 0.0f;
      for (int d = 0; d < D; ++d) {
        dot += sq[lane * D + d] * sk[warp * D + d];
        dov += sdo[lane * D + d] * sv[warp * D + d];
      }
      float pr = expf(dot * scale - sl[lane]);
      if (qr >= Sq || kr >= Sk || (causal && kr > qr)) pr = 0.0f;
      const float ds = pr * (dov - sdelta[lane]);
      for (int qq = 0; qq < kF32Tile; ++qq) {
        const float pq = __shfl_sync(0xffffffffu, pr, qq);
        const float dsq = __shfl_sync(0xffffffffu, ds, qq);
#pragma unroll
        for (int i = 0; i < kF32MaxD / 32; ++i) {
          const int d = lane + 32 * i;
          if (d < D) {
            gv[i] += pq * sdo[qq * D + d];
            gk[i] += dsq * sq[qq * D + d] * scale;
          }
        }
      }
    }
  }
  if (kr < Sk) {
    float* ok = dk + ((size_t)bkv * Sk + kr) * D;
    float* ov = dv + ((size_t)bkv * Sk + kr) * D;
#pragma unroll
    for (int i = 0; i < kF32MaxD / 32; ++i) {
      const int d = lane + 32 * i;
      if (d < D) {
        ok[d] = gk[i];
        ov[d] = gv[i];
      }
    }
  }
}

}  // namespace tfb
