// norm_act.cuh -- the Llama block's elementwise/row kernels around the
// attention path (needed for the tensor-parallel layer, BASELINE config #5):
//   - RMSNorm, optionally fused with the residual add: h = x + r,
//     y = h * rsqrt(mean(h^2) + eps) * gamma
//     (teenyformers src/kernels/fused_add_rmsnorm.rs:53-110; the layers use
//     teeny-core RmsNorm, src/layers/mod.rs:61-65, i.e. the same with r = 0)
//   - SwiGLU: out[m, n] = silu(z[m, n]) * z[m, n + d_ff] on z = [gate || up]
//     (src/kernels/swiglu.rs:56-95)
// bf16 in/out, fp32 arithmetic.  Both are HBM-bound: every element is read
// and written once with 16-byte vector accesses.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace tfb {

__device__ __forceinline__ void bf16x8_to_f32(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
__device__ __forceinline__ uint4 f32_to_bf16x8(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(f[2 * i + 1]), "f"(f[2 * i]));
    w[i] = r;
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// One CTA of 128 threads per row; a row of N (N % 8 == 0, N <= 128 * 8 * VPT)
// elements stays in registers between the sum-of-squares and the scaling pass.
template <int VPT>  // 16-byte vectors per thread
__global__ void __launch_bounds__(128)
    rmsnorm_rows_kernel(const __nv_bfloat16* __restrict__ x,
                        const __nv_bfloat16* __restrict__ residual,
                        const __nv_bfloat16* __restrict__ weight, __nv_bfloat16* __restrict__ y,
                        __nv_bfloat16* __restrict__ h_out, int N, float eps) {
  const size_t row = blockIdx.x;
  const int nvec = N / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * N);
  const uint4* rr = residual ? reinterpret_cast<const uint4*>(residual + row * N) : nullptr;
  float h[VPT][8];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * 128;
    if (v < nvec) {
      bf16x8_to_f32(xr[v], h[i]);
      if (rr) {
        float r8[8];
        bf16x8_to_f32(rr[v], r8);
#pragma unroll
        for (int e = 0; e < 8; ++e) h[i][e] += r8[e];
        if (h_out) reinterpret_cast<uint4*>(h_out + row * N)[v] = f32_to_bf16x8(h[i]);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(h[i][e], h[i][e], ss);
    }
  }
  __shared__ float red[4];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  const float total = (red[0] + red[1]) + (red[2] + red[3]);
  const float rstd = rsqrtf(total / (float)N + eps);
  const uint4* wr = reinterpret_cast<const uint4*>(weight);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * 128;
    if (v < nvec) {
      float w8[8], o8[8];
      bf16x8_to_f32(wr[v], w8);
#pragma unroll
      for (int e = 0; e < 8; ++e) o8[e] = h[i][e] * rstd * w8[e];
      reinterpret_cast<uint4*>(y + row * N)[v] = f32_to_bf16x8(o8);
    }
  }
}

// grid-stride over 8-element groups of the [M, d_ff] output
__global__ void __launch_bounds__(256)
    swiglu_kernel(const __nv_bfloat16* __restrict__ z, __nv_bfloat16* __restrict__ out,
                  long long rows, int d_ff) {
  const int vpr = d_ff / 8;
  const long long total = rows * vpr;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long m = i / vpr;
    const int c = (int)(i % vpr);
    const uint4* zr = reinterpret_cast<const uint4*>(z + (size_t)m * 2 * d_ff);
    float g[8], u[8], o[8];
    bf16x8_to_f32(zr[c], g);
    bf16x8_to_f32(zr[c + vpr], u);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = g[e] / (1.0f + __expf(-g[e])) * u[e];
    reinterpret_cast<uint4*>(out + (size_t)m * d_ff)[c] = f32_to_bf16x8(o);
  }
}

}  // namespace tfb
