// rope_transpose.cuh -- RoPE and the [B,S,H,D] <-> [B,H,S,D] head transpose.
//
// Reference kernels (teenyformers):
//   rope_forward / rope_backward       src/kernels/rope.rs:57-140
//   transpose_heads / merge_heads      src/kernels/transpose_heads.rs:49-96
// The attention layer applies transpose_heads and then RoPE
// (src/layers/attention.rs:97-123); the two commute per (s, h) row, so the
// fused kernel reads a [B,S,H,D] row, rotates it and writes it to its
// [B,H,S,D] place in one pass (and the inverse for the backward).
//
// Angles follow rope.rs:86-93: inv_freq_k = exp(k * (-2 ln(base) / D)),
// theta = pos * inv_freq_k, pos = s.  Pairs are interleaved (2k, 2k+1) as in
// the reference, or rotate-half (k, k + D/2).  Arithmetic in fp32.
//
// HBM-bound: every element is read once and written once with 16-byte
// vector accesses; each row is a contiguous D*elem-byte run on both sides.
// One CTA handles one position s for a block of (b, h) rows: the position's
// D/2 (cos, sin) pairs are computed once into shared memory and reused across
// the rows.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace tfb {

enum RopeLayout { LAYOUT_BSHD = 0, LAYOUT_BHSD = 1 };

template <typename T>
struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
};

__device__ __forceinline__ void unpack16(const uint4& v, float (&f)[8], __nv_bfloat16) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
__device__ __forceinline__ uint4 pack16(const float (&f)[8], __nv_bfloat16) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(f[2 * i + 1]), "f"(f[2 * i]));
    w[i] = r;
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
__device__ __forceinline__ void unpack16(const uint4& v, float (&f)[4], float) {
  f[0] = __uint_as_float(v.x);
  f[1] = __uint_as_float(v.y);
  f[2] = __uint_as_float(v.z);
  f[3] = __uint_as_float(v.w);
}
__device__ __forceinline__ uint4 pack16(const float (&f)[4], float) {
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                    __float_as_uint(f[3]));
}

__device__ __forceinline__ size_t row_offset(int layout, int b, int s, int h, int S, int H) {
  return layout == LAYOUT_BSHD ? ((size_t)b * S + s) * H + h : ((size_t)b * H + h) * S + s;
}

constexpr int kRopeMaxHalf = 1024;  // D <= 2048

// grid = (S, ceil(B*H / rows_per_cta)), block = 256.
// STYLE 0: interleaved pairs; 1: rotate-half.  INV: inverse rotation.
template <typename T, int STYLE, bool INV>
__global__ void __launch_bounds__(256)
    rope_rows_kernel(const T* __restrict__ x, T* __restrict__ y, int B, int S, int H, int D,
                     int in_layout, int out_layout, float coef, int rows_per_cta) {
  constexpr int EPV = Vec16<T>::N;  // elements per 16-byte vector
  const int s = blockIdx.x;
  // each thread handles two 16-byte vectors of a row, c and c + D / (2 EPV):
  // the partner halves for rotate-half; for interleaved pairs (which sit
  // inside a vector) the same layout keeps both styles' accesses identical
  const int cpr = D / (2 * EPV);
  const int rows_per_pass = blockDim.x / cpr;
  const int c = threadIdx.x % cpr;
  const int r0 = threadIdx.x / cpr;
  const int row_lo = blockIdx.y * rows_per_cta;
  const int row_hi = min(B * H, row_lo + rows_per_cta);

  const size_t row_elems = (size_t)D;
  const int half_vecs = D / (2 * EPV);
  auto src_of = [&](int r) {
    const int b = r / H, h = r % H;
    return reinterpret_cast<const uint4*>(x + row_offset(in_layout, b, s, h, S, H) * row_elems);
  };
  // The first kPre rows' loads (vector pairs) go out before the angles are
  // computed, so the memory system is busy while the CTA evaluates them.
  constexpr int kPre = 4;
  const bool active = r0 < rows_per_pass;
  uint4 pre0[kPre], pre1[kPre];
#pragma unroll
  for (int j = 0; j < kPre; ++j) {
    const int r = row_lo + r0 + j * rows_per_pass;
    if (active && r < row_hi) {
      const uint4* sp = src_of(r);
      pre0[j] = __ldcs(sp + c);
      pre1[j] = __ldcs(sp + c + half_vecs);
    }
  }

  // The D/2 angles of this position, computed once per CTA (each pair by one
  // thread) and shared: a thread then reads the pairs it owns.
  __shared__ float2 ang[kRopeMaxHalf];
  for (int k = threadIdx.x; k < D / 2; k += blockDim.x) {
    const float inv_freq = expf((float)k * coef);
    const float theta = (float)s * inv_freq;
    float sv, cv;
    sincosf(theta, &sv, &cv);
    ang[k] = make_float2(cv, INV ? -sv : sv);
  }
  __syncthreads();
  if (!active) return;
  // this thread's EPV angles: interleaved, the pairs of vector c then of
  // vector c + half_vecs; rotate-half, pairs c EPV .. c EPV + EPV - 1
  float cs[EPV], sn[EPV];
#pragma unroll
  for (int i = 0; i < EPV; ++i) {
    const int k = STYLE == 0 ? (i < EPV / 2 ? c * (EPV / 2) + i
                                            : (c + half_vecs) * (EPV / 2) + i - EPV / 2)
                             : c * EPV + i;
    const float2 a = ang[k];
    cs[i] = a.x;
    sn[i] = a.y;
  }

  // rotates row r's vector(s) v0 (and v1 for rotate-half) and stores them
  auto rotate_store = [&](int r, const uint4& v0, const uint4& v1) {
    const int b = r / H, h = r % H;
    uint4* dst = reinterpret_cast<uint4*>(y + row_offset(out_layout, b, s, h, S, H) * row_elems);
    if (STYLE == 0) {
      float f0[EPV], f1[EPV];
      unpack16(v0, f0, T());
      unpack16(v1, f1, T());
#pragma unroll
      for (int i = 0; i < EPV / 2; ++i) {
        const float a = f0[2 * i], bb = f0[2 * i + 1];
        f0[2 * i] = a * cs[i] - bb * sn[i];
        f0[2 * i + 1] = a * sn[i] + bb * cs[i];
        const float a1 = f1[2 * i], b1 = f1[2 * i + 1];
        f1[2 * i] = a1 * cs[EPV / 2 + i] - b1 * sn[EPV / 2 + i];
        f1[2 * i + 1] = a1 * sn[EPV / 2 + i] + b1 * cs[EPV / 2 + i];
      }
      __stcs(dst + c, pack16(f0, T()));
      __stcs(dst + c + half_vecs, pack16(f1, T()));
    } else {
      float f0[EPV], f1[EPV];
      unpack16(v0, f0, T());
      unpack16(v1, f1, T());
#pragma unroll
      for (int i = 0; i < EPV; ++i) {
        const float a = f0[i], bb = f1[i];
        f0[i] = a * cs[i] - bb * sn[i];
        f1[i] = a * sn[i] + bb * cs[i];
      }
      __stcs(dst + c, pack16(f0, T()));
      __stcs(dst + c + half_vecs, pack16(f1, T()));
    }
  };
#pragma unroll
  for (int j = 0; j < kPre; ++j) {
    const int r = row_lo + r0 + j * rows_per_pass;
    if (r < row_hi) rotate_store(r, pre0[j], pre1[j]);
  }
#pragma unroll 8
  for (int r = row_lo + r0 + kPre * rows_per_pass; r < row_hi; r += rows_per_pass) {
    const uint4* sp = src_of(r);
    const uint4 v0 = __ldcs(sp + c);
    const uint4 v1 = __ldcs(sp + c + half_vecs);
    rotate_store(r, v0, v1);
  }
}

// (cos, sin) of every (position s, pair k) with the angle arithmetic of
// rope_rows_kernel: cs[s * half + k] = (cos, sin)(s * exp(k * coef)).  The
// GEMM epilogue that applies RoPE reads this table.
__global__ void __launch_bounds__(256)
    rope_table_kernel(float2* __restrict__ cs, int S, int half, float coef) {
  const long long total = (long long)S * half;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int s = (int)(i / half), k = (int)(i % half);
    const float inv_freq = expf((float)k * coef);
    const float theta = (float)s * inv_freq;
    float sv, cv;
    sincosf(theta, &sv, &cv);
    cs[i] = make_float2(cv, sv);
  }
}

// Pure copy between [B,S,H,D] and [B,H,S,D] (either direction) for rows of
// whole 16-byte vectors (vpr per row): laid out like rope_rows_kernel -- one
// CTA per position s covers its (b, h) rows (split over blockIdx.y when S is
// small), a thread copies one vector column of a row per pass, streaming
// loads and stores.  Bit-exact.
__global__ void __launch_bounds__(256)
    transpose_rows16_kernel(const uint4* __restrict__ x, uint4* __restrict__ y, int B, int S,
                            int H, int vpr, int in_layout, int out_layout, int rows_per_cta) {
  const int s = blockIdx.x;
  const int rows_per_pass = blockDim.x / vpr;
  const int c = threadIdx.x % vpr;
  const int r0 = threadIdx.x / vpr;
  if (r0 >= rows_per_pass) return;
  const int row_lo = blockIdx.y * rows_per_cta;
  const int row_hi = min(B * H, row_lo + rows_per_cta);
#pragma unroll 8
  for (int r = row_lo + r0; r < row_hi; r += rows_per_pass) {
    const int b = r / H, h = r % H;
    const uint4 v = __ldcs(x + row_offset(in_layout, b, s, h, S, H) * vpr + c);
    __stcs(y + row_offset(out_layout, b, s, h, S, H) * vpr + c, v);
  }
}

// Pure copy between [B,S,H,D] and [B,H,S,D] (either direction), any element
// size: bit-exact.  VEC = bytes moved per access (16, 8, 4, 2 or 1).  Used
// when rows are not whole 16-byte vectors or pointers are not 16-byte aligned.
template <typename V>
__global__ void __launch_bounds__(256)
    transpose_rows_kernel(const V* __restrict__ x, V* __restrict__ y, int B, int S, int H,
                          int vecs_per_row, int in_layout, int out_layout, long long total) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % vecs_per_row);
    const long long row = i / vecs_per_row;  // enumerated in the input layout
    int b, s, h;
    if (in_layout == LAYOUT_BSHD) {
      h = (int)(row % H);
      s = (int)((row / H) % S);
      b = (int)(row / ((long long)H * S));
    } else {
      s = (int)(row % S);
      h = (int)((row / S) % H);
      b = (int)(row / ((long long)H * S));
    }
    const size_t out_row = row_offset(out_layout, b, s, h, S, H);
    y[out_row * vecs_per_row + c] = x[(size_t)row * vecs_per_row + c];
  }
}

}  // namespace tfb
