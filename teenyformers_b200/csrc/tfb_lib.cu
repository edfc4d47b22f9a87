// tfb_lib.cu -- the C ABI (include/teenyformers_b200.h) over the sm_100a
// kernels.  One translation unit: the kernels share the device status word.
//
// Every entry point validates shapes, pointers and alignment on the host and
// returns a tf_status; nothing here allocates device memory or synchronises
// (except tf_b200_device_status).  Global state is limited to per-device
// one-time kernel attribute setup and the cached driver entry point for
// tensor-map encoding, both initialised under std::call_once.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <atomic>
#include <mutex>

#include "../../include/teenyformers_b200.h"
#include "sm100.cuh"
#include "attn_fwd.cuh"
#include "attn_bwd.cuh"
#include "attn_bwd_fused.cuh"
#include "attn_decode.cuh"
#include "attn_f32.cuh"
#include "rope_transpose.cuh"
#include "norm_act.cuh"
#include "comm_norm.cuh"
#include "gemm_sm100.cuh"

using namespace tfb;

namespace {

constexpr int kMaxDevices = 64;

bool is_aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int launch_status() {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TF_OK : TF_ERR_CUDA;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 3-D bf16 tensor map over [outer, rows, D] with a (64 x 128 x 1) box and
// 128-byte swizzle: the K-major SW128 canonical layout the MMAs read.
bool make_bf16_map(CUtensorMap* map, const void* base, int D, int rows, int outer,
                   int box_rows) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)rows, (cuuint64_t)outer};
  cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)D * 2 * (cuuint64_t)rows};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r =
      enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
          estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2-D fp32 tensor map over the [rows, D] dQ accumulator, (32 x 128) box,
// 128-byte swizzle (the staging tile the reduction warps write).
bool make_f32_acc_map(CUtensorMap* map, const void* base, int D, long long rows) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)D * 4};
  cuuint32_t box[2] = {32, 128};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r =
      enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box,
          estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2-D bf16 tensor map over a row-major [rows, inner] matrix, (64 x box_rows)
// box, 128-byte swizzle (the GEMM operand k-blocks).
bool make_bf16_2d_map(CUtensorMap* map, const void* base, long long inner, long long rows,
                      int box_rows) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)inner * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r =
      enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
          estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}

int g_num_sms[kMaxDevices];
int g_pair_clusters[kMaxDevices];

// Raises the dynamic shared-memory limit of every kernel that needs more
// than 48 KB and records the SM count, once per device.
int ensure_device_setup() {
  static std::once_flag flags[kMaxDevices];
  static int status[kMaxDevices];
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return TF_ERR_CUDA;
  std::call_once(flags[dev], [dev] {
    cudaError_t e = cudaDeviceGetAttribute(&g_num_sms[dev], cudaDevAttrMultiProcessorCount, dev);
    auto set = [&](const void* fn, int bytes) {
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    };
    set((const void*)fa_fwd_sm100_kernel<64>, FwdCfg<64>::SMEM_BYTES);
    set((const void*)fa_fwd_sm100_kernel<128>, FwdCfg<128>::SMEM_BYTES);
    set((const void*)fa_bwd_dkdv_sm100_kernel<64>, BwdKvCfg<64>::SMEM_BYTES);
    set((const void*)fa_bwd_dkdv_sm100_kernel<128>, BwdKvCfg<128>::SMEM_BYTES);
    set((const void*)fa_bwd_dq_sm100_kernel<64>, BwdQCfg<64>::SMEM_BYTES);
    set((const void*)fa_bwd_dq_sm100_kernel<128>, BwdQCfg<128>::SMEM_BYTES);
    set((const void*)fa_bwd_fused_sm100_kernel<64>, BwdFusedCfg<64>::SMEM_BYTES);
    set((const void*)fa_bwd_fused_sm100_kernel<128>, BwdFusedCfg<128>::SMEM_BYTES);
    set((const void*)fa_decode_kernel<64>, DecCfg<64>::SMEM_BYTES);
    set((const void*)fa_decode_kernel<128>, DecCfg<128>::SMEM_BYTES);
    set((const void*)gemm_bf16_sm100_pair_kernel<GEMM_EPI_STORE>, GemmPairCfg::SMEM_ALLOC);
    set((const void*)gemm_bf16_sm100_pair_kernel<GEMM_EPI_SWIGLU>, GemmPairCfg::SMEM_ALLOC);
    set((const void*)gemm_bf16_sm100_pair_kernel<GEMM_EPI_QKV_ROPE>, GemmPairCfg::SMEM_ALLOC);
    set((const void*)gemm_bf16_sm100_pair_kernel<GEMM_EPI_PUSH>, GemmPairCfg::SMEM_ALLOC);
    // CTA pairs that fit at once (SMs pair up within a GPC; one CTA per SM)
    g_pair_clusters[dev] = g_num_sms[dev] / 2;
    if (e == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2, 1, 1);
      cfg.blockDim = dim3(kGemmThreads, 1, 1);
      cfg.dynamicSmemBytes = GemmPairCfg::SMEM_ALLOC;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(
              &n, (const void*)gemm_bf16_sm100_pair_kernel<GEMM_EPI_STORE>, &cfg) == cudaSuccess &&
          n > 0)
        g_pair_clusters[dev] = n;
      else
        (void)cudaGetLastError();
    }
    const int f32_max = (3 * kF32Rows + 3 * kF32Tile) * kF32MaxD * 4 + 2 * kF32Tile * 4;
    set((const void*)fa_fwd_f32_kernel, f32_max);
    set((const void*)fa_bwd_dq_f32_kernel, f32_max);
    set((const void*)fa_bwd_dkdv_f32_kernel, f32_max);
    status[dev] = e == cudaSuccess ? TF_OK : TF_ERR_CUDA;
  });
  return status[dev];
}

bool fits_i32(long long v) { return v >= 0 && v <= 0x7fffffffLL; }

// Persistent grids: one CTA per SM (these kernels hold one CTA per SM).
unsigned persistent_grid(long long items) {
  const int dev = current_device();
  const long long sms = (dev >= 0 && dev < kMaxDevices && g_num_sms[dev] > 0) ? g_num_sms[dev] : 148;
  return (unsigned)(items < sms ? items : sms);
}

}  // namespace

// ===================================================================== library
extern "C" int tf_b200_version(void) { return 1; }

extern "C" const char* tf_b200_status_string(int s) {
  switch (s) {
    case TF_OK: return "ok";
    case TF_ERR_INVALID_ARG: return "invalid argument";
    case TF_ERR_UNSUPPORTED: return "unsupported configuration";
    case TF_ERR_MISALIGNED: return "misaligned pointer";
    case TF_ERR_CUDA: return "CUDA error";
    case TF_ERR_TOO_LARGE: return "problem too large";
    case TF_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    default: return "unknown status";
  }
}

extern "C" int tf_b200_device_status(int clear) {
  if (cudaDeviceSynchronize() != cudaSuccess) return TF_ERR_CUDA;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, tfb::g_device_status, sizeof(int)) != cudaSuccess)
    return TF_ERR_CUDA;
  if (clear) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(tfb::g_device_status, &zero, sizeof(int)) != cudaSuccess)
      return TF_ERR_CUDA;
  }
  return v;
}

// ===================================================================== attention bf16
extern "C" int tf_b200_flash_attn2_fwd_bf16(const void* q, const void* k, const void* v,
                                            void* o, float* lse, int batch, int n_heads_q,
                                            int n_heads_kv, int n_ctx_q, int n_ctx_k,
                                            int head_dim, float softmax_scale, int causal,
                                            void* stream) {
  if (batch < 0 || n_heads_q < 0 || n_heads_kv < 0 || n_ctx_q < 0 || n_ctx_k < 0)
    return TF_ERR_INVALID_ARG;
  if (batch == 0 || n_heads_q == 0 || n_ctx_q == 0) return TF_OK;
  if (n_ctx_k == 0 || n_heads_kv == 0) return TF_ERR_INVALID_ARG;
  if (n_heads_q % n_heads_kv != 0) return TF_ERR_UNSUPPORTED;
  if (head_dim != 64 && head_dim != 128) return TF_ERR_UNSUPPORTED;
  if (!q || !k || !v || !o || !lse) return TF_ERR_INVALID_ARG;
  if (!is_aligned(q, 16) || !is_aligned(k, 16) || !is_aligned(v, 16) || !is_aligned(o, 16) ||
      !is_aligned(lse, 4))
    return TF_ERR_MISALIGNED;
  if (!(softmax_scale > 0.0f) || !std::isfinite(softmax_scale)) return TF_ERR_INVALID_ARG;
  const long long bhq = (long long)batch * n_heads_q;
  const long long n_pairs = (n_ctx_q + 255) / 256;
  if (!fits_i32(bhq) || !fits_i32(bhq * n_pairs) || !fits_i32((long long)batch * n_heads_kv))
    return TF_ERR_TOO_LARGE;
  if (int st = ensure_device_setup()) return st;

  CUtensorMap tq, tk, tv, to;
  if (!make_bf16_map(&tq, q, head_dim, n_ctx_q, (int)bhq, 128) ||
      !make_bf16_map(&tk, k, head_dim, n_ctx_k, batch * n_heads_kv, 128) ||
      !make_bf16_map(&tv, v, head_dim, n_ctx_k, batch * n_heads_kv, 128) ||
      !make_bf16_map(&to, o, head_dim, n_ctx_q, (int)bhq, 128))
    return TF_ERR_CUDA;
  FwdParams prm;
  prm.o = static_cast<__nv_bfloat16*>(o);
  prm.lse = lse;
  prm.Sq = n_ctx_q;
  prm.Sk = n_ctx_k;
  prm.Hq = n_heads_q;
  prm.Hkv = n_heads_kv;
  prm.BHq = (int)bhq;
  prm.n_pairs = (int)n_pairs;
  // causal with all of K and V within the L2 size (126 MB): longest-first item order
  prm.heavy_first = (causal && 2LL * batch * n_heads_kv * n_ctx_k * head_dim * 2 <= (128LL << 20)) ? 1 : 0;
  prm.scale_log2 = softmax_scale * 1.4426950408889634f;
  prm.causal = causal ? 1 : 0;
  const dim3 grid(persistent_grid(bhq * n_pairs));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (head_dim == 128)
    fa_fwd_sm100_kernel<128><<<grid, FwdCfg<128>::kThreads, FwdCfg<128>::SMEM_BYTES, st>>>(
        tq, tk, tv, to, prm);
  else
    fa_fwd_sm100_kernel<64><<<grid, FwdCfg<64>::kThreads, FwdCfg<64>::SMEM_BYTES, st>>>(
        tq, tk, tv, to, prm);
  return launch_status();
}

extern "C" size_t tf_b200_flash_attn2_bwd_workspace_size(int batch, int n_heads_q,
                                                         int n_ctx_q) {
  if (batch <= 0 || n_heads_q <= 0 || n_ctx_q <= 0) return 0;
  // sizes the backward itself rejects as too large get 0 (and no overflow)
  const long long bhq = (long long)batch * n_heads_q;
  if (!fits_i32(bhq) || !fits_i32(bhq * ((n_ctx_q + 127) / 128))) return 0;
  return bwd_fused_workspace_bytes(bhq, n_ctx_q);
}

namespace {

// fused = true: prep (+ accumulator zeroing), fused kernel, dQ conversion;
// workspace of bwd_fused_workspace_bytes.  fused = false: the deterministic
// two-kernel path (prep, dK/dV kernel, dQ kernel); bwd_workspace_bytes.
int bwd_bf16_impl(const void* q, const void* k, const void* v, const void* o, const void* d_o,
                  const float* lse, void* dq, void* dk, void* dv, void* workspace, int batch,
                  int n_heads_q, int n_heads_kv, int n_ctx_q, int n_ctx_k, int head_dim,
                  float softmax_scale, int causal, void* stream, bool fused) {
  if (batch < 0 || n_heads_q < 0 || n_heads_kv < 0 || n_ctx_q < 0 || n_ctx_k < 0)
    return TF_ERR_INVALID_ARG;
  if (batch == 0 || n_heads_q == 0 || (n_ctx_q == 0 && n_ctx_k == 0)) return TF_OK;
  if (n_heads_kv == 0 || n_ctx_k == 0 || n_ctx_q == 0) return TF_ERR_INVALID_ARG;
  if (n_heads_q % n_heads_kv != 0) return TF_ERR_UNSUPPORTED;
  if (head_dim != 64 && head_dim != 128) return TF_ERR_UNSUPPORTED;
  if (!q || !k || !v || !o || !d_o || !lse || !dq || !dk || !dv || !workspace)
    return TF_ERR_INVALID_ARG;
  if (!is_aligned(q, 16) || !is_aligned(k, 16) || !is_aligned(v, 16) || !is_aligned(o, 16) ||
      !is_aligned(d_o, 16) || !is_aligned(dq, 16) || !is_aligned(dk, 16) ||
      !is_aligned(dv, 16) || !is_aligned(lse, 4) || !is_aligned(workspace, 16))
    return TF_ERR_MISALIGNED;
  if (!(softmax_scale > 0.0f) || !std::isfinite(softmax_scale)) return TF_ERR_INVALID_ARG;
  const long long bhq = (long long)batch * n_heads_q;
  const long long bhkv = (long long)batch * n_heads_kv;
  // head counts first, so the products below stay far inside 64 bits
  if (!fits_i32(bhq) || !fits_i32(bhkv)) return TF_ERR_TOO_LARGE;
  if (!fits_i32(bhq * ((n_ctx_q + 127) / 128)) || !fits_i32(bhkv * ((n_ctx_k + 127) / 128)) ||
      !fits_i32(bhq * (long long)n_ctx_q))
    return TF_ERR_TOO_LARGE;
  if (int st = ensure_device_setup()) return st;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int sq_pad = (int)bwd_sq_pad(n_ctx_q);
  float* ws_lse2 = static_cast<float*>(workspace);
  float* ws_delta = ws_lse2 + bhq * sq_pad;
  const long long rows = bhq * sq_pad;
  float* dq_acc = fused ? ws_delta + bhq * sq_pad : nullptr;  // 256-byte aligned
  int* counter = fused ? reinterpret_cast<int*>(dq_acc + bhq * sq_pad * 128) : nullptr;
  if (head_dim == 128)
    fa_bwd_prep_kernel<128><<<(unsigned)((rows + 15) / 16), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(o), static_cast<const __nv_bfloat16*>(d_o), lse,
        ws_lse2, ws_delta, dq_acc, counter, n_ctx_q, sq_pad, rows);
  else
    fa_bwd_prep_kernel<64><<<(unsigned)((rows + 15) / 16), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(o), static_cast<const __nv_bfloat16*>(d_o), lse,
        ws_lse2, ws_delta, dq_acc, counter, n_ctx_q, sq_pad, rows);
  if (int e = launch_status()) return e;

  CUtensorMap tq, tdo, tk, tv;
  if (!make_bf16_map(&tq, q, head_dim, n_ctx_q, (int)bhq, 128) ||
      !make_bf16_map(&tdo, d_o, head_dim, n_ctx_q, (int)bhq, 128) ||
      !make_bf16_map(&tk, k, head_dim, n_ctx_k, (int)bhkv, 128) ||
      !make_bf16_map(&tv, v, head_dim, n_ctx_k, (int)bhkv, 128))
    return TF_ERR_CUDA;
  BwdParams prm;
  prm.dq = static_cast<__nv_bfloat16*>(dq);
  prm.dk = static_cast<__nv_bfloat16*>(dk);
  prm.dv = static_cast<__nv_bfloat16*>(dv);
  prm.ws_lse2 = ws_lse2;
  prm.ws_delta = ws_delta;
  prm.Sq = n_ctx_q;
  prm.Sk = n_ctx_k;
  prm.Sq_pad = sq_pad;
  prm.Hq = n_heads_q;
  prm.Hkv = n_heads_kv;
  prm.BHq = (int)bhq;
  prm.BHkv = (int)bhkv;
  prm.n_qt = (n_ctx_q + 127) / 128;
  prm.n_kt = (n_ctx_k + 127) / 128;
  prm.scale = softmax_scale;
  prm.scale_log2 = softmax_scale * 1.4426950408889634f;
  prm.causal = causal ? 1 : 0;
  prm.work_counter = counter;
  prm.n_items = (int)(bhkv * prm.n_kt);
  const dim3 grid_kv((unsigned)(bhkv * prm.n_kt));
  if (fused) {
    if (!fits_i32(rows)) return TF_ERR_TOO_LARGE;  // accumulator row index is int
    CUtensorMap tacc, tdk, tdv;
    if (!make_f32_acc_map(&tacc, dq_acc, head_dim, rows) ||
        !make_bf16_map(&tdk, dk, head_dim, n_ctx_k, (int)bhkv, 128) ||
        !make_bf16_map(&tdv, dv, head_dim, n_ctx_k, (int)bhkv, 128))
      return TF_ERR_CUDA;
    const long long out_rows = bhq * (long long)n_ctx_q;
    const long long groups = out_rows * (head_dim / 8);
    const unsigned cgrid = (unsigned)std::min<long long>((groups + 255) / 256, 148LL * 16);
    if (head_dim == 128) {
      fa_bwd_fused_sm100_kernel<128><<<persistent_grid(prm.n_items), kFusedThreads,
                                       BwdFusedCfg<128>::SMEM_BYTES, st>>>(tq, tdo, tk, tv, tacc,
                                                                           tdk, tdv, prm);
      fa_bwd_dq_convert_kernel<128><<<cgrid, 256, 0, st>>>(
          dq_acc, prm.dq, n_ctx_q, sq_pad, out_rows, softmax_scale);
    } else {
      fa_bwd_fused_sm100_kernel<64><<<persistent_grid(prm.n_items), kFusedThreads,
                                      BwdFusedCfg<64>::SMEM_BYTES, st>>>(tq, tdo, tk, tv, tacc,
                                                                         tdk, tdv, prm);
      fa_bwd_dq_convert_kernel<64><<<cgrid, 256, 0, st>>>(
          dq_acc, prm.dq, n_ctx_q, sq_pad, out_rows, softmax_scale);
    }
    return launch_status();
  }
  const dim3 grid_q(persistent_grid(bhq * prm.n_qt));
  if (head_dim == 128) {
    fa_bwd_dkdv_sm100_kernel<128><<<grid_kv, BwdKvCfg<128>::kThreads, BwdKvCfg<128>::SMEM_BYTES,
                                    st>>>(tq, tdo, tk, tv, prm);
    fa_bwd_dq_sm100_kernel<128><<<grid_q, BwdQCfg<128>::kThreads, BwdQCfg<128>::SMEM_BYTES, st>>>(
        tk, tv, prm, static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(d_o));
  } else {
    fa_bwd_dkdv_sm100_kernel<64><<<grid_kv, BwdKvCfg<64>::kThreads, BwdKvCfg<64>::SMEM_BYTES,
                                   st>>>(tq, tdo, tk, tv, prm);
    fa_bwd_dq_sm100_kernel<64><<<grid_q, BwdQCfg<64>::kThreads, BwdQCfg<64>::SMEM_BYTES, st>>>(
        tk, tv, prm, static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(d_o));
  }
  return launch_status();
}

}  // namespace

extern "C" int tf_b200_flash_attn2_bwd_bf16(const void* q, const void* k, const void* v,
                                            const void* o, const void* d_o, const float* lse,
                                            void* dq, void* dk, void* dv, void* workspace,
                                            int batch, int n_heads_q, int n_heads_kv,
                                            int n_ctx_q, int n_ctx_k, int head_dim,
                                            float softmax_scale, int causal, void* stream) {
  return bwd_bf16_impl(q, k, v, o, d_o, lse, dq, dk, dv, workspace, batch, n_heads_q,
                       n_heads_kv, n_ctx_q, n_ctx_k, head_dim, softmax_scale, causal, stream,
                       true);
}

// ===================================================================== decode
namespace {

// Key splits of a decode call: about four CTAs per SM on a 148-SM part (two
// are resident at a time; smaller units balance varying cache lengths), at
// least 256 keys (four tiles) per split.  A pure function of the shape, so
// the workspace query and the launch agree.
struct DecodeSplit {
  int row_blocks, splits, chunk;
};
DecodeSplit decode_split(int batch, int n_heads_q, int n_heads_kv, int n_q, int cap) {
  DecodeSplit d;
  const int G = n_heads_q / n_heads_kv;
  d.row_blocks = (G * n_q + 15) / 16;
  const long long base = (long long)batch * n_heads_kv * d.row_blocks;
  long long want = (4LL * 148 + base - 1) / base;
  const long long max_splits = std::max<long long>(1, (cap + 255) / 256);
  want = std::max<long long>(1, std::min(want, max_splits));
  const long long per = (cap + want - 1) / want;
  d.chunk = (int)((per + kDecTileKeys - 1) / kDecTileKeys * kDecTileKeys);
  d.splits = (cap + d.chunk - 1) / d.chunk;
  return d;
}

}  // namespace

extern "C" size_t tf_b200_flash_attn2_decode_workspace_size(int batch, int n_heads_q,
                                                            int n_heads_kv, int n_q,
                                                            int cache_capacity, int head_dim) {
  if (batch <= 0 || n_heads_q <= 0 || n_heads_kv <= 0 || n_q <= 0 || cache_capacity <= 0 ||
      head_dim <= 0 || n_heads_q % n_heads_kv != 0)
    return 0;
  const DecodeSplit d = decode_split(batch, n_heads_q, n_heads_kv, n_q, cache_capacity);
  if (d.splits == 1) return 0;
  const size_t rows = (size_t)batch * n_heads_q * n_q;
  return (size_t)d.splits * rows * ((size_t)head_dim + 1) * 4 + 256;
}

extern "C" int tf_b200_flash_attn2_decode_bf16(const void* q, const void* k_cache,
                                               const void* v_cache, void* o, float* lse,
                                               const int* cache_seqlens, int batch,
                                               int n_heads_q, int n_heads_kv, int n_q,
                                               int cache_capacity, int head_dim,
                                               float softmax_scale, void* workspace,
                                               void* stream) {
  if (batch < 0 || n_heads_q < 0 || n_heads_kv < 0 || n_q < 0 || cache_capacity < 0)
    return TF_ERR_INVALID_ARG;
  if (batch == 0 || n_heads_q == 0 || n_q == 0) return TF_OK;
  if (n_heads_kv == 0 || cache_capacity < n_q) return TF_ERR_INVALID_ARG;
  if (n_heads_q % n_heads_kv != 0) return TF_ERR_UNSUPPORTED;
  if (head_dim != 64 && head_dim != 128) return TF_ERR_UNSUPPORTED;
  if (!q || !k_cache || !v_cache || !o || !lse || !cache_seqlens) return TF_ERR_INVALID_ARG;
  if (!is_aligned(q, 16) || !is_aligned(k_cache, 16) || !is_aligned(v_cache, 16) ||
      !is_aligned(o, 16) || !is_aligned(lse, 4) || !is_aligned(cache_seqlens, 4))
    return TF_ERR_MISALIGNED;
  if (!(softmax_scale > 0.0f) || !std::isfinite(softmax_scale)) return TF_ERR_INVALID_ARG;
  const long long bhkv = (long long)batch * n_heads_kv;
  const long long rows = (long long)batch * n_heads_q * n_q;
  const DecodeSplit d = decode_split(batch, n_heads_q, n_heads_kv, n_q, cache_capacity);
  if (!fits_i32(bhkv) || !fits_i32(rows * head_dim) || batch > 65535 ||
      (long long)n_heads_kv * d.row_blocks > 65535)
    return TF_ERR_TOO_LARGE;
  if (d.splits > 1 && (!workspace || !is_aligned(workspace, 16))) return TF_ERR_INVALID_ARG;
  if (int st = ensure_device_setup()) return st;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUtensorMap tk, tv;
  if (!make_bf16_map(&tk, k_cache, head_dim, cache_capacity, (int)bhkv, kDecTileKeys) ||
      !make_bf16_map(&tv, v_cache, head_dim, cache_capacity, (int)bhkv, kDecTileKeys))
    return TF_ERR_CUDA;
  DecodeParams prm;
  prm.q = static_cast<const __nv_bfloat16*>(q);
  prm.o = static_cast<__nv_bfloat16*>(o);
  prm.lse = lse;
  prm.seqlens = cache_seqlens;
  prm.part_lse = static_cast<float*>(workspace);
  prm.part_o = d.splits > 1 ? prm.part_lse + (((size_t)d.splits * rows + 63) / 64 * 64) : nullptr;
  prm.Hq = n_heads_q;
  prm.Hkv = n_heads_kv;
  prm.n_q = n_q;
  prm.cap = cache_capacity;
  prm.splits = d.splits;
  prm.chunk = d.chunk;
  prm.row_blocks = d.row_blocks;
  prm.scale_log2 = softmax_scale * 1.4426950408889634f;
  const dim3 grid((unsigned)d.splits, (unsigned)(n_heads_kv * d.row_blocks), (unsigned)batch);
  if (head_dim == 128)
    fa_decode_kernel<128><<<grid, kDecThreads, DecCfg<128>::SMEM_BYTES, st>>>(tk, tv, prm);
  else
    fa_decode_kernel<64><<<grid, kDecThreads, DecCfg<64>::SMEM_BYTES, st>>>(tk, tv, prm);
  if (d.splits > 1) {
    const unsigned cg = (unsigned)((rows + 7) / 8);
    if (head_dim == 128)
      fa_decode_combine_kernel<128><<<cg, 256, 0, st>>>(prm.part_o, prm.part_lse, prm.o, lse,
                                                        rows, d.splits);
    else
      fa_decode_combine_kernel<64><<<cg, 256, 0, st>>>(prm.part_o, prm.part_lse, prm.o, lse,
                                                       rows, d.splits);
  }
  return launch_status();
}

// ===================================================================== attention fp32
extern "C" int tf_b200_flash_attn2_fwd_f32(const float* q, const float* k, const float* v,
                                           float* o, float* l, int bh, int head_dim,
                                           int n_ctx_q, int n_ctx_k, float softmax_scale,
                                           float neg_inf, int causal, void* stream) {
  if (bh < 0 || head_dim < 0 || n_ctx_q < 0 || n_ctx_k < 0) return TF_ERR_INVALID_ARG;
  if (bh == 0 || n_ctx_q == 0 || head_dim == 0) return TF_OK;
  if (n_ctx_k == 0) return TF_ERR_INVALID_ARG;
  if (head_dim > kF32MaxD) return TF_ERR_UNSUPPORTED;
  if (!q || !k || !v || !o || !l) return TF_ERR_INVALID_ARG;
  if (!is_aligned(q, 4) || !is_aligned(k, 4) || !is_aligned(v, 4) || !is_aligned(o, 4) ||
      !is_aligned(l, 4))
    return TF_ERR_MISALIGNED;
  if (bh > 65535) return TF_ERR_TOO_LARGE;
  if (int st = ensure_device_setup()) return st;
  const dim3 grid((n_ctx_q + kF32Rows - 1) / kF32Rows, bh);
  const int smem = (kF32Rows + 2 * kF32Tile) * head_dim * 4;
  fa_fwd_f32_kernel<<<grid, 256, smem, static_cast<cudaStream_t>(stream)>>>(
      q, k, v, o, l, n_ctx_q, n_ctx_k, head_dim, softmax_scale, neg_inf, causal ? 1 : 0, 1, 1);
  return launch_status();
}

extern "C" int tf_b200_flash_attn2_bwd_f32(const float* q, const float* k, const float* v,
                                           const float* o, const float* d_o, const float* l,
                                           float* dq, float* dk, float* dv, int bh,
                                           int head_dim, int n_ctx_q, int n_ctx_k,
                                           float softmax_scale, int causal, void* stream) {
  if (bh < 0 || head_dim < 0 || n_ctx_q < 0 || n_ctx_k < 0) return TF_ERR_INVALID_ARG;
  if (bh == 0 || head_dim == 0 || (n_ctx_q == 0 && n_ctx_k == 0)) return TF_OK;
  if (n_ctx_q == 0 || n_ctx_k == 0) return TF_ERR_INVALID_ARG;
  if (head_dim > kF32MaxD) return TF_ERR_UNSUPPORTED;
  if (!q || !k || !v || !o || !d_o || !l || !dq || !dk || !dv) return TF_ERR_INVALID_ARG;
  if (bh > 65535) return TF_ERR_TOO_LARGE;
  if (int st = ensure_device_setup()) return st;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 gq((n_ctx_q + kF32Rows - 1) / kF32Rows, bh);
  const int smem_q = (3 * kF32Rows + 2 * kF32Tile) * head_dim * 4;
  fa_bwd_dq_f32_kernel<<<gq, 256, smem_q, st>>>(q, k, v, o, d_o, l, dq, n_ctx_q, n_ctx_k,
                                                head_dim, softmax_scale, causal ? 1 : 0, 1, 1);
  const dim3 gk((n_ctx_k + kF32Rows - 1) / kF32Rows, bh);
  const int smem_k = (2 * kF32Rows + 3 * kF32Tile) * head_dim * 4 + 2 * kF32Tile * 4;
  fa_bwd_dkdv_f32_kernel<<<gk, 256, smem_k, st>>>(q, k, v, o, d_o, l, dk, dv, n_ctx_q, n_ctx_k,
                                                  head_dim, softmax_scale, causal ? 1 : 0, 1,
                                                  1);
  return launch_status();
}

// ===================================================================== RoPE / transpose
namespace {

template <typename T>
int launch_rope(const T* x, T* y, int B, int S, int H, int D, float ln_base, int style,
                int inverse, int in_layout, int out_layout, cudaStream_t st) {
  constexpr int EPV = Vec16<T>::N;
  if (style != TF_ROPE_INTERLEAVED && style != TF_ROPE_ROTATE_HALF) return TF_ERR_INVALID_ARG;
  if (D % (2 * EPV) != 0 || D > 2048) return TF_ERR_UNSUPPORTED;
  if (!is_aligned(x, 16) || !is_aligned(y, 16)) return TF_ERR_MISALIGNED;
  const long long rows = (long long)B * H;
  if (!fits_i32(rows) || !fits_i32(rows * S) || S > 0x7fffffff) return TF_ERR_TOO_LARGE;
  const int cpr = D / (2 * EPV);  // threads per row (two vectors each)
  if (cpr > 256) return TF_ERR_UNSUPPORTED;
  const int rows_per_pass = 256 / cpr;
  // Enough CTAs to fill the GPU: split the (b, h) rows of a position only
  // when there are few positions.
  const long long target = 148LL * 8;
  long long per_cta = rows;
  if (S < target) {
    const long long split = (target + S - 1) / S;
    per_cta = (rows + split - 1) / split;
  }
  per_cta = ((per_cta + rows_per_pass - 1) / rows_per_pass) * rows_per_pass;
  const long long gy = (rows + per_cta - 1) / per_cta;
  if (gy > 65535) return TF_ERR_TOO_LARGE;
  const float coef = (-2.0f * ln_base) / (float)D;
  const dim3 grid((unsigned)S, (unsigned)gy);
#define TFB_ROPE_LAUNCH(STY, INV)                                                          \
  rope_rows_kernel<T, STY, INV><<<grid, 256, 0, st>>>(x, y, B, S, H, D, in_layout, out_layout, \
                                                      coef, (int)per_cta)
  if (style == 0 && !inverse) TFB_ROPE_LAUNCH(0, false);
  if (style == 0 && inverse) TFB_ROPE_LAUNCH(0, true);
  if (style == 1 && !inverse) TFB_ROPE_LAUNCH(1, false);
  if (style == 1 && inverse) TFB_ROPE_LAUNCH(1, true);
#undef TFB_ROPE_LAUNCH
  return launch_status();
}

int launch_transpose(const void* src, void* dst, int B, int S, int H, int D, int elem_bytes,
                     int in_layout, int out_layout, cudaStream_t st) {
  const long long row_bytes = (long long)D * elem_bytes;
  int vec = 16;
  while (vec > 1 && (row_bytes % vec != 0 || !is_aligned(src, vec) || !is_aligned(dst, vec)))
    vec >>= 1;
  if (!is_aligned(src, elem_bytes) || !is_aligned(dst, elem_bytes)) return TF_ERR_MISALIGNED;
  const long long vpr = row_bytes / vec;
  const long long total = (long long)B * S * H * vpr;
  if (!fits_i32(vpr) || !fits_i32((long long)B * S) || !fits_i32((long long)B * H))
    return TF_ERR_TOO_LARGE;
  if (vec == 16 && vpr <= 256 && S <= 0x7fffffff) {
    // whole 16-byte vectors: row-wise kernel, one CTA per position (sized as
    // for RoPE: the rows of a position split only when positions are few)
    const long long rows = (long long)B * H;
    const int rows_per_pass = (int)(256 / vpr);
    const long long target = 148LL * 8;
    long long per_cta = rows;
    if (S < target) per_cta = (rows + (target + S - 1) / S - 1) / ((target + S - 1) / S);
    per_cta = ((per_cta + rows_per_pass - 1) / rows_per_pass) * rows_per_pass;
    const long long gy = (rows + per_cta - 1) / per_cta;
    if (gy <= 65535) {
      transpose_rows16_kernel<<<dim3((unsigned)S, (unsigned)gy), 256, 0, st>>>(
          static_cast<const uint4*>(src), static_cast<uint4*>(dst), B, S, H, (int)vpr,
          in_layout, out_layout, (int)per_cta);
      return launch_status();
    }
  }
  const long long blocks_needed = (total + 255) / 256;
  const unsigned blocks = (unsigned)(blocks_needed < 148LL * 32 ? blocks_needed : 148LL * 32);
#define TFB_TR(VT)                                                                       \
  transpose_rows_kernel<VT><<<blocks, 256, 0, st>>>(static_cast<const VT*>(src),         \
                                                    static_cast<VT*>(dst), B, S, H,      \
                                                    (int)vpr, in_layout, out_layout, total)
  switch (vec) {
    case 16: TFB_TR(uint4); break;
    case 8: TFB_TR(uint2); break;
    case 4: TFB_TR(uint32_t); break;
    case 2: TFB_TR(uint16_t); break;
    default: TFB_TR(uint8_t); break;
  }
#undef TFB_TR
  return launch_status();
}

}  // namespace

extern "C" int tf_b200_rope_f32(const float* x, float* y, int bh, int n_ctx, int head_dim,
                                float ln_rope_base, int style, int inverse, void* stream) {
  if (bh < 0 || n_ctx < 0 || head_dim < 0) return TF_ERR_INVALID_ARG;
  if (bh == 0 || n_ctx == 0 || head_dim == 0) return TF_OK;
  if (!x || !y) return TF_ERR_INVALID_ARG;
  return launch_rope<float>(x, y, 1, n_ctx, bh, head_dim, ln_rope_base, style, inverse,
                            LAYOUT_BHSD, LAYOUT_BHSD, static_cast<cudaStream_t>(stream));
}

extern "C" int tf_b200_rope_bf16(const void* x, void* y, int bh, int n_ctx, int head_dim,
                                 float ln_rope_base, int style, int inverse, void* stream) {
  if (bh < 0 || n_ctx < 0 || head_dim < 0) return TF_ERR_INVALID_ARG;
  if (bh == 0 || n_ctx == 0 || head_dim == 0) return TF_OK;
  if (!x || !y) return TF_ERR_INVALID_ARG;
  return launch_rope<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(x),
                                    static_cast<__nv_bfloat16*>(y), 1, n_ctx, bh, head_dim,
                                    ln_rope_base, style, inverse, LAYOUT_BHSD, LAYOUT_BHSD,
                                    static_cast<cudaStream_t>(stream));
}

extern "C" int tf_b200_rope_transpose_bf16(const void* x, void* y, int batch, int seq_len,
                                           int n_heads, int head_dim, float ln_rope_base,
                                           int style, int inverse, void* stream) {
  if (batch < 0 || seq_len < 0 || n_heads < 0 || head_dim < 0) return TF_ERR_INVALID_ARG;
  if (batch == 0 || seq_len == 0 || n_heads == 0 || head_dim == 0) return TF_OK;
  if (!x || !y || x == y) return TF_ERR_INVALID_ARG;
  return launch_rope<__nv_bfloat16>(
      static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(y), batch, seq_len,
      n_heads, head_dim, ln_rope_base, style, inverse, inverse ? LAYOUT_BHSD : LAYOUT_BSHD,
      inverse ? LAYOUT_BSHD : LAYOUT_BHSD, static_cast<cudaStream_t>(stream));
}

extern "C" int tf_b200_transpose_heads(const void* src, void* dst, int batch, int seq_len,
                                       int n_heads, int head_dim, int elem_bytes,
                                       void* stream) {
  if (batch < 0 || seq_len < 0 || n_heads < 0 || head_dim < 0) return TF_ERR_INVALID_ARG;
  if (elem_bytes != 2 && elem_bytes != 4) return TF_ERR_INVALID_ARG;
  if (batch == 0 || seq_len == 0 || n_heads == 0 || head_dim == 0) return TF_OK;
  if (!src || !dst || src == dst) return TF_ERR_INVALID_ARG;
  return launch_transpose(src, dst, batch, seq_len, n_heads, head_dim, elem_bytes, LAYOUT_BSHD,
                          LAYOUT_BHSD, static_cast<cudaStream_t>(stream));
}

extern "C" int tf_b200_merge_heads(const void* src, void* dst, int batch, int seq_len,
                                   int n_heads, int head_dim, int elem_bytes, void* stream) {
  if (batch < 0 || seq_len < 0 || n_heads < 0 || head_dim < 0) return TF_ERR_INVALID_ARG;
  if (elem_bytes != 2 && elem_bytes != 4) return TF_ERR_INVALID_ARG;
  if (batch == 0 || seq_len == 0 || n_heads == 0 || head_dim == 0) return TF_OK;
  if (!src || !dst || src == dst) return TF_ERR_INVALID_ARG;
  return launch_transpose(src, dst, batch, seq_len, n_heads, head_dim, elem_bytes, LAYOUT_BHSD,
                          LAYOUT_BSHD, static_cast<cudaStream_t>(stream));
}

// ===================================================================== Llama-block row kernels
extern "C" int tf_b200_rmsnorm_bf16(const void* x, const void* residual, const void* weight,
                                    void* y, void* h_out, int rows, int cols, float eps,
                                    void* stream) {
  if (rows < 0 || cols < 0) return TF_ERR_INVALID_ARG;
  if (rows == 0 || cols == 0) return TF_OK;
  if (!x || !weight || !y || (h_out && !residual)) return TF_ERR_INVALID_ARG;
  if (cols % 8 != 0 || cols > 128 * 8 * 8) return TF_ERR_UNSUPPORTED;
  if (!is_aligned(x, 16) || !is_aligned(weight, 16) || !is_aligned(y, 16) ||
      (residual && !is_aligned(residual, 16)) || (h_out && !is_aligned(h_out, 16)))
    return TF_ERR_MISALIGNED;
  if (!(eps >= 0.0f) || !std::isfinite(eps)) return TF_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const auto* xp = static_cast<const __nv_bfloat16*>(x);
  const auto* rp = static_cast<const __nv_bfloat16*>(residual);
  const auto* wp = static_cast<const __nv_bfloat16*>(weight);
  auto* yp = static_cast<__nv_bfloat16*>(y);
  auto* hp = static_cast<__nv_bfloat16*>(h_out);
  const int vpt = (cols / 8 + 127) / 128;
  if (vpt <= 2)
    rmsnorm_rows_kernel<2><<<rows, 128, 0, st>>>(xp, rp, wp, yp, hp, cols, eps);
  else if (vpt <= 4)
    rmsnorm_rows_kernel<4><<<rows, 128, 0, st>>>(xp, rp, wp, yp, hp, cols, eps);
  else
    rmsnorm_rows_kernel<8><<<rows, 128, 0, st>>>(xp, rp, wp, yp, hp, cols, eps);
  return launch_status();
}

extern "C" int tf_b200_allreduce_residual_rmsnorm_bf16(
    const void* const* peer_src, void* const* peer_h, void* const* peer_signal,
    const void* residual, const void* weight, void* y, int rank, int world, int rows, int cols,
    float eps, unsigned epoch, void* stream) {
  if (rows < 0 || cols < 0 || world < 1 || world > kArMaxWorld || rank < 0 || rank >= world)
    return TF_ERR_INVALID_ARG;
  if (rows == 0 || cols == 0) return TF_OK;
  if (!peer_src || !peer_h || !peer_signal) return TF_ERR_INVALID_ARG;
  if ((weight == nullptr) != (y == nullptr)) return TF_ERR_INVALID_ARG;
  if (rows % world != 0 || cols % 8 != 0) return TF_ERR_UNSUPPORTED;
  if (!is_aligned(residual, 16) || !is_aligned(weight, 16) || !is_aligned(y, 16))
    return TF_ERR_MISALIGNED;
  if (epoch == 0) return TF_ERR_INVALID_ARG;  // flags start at 0: epochs count from 1
  auto launch = [&](auto kernel) {
    kernel<<<kArCtas, kArThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const __nv_bfloat16* const*>(peer_src),
        reinterpret_cast<__nv_bfloat16* const*>(peer_h),
        reinterpret_cast<uint32_t* const*>(peer_signal), static_cast<const __nv_bfloat16*>(residual),
        static_cast<const __nv_bfloat16*>(weight), static_cast<__nv_bfloat16*>(y), rank, world, rows,
        cols, eps, epoch);
  };
  if (world <= 2)
    launch(allreduce_residual_rmsnorm_kernel<2>);
  else if (world <= 4)
    launch(allreduce_residual_rmsnorm_kernel<4>);
  else
    launch(allreduce_residual_rmsnorm_kernel<8>);
  return launch_status();
}

extern "C" int tf_b200_swiglu_bf16(const void* z, void* out, int rows, int d_ff, void* stream) {
  if (rows < 0 || d_ff < 0) return TF_ERR_INVALID_ARG;
  if (rows == 0 || d_ff == 0) return TF_OK;
  if (!z || !out) return TF_ERR_INVALID_ARG;
  if (d_ff % 8 != 0) return TF_ERR_UNSUPPORTED;
  if (!is_aligned(z, 16) || !is_aligned(out, 16)) return TF_ERR_MISALIGNED;
  const long long total = (long long)rows * (d_ff / 8);
  const long long blocks = (total + 255) / 256;
  swiglu_kernel<<<(unsigned)(blocks < 148LL * 16 ? blocks : 148LL * 16), 256, 0,
                  static_cast<cudaStream_t>(stream)>>>(static_cast<const __nv_bfloat16*>(z),
                                                       static_cast<__nv_bfloat16*>(out), rows,
                                                       d_ff);
  return launch_status();
}

// ===================================================================== GEMMs with fused epilogues
namespace {

// Shared validation + launch of gemm_bf16_sm100_pair_kernel.  A is row-major
// [m, k], or (a_seq > 0) the attention output [m / a_seq, k / 128, a_seq, 128].
template <int EPI>
int gemm_launch(const void* a, const void* b, int m, int n, int k, int a_seq, GemmParams& prm,
                cudaStream_t st) {
  if (!a || !b) return TF_ERR_INVALID_ARG;
  if (k % 8 != 0 || n % 8 != 0) return TF_ERR_UNSUPPORTED;
  if (!is_aligned(a, 16) || !is_aligned(b, 16)) return TF_ERR_MISALIGNED;
  if (a_seq < 0) return TF_ERR_INVALID_ARG;
  if (a_seq > 0 && (k % kGemmHeadDim != 0 || a_seq % kGemmBM != 0 || m % a_seq != 0))
    return TF_ERR_UNSUPPORTED;
  if (ensure_device_setup() != TF_OK) return TF_ERR_CUDA;
  CUtensorMap ta, tb;
  bool ok;
  if (a_seq > 0) {
    const long long outer = (long long)(m / a_seq) * (k / kGemmHeadDim);
    if (!fits_i32(outer)) return TF_ERR_TOO_LARGE;
    ok = make_bf16_map(&ta, a, kGemmHeadDim, a_seq, (int)outer, kGemmBM);
  } else {
    ok = make_bf16_2d_map(&ta, a, k, m, kGemmBM);
  }
  // CTA pairs: 256 x 256 tiles, each CTA loads 128 rows of A and of B
  if (!ok || !make_bf16_2d_map(&tb, b, k, n, 128)) return TF_ERR_CUDA;
  prm.M = m, prm.N = n, prm.K = k;
  prm.n_mblk = (m + 255) / 256;
  prm.n_nblk = (n + kGemmBN - 1) / kGemmBN;
  prm.n_kblk = (k + kGemmBK - 1) / kGemmBK;
  const long long tiles = (long long)prm.n_mblk * prm.n_nblk;
  if (!fits_i32(tiles)) return TF_ERR_TOO_LARGE;
  prm.n_tiles = (int)tiles;
  prm.group_m = std::min(prm.n_mblk, 8);
  // PUSH: rank r's walk starts with the rows of owner (r + 1) % world (each owner's
  // rows are a contiguous run of row blocks, so of tiles) and ends with its own
  prm.tile_rotate = 0;
  if (EPI == GEMM_EPI_PUSH && prm.world > 1)
    prm.tile_rotate = (int)(((long long)((prm.rank + 1) % prm.world) * tiles / prm.world) % tiles);
  prm.a_heads = a_seq > 0 ? 1 : 0;
  prm.a_seq = a_seq > 0 ? a_seq : 1;
  prm.a_n_heads = a_seq > 0 ? k / kGemmHeadDim : 0;
  const long long clusters = std::min<long long>(tiles, g_pair_clusters[current_device()]);
  gemm_bf16_sm100_pair_kernel<EPI>
      <<<(unsigned)(2 * clusters), kGemmThreads, GemmPairCfg::SMEM_ALLOC, st>>>(ta, tb, prm);
  return launch_status();
}

bool gemm_extents(int m, int n, int k, int* early) {
  *early = TF_OK;
  if (m < 0 || n < 0 || k < 0) {
    *early = TF_ERR_INVALID_ARG;
    return false;
  }
  if (m == 0 || n == 0) return false;  // nothing to write: a successful no-op
  if (k == 0) {
    *early = TF_ERR_UNSUPPORTED;
    return false;
  }
  return true;
}

}  // namespace

extern "C" int tf_b200_gemm_bf16(const void* a, const void* b, const void* residual, void* c,
                                 int m, int n, int k, int a_seq, void* stream) {
  int early;
  if (!gemm_extents(m, n, k, &early)) return early;
  if (!c) return TF_ERR_INVALID_ARG;
  if (!is_aligned(c, 16) || (residual && !is_aligned(residual, 16))) return TF_ERR_MISALIGNED;
  GemmParams prm{};
  prm.out = static_cast<__nv_bfloat16*>(c);
  prm.ld_out = n;
  prm.residual = static_cast<const __nv_bfloat16*>(residual);
  return gemm_launch<GEMM_EPI_STORE>(a, b, m, n, k, a_seq, prm,
                                     static_cast<cudaStream_t>(stream));
}

extern "C" int tf_b200_gemm_swiglu_bf16(const void* a, const void* w_gate_up, void* out, int m,
                                        int d_ff, int k, void* stream) {
  int early;
  if (d_ff < 0) return TF_ERR_INVALID_ARG;
  if (!gemm_extents(m, d_ff, k, &early)) return early;
  if (!out) return TF_ERR_INVALID_ARG;
  if (d_ff % 128 != 0 || !fits_i32(2LL * d_ff)) return TF_ERR_UNSUPPORTED;
  if (!is_aligned(out, 16)) return TF_ERR_MISALIGNED;
  GemmParams prm{};
  prm.out = static_cast<__nv_bfloat16*>(out);
  prm.ld_out = d_ff;
  return gemm_launch<GEMM_EPI_SWIGLU>(a, w_gate_up, m, 2 * d_ff, k, 0, prm,
                                      static_cast<cudaStream_t>(stream));
}

extern "C" int tf_b200_rope_table_f32(void* cs, int seq_len, int head_dim, float ln_rope_base,
                                      void* stream) {
  if (seq_len < 0 || head_dim < 0) return TF_ERR_INVALID_ARG;
  if (seq_len == 0 || head_dim == 0) return TF_OK;
  if (!cs || head_dim % 2 != 0) return TF_ERR_INVALID_ARG;
  if (!is_aligned(cs, 16)) return TF_ERR_MISALIGNED;
  if (!std::isfinite(ln_rope_base)) return TF_ERR_INVALID_ARG;
  const long long total = (long long)seq_len * (head_dim / 2);
  const long long blocks = (total + 255) / 256;
  const float coef = (-2.0f * ln_rope_base) / (float)head_dim;
  rope_table_kernel<<<(unsigned)std::min(blocks, 148LL * 8), 256, 0,
                      static_cast<cudaStream_t>(stream)>>>(static_cast<float2*>(cs), seq_len,
                                                           head_dim / 2, coef);
  return launch_status();
}

extern "C" int tf_b200_gemm_qkv_rope_bf16(const void* x, const void* w_qkv, void* q, void* k_out,
                                          void* v, const void* rope_cs, int batch, int seq_len,
                                          int n_heads_q, int n_heads_kv, int d_model,
                                          int rope_style, void* stream) {
  if (batch < 0 || seq_len < 0 || n_heads_q < 0 || n_heads_kv < 0 || d_model < 0)
    return TF_ERR_INVALID_ARG;
  const long long m = (long long)batch * seq_len;
  const long long n = (long long)(n_heads_q + 2LL * n_heads_kv) * kGemmHeadDim;
  if (!fits_i32(m) || !fits_i32(n)) return TF_ERR_TOO_LARGE;
  int early;
  if (!gemm_extents((int)m, (int)n, d_model, &early)) return early;
  if (!q || (n_heads_kv > 0 && (!k_out || !v))) return TF_ERR_INVALID_ARG;
  if (rope_style != 0 && rope_style != 1) return TF_ERR_INVALID_ARG;
  if (seq_len % kGemmBM != 0) return TF_ERR_UNSUPPORTED;
  if (!is_aligned(q, 16) || (k_out && !is_aligned(k_out, 16)) || (v && !is_aligned(v, 16)) ||
      (rope_cs && !is_aligned(rope_cs, 16)))
    return TF_ERR_MISALIGNED;
  GemmParams prm{};
  prm.q_out = static_cast<__nv_bfloat16*>(q);
  prm.k_out = static_cast<__nv_bfloat16*>(k_out);
  prm.v_out = static_cast<__nv_bfloat16*>(v);
  prm.rope_cs = static_cast<const float4*>(rope_cs);
  prm.seq = seq_len;
  prm.n_q_heads = n_heads_q;
  prm.n_kv_heads = n_heads_kv;
  prm.rope_style = rope_style;
  return gemm_launch<GEMM_EPI_QKV_ROPE>(x, w_qkv, (int)m, (int)n, d_model, 0, prm,
                                        static_cast<cudaStream_t>(stream));
}

extern "C" int tf_b200_gemm_push_bf16(const void* a, const void* b, void* const* peer_recv,
                                      int m, int n, int k, int a_seq, int rank, int world,
                                      void* stream) {
  int early;
  if (!gemm_extents(m, n, k, &early)) return early;
  if (!peer_recv || world < 1 || world > kGemmMaxPeers || rank < 0 || rank >= world)
    return TF_ERR_INVALID_ARG;
  if (m % world != 0 || (m / world) % kGemmBM != 0) return TF_ERR_UNSUPPORTED;
  GemmParams prm{};
  for (int r = 0; r < world; ++r) {
    if (!peer_recv[r]) return TF_ERR_INVALID_ARG;
    if (!is_aligned(peer_recv[r], 16)) return TF_ERR_MISALIGNED;
    prm.peer_out[r] = static_cast<__nv_bfloat16*>(peer_recv[r]);
  }
  prm.rank = rank;
  prm.world = world;
  prm.slice_rows = m / world;
  return gemm_launch<GEMM_EPI_PUSH>(a, b, m, n, k, a_seq, prm, static_cast<cudaStream_t>(stream));
}

// ===================================================================== backward, no scratch argument
namespace {

// Scratch for the allocation-free backward: the -LSE*log2(e) and -rowsum(O*dO)
// rows (2 x 1,048,576 floats = 8 MiB), written in full by every call's prep
// kernel before use, so nothing needs clearing between calls.
constexpr size_t kNoAllocWsBytes = size_t(8) << 20;
constexpr long long kNoAllocRows = (long long)(kNoAllocWsBytes / (2 * sizeof(float)));
__device__ __align__(256) float g_noalloc_ws[kNoAllocWsBytes / sizeof(float)];

// Device address of g_noalloc_ws for the current device (host code only holds
// a stand-in symbol for it).  Only a successful lookup is cached: a failed one
// (e.g. a first call made while the stream is being captured) is retried by
// the next call.  Threads racing on the first lookup store the same address.
void* noalloc_workspace(int* status) {
  static std::atomic<void*> ptrs[kMaxDevices];
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) {
    *status = TF_ERR_CUDA;
    return nullptr;
  }
  void* ptr = ptrs[dev].load(std::memory_order_acquire);
  if (ptr == nullptr) {
    if (cudaGetSymbolAddress(&ptr, g_noalloc_ws) != cudaSuccess || ptr == nullptr) {
      *status = TF_ERR_CUDA;
      return nullptr;
    }
    ptrs[dev].store(ptr, std::memory_order_release);
  }
  *status = TF_OK;
  return ptr;
}

}  // namespace

extern "C" int tf_b200_flash_attn2_bwd_bf16_noalloc(const void* q, const void* k, const void* v,
                                                   const void* o, const void* d_o,
                                                   const float* lse, void* dq, void* dk, void* dv,
                                                   int batch, int n_heads_q, int n_heads_kv,
                                                   int n_ctx_q, int n_ctx_k, int head_dim,
                                                   float softmax_scale, int causal,
                                                   void* stream) {
  if (batch < 0 || n_heads_q < 0 || n_heads_kv < 0 || n_ctx_q < 0 || n_ctx_k < 0)
    return TF_ERR_INVALID_ARG;
  if (batch == 0 || n_heads_q == 0 || (n_ctx_q == 0 && n_ctx_k == 0)) return TF_OK;
  // rows of per-row statistics the call needs: B * Hq * round_up(Sq, 128)
  // (both factors below 2^32, so the product cannot overflow)
  const long long bhq = (long long)batch * n_heads_q;
  if (!fits_i32(bhq) || bhq * bwd_sq_pad(n_ctx_q) > kNoAllocRows) return TF_ERR_TOO_LARGE;
  int st = TF_OK;
  void* ws = noalloc_workspace(&st);
  if (st != TF_OK) return st;
  // the deterministic two-kernel path: its scratch is only the per-row statistics
  return bwd_bf16_impl(q, k, v, o, d_o, lse, dq, dk, dv, ws, batch, n_heads_q, n_heads_kv,
                       n_ctx_q, n_ctx_k, head_dim, softmax_scale, causal, stream, false);
}
