/*
 * teenyformers_b200.h -- C ABI of the B200 (sm_100a) attention hot path.
 *
 * Drop-in boundary for teenyformers' attention custom ops.  In the reference
 * every op is a CustomOp/RuntimeOp pair whose kernel is reached through a
 * generated `extern "C" fn entry_point(<ptrs>, <i32s>, <f32s>)` and launched
 * by the external executor with grid()/block() and visitor-packed arguments
 * (src/kernels/flash_attn2.rs:284-575, src/kernels/rope.rs:148-281,
 * src/kernels/transpose_heads.rs:100-312).  The entry points below replace
 * those launches: same pointer order and argument meaning, plus the shape
 * values the reference passes through grid() (BH, head_dim) and a stream.
 *
 * Conventions (all entry points):
 *   - plain device pointers, caller-owned; nothing here allocates device
 *     memory.  Pointers must be 16-byte aligned (bf16 paths) or 4-byte
 *     aligned (fp32 paths).
 *   - stream-ordered on `stream` (a cudaStream_t; NULL = legacy default).
 *   - return 0 (TF_OK) on success, a negative tf_status on invalid input or
 *     launch failure; they never abort the process.  An empty problem
 *     (a zero batch/head/sequence extent) is a successful no-op.
 *   - layouts are dense row-major; "BH" = batch * heads.
 *   - bf16 tensors are passed as `void*` (IEEE bfloat16 bits), fp32 as float*.
 */
#ifndef TEENYFORMERS_B200_H
#define TEENYFORMERS_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TF_API __attribute__((visibility("default")))
#else
#define TF_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum tf_status {
  TF_OK = 0,
  TF_ERR_INVALID_ARG = -1,    /* null pointer, negative extent, bad enum */
  TF_ERR_UNSUPPORTED = -2,    /* head_dim / GQA ratio outside what is built */
  TF_ERR_MISALIGNED = -3,     /* pointer alignment below the requirement */
  TF_ERR_CUDA = -4,           /* CUDA launch or driver error */
  TF_ERR_TOO_LARGE = -5,      /* extents beyond 32-bit indexing / TMA limits */
  TF_ERR_DEVICE_TIMEOUT = -6  /* a kernel's bounded wait expired (see tf_b200_device_status) */
} tf_status;

typedef enum tf_rope_style {
  TF_ROPE_INTERLEAVED = 0, /* pairs (2k, 2k+1): the reference (rope.rs:21-26) */
  TF_ROPE_ROTATE_HALF = 1  /* pairs (k, k + D/2) */
} tf_rope_style;

/* ---------------- library ---------------- */

TF_API int tf_b200_version(void);
TF_API const char* tf_b200_status_string(int status);
/* Reads (and with clear != 0 resets) the device-side error word of the
 * current device: 0, or the site code of the first kernel wait that timed
 * out.  Synchronises the device. */
TF_API int tf_b200_device_status(int clear);

/* ---------------- flash attention, bf16, tcgen05 (sm_100a) ----------------
 * Replaces FlashAttn2RuntimeOp / CausalFlashAttn2RuntimeOp launches
 * (src/kernels/flash_attn2.rs:284-384 and :436-530), whose kernel ABI is
 * entry_point(q, k, v, o, l, n_ctx_q, n_ctx_k, softmax_scale, neg_inf)
 * (tests/snapshots/kernel_sources__causal_flash_attn2_fwd_source.snap:5).
 *   q, o  [batch * n_heads_q,  n_ctx_q, head_dim] bf16
 *   k, v  [batch * n_heads_kv, n_ctx_k, head_dim] bf16
 *   lse   [batch * n_heads_q,  n_ctx_q] fp32: m + ln(l), natural log of the
 *         scaled scores (the reference's `l` cache, flash_attn2.rs:120-122)
 *   causal != 0: key k hidden from query q when k > q (top-left aligned,
 *         flash_attn2.rs:103-107).
 *   GQA: query head h uses KV head h / (n_heads_q / n_heads_kv); the
 *   reference has MHA only (n_heads_kv == n_heads_q).
 *   head_dim: 64 or 128. */
TF_API int tf_b200_flash_attn2_fwd_bf16(const void* q, const void* k, const void* v, void* o,
                                 float* lse, int batch, int n_heads_q, int n_heads_kv,
                                 int n_ctx_q, int n_ctx_k, int head_dim, float softmax_scale,
                                 int causal, void* stream);

/* Backward.  Replaces the reference's pack_backward_args launch
 * (q, k, v, o, do, l, dq, dk, dv, n_ctx_q, n_ctx_k, softmax_scale;
 * src/kernels/flash_attn2.rs:492-519).  dq/dk/dv are fully written (the
 * reference needs dK/dV zero-initialised for its atomics; this does not).
 * `workspace` is caller-provided scratch of
 * tf_b200_flash_attn2_bwd_workspace_size(...) bytes (per-row softmax
 * statistics and an fp32 dQ accumulator, sized for head_dim <= 128); it must
 * stay untouched until the call's work completes.  dK/dV are bitwise
 * repeatable; dQ sums fp32 partials over key tiles in no fixed order (as the
 * reference's atomics do), so repeats agree to fp32 rounding. */
TF_API size_t tf_b200_flash_attn2_bwd_workspace_size(int batch, int n_heads_q, int n_ctx_q);
TF_API int tf_b200_flash_attn2_bwd_bf16(const void* q, const void* k, const void* v, const void* o,
                                 const void* d_o, const float* lse, void* dq, void* dk, void* dv,
                                 void* workspace, int batch, int n_heads_q, int n_heads_kv,
                                 int n_ctx_q, int n_ctx_k, int head_dim, float softmax_scale,
                                 int causal, void* stream);

/* Backward without caller-provided scratch.  No counterpart in the reference.
 * For callers that cannot allocate device memory at the point of the call:
 * an executor that plans every buffer up front from the ops' declared
 * shapes and hands a backward only its tensors, with no slot for extra
 * scratch, or a process that forbids allocation once it is running.
 * The per-row softmax statistics live instead in a fixed 8 MiB array inside
 * the library (held on every GPU that loads it, until exit), so
 * batch * n_heads_q * round_up(n_ctx_q, 128) must be <= 1,048,576
 * (e.g. B*H = 256 at S = 4096); larger problems return TF_ERR_TOO_LARGE.
 * The first call on a device looks the array up (cudaGetSymbolAddress) with
 * that device current; make that first call before any stream capture.  A
 * lookup that fails returns TF_ERR_CUDA and is tried again by the next call.
 * Nothing here calls cudaMalloc/cudaFree.  Every call shares the one array,
 * so calls that can overlap on the GPU (different streams) race: serialise
 * them.  Same arguments and results as tf_b200_flash_attn2_bwd_bf16 minus
 * the workspace; it runs the deterministic two-kernel backward (dQ
 * recomputed per query tile), so its results are bitwise repeatable. */
TF_API int tf_b200_flash_attn2_bwd_bf16_noalloc(const void* q, const void* k, const void* v,
                                               const void* o, const void* d_o, const float* lse,
                                               void* dq, void* dk, void* dv, int batch,
                                               int n_heads_q, int n_heads_kv, int n_ctx_q,
                                               int n_ctx_k, int head_dim, float softmax_scale,
                                               int causal, void* stream);

/* KV-cache decode attention.  No counterpart kernel in the reference: its
 * generation loop re-runs the whole prefix through the causal op for every
 * new token (examples/llama_generate.rs:373-400); this is the same softmax
 * attention (flash_attn2.rs:77-125 semantics) for the new rows only.
 *   q: [batch, n_heads_q, n_q, head_dim] bf16 (n_q new tokens per sequence)
 *   k_cache, v_cache: [batch, n_heads_kv, cache_capacity, head_dim] bf16
 *   cache_seqlens: [batch] int32 on the device, keys held per sequence
 *     (n_q <= L_b <= cache_capacity; values outside are clamped), the last
 *     n_q of which are the new tokens': query i sits at position
 *     L_b - n_q + i and sees keys 0 .. L_b - n_q + i (bottom-right causal).
 *   o: [batch, n_heads_q, n_q, head_dim] bf16; lse: [batch, n_heads_q, n_q]
 *     fp32, natural log of the scaled scores' sum.
 *   workspace: tf_b200_flash_attn2_decode_workspace_size(...) bytes (0 = none
 *     needed; NULL allowed then), 16-byte aligned.
 * head_dim 64 or 128; GQA as in the forward. */
TF_API size_t tf_b200_flash_attn2_decode_workspace_size(int batch, int n_heads_q, int n_heads_kv,
                                                        int n_q, int cache_capacity, int head_dim);
TF_API int tf_b200_flash_attn2_decode_bf16(const void* q, const void* k_cache, const void* v_cache,
                                           void* o, float* lse, const int* cache_seqlens,
                                           int batch, int n_heads_q, int n_heads_kv, int n_q,
                                           int cache_capacity, int head_dim, float softmax_scale,
                                           void* workspace, void* stream);

/* Tensor-parallel all-reduce fused with the residual add and RMSNorm after it.
 * No counterpart in the reference (its layer is single-device); it stands for
 * "sum the ranks' partial o_proj / down_proj outputs, then fused add + RMSNorm"
 * (src/layers/llama_block.rs:55-65, fused_add_rmsnorm.rs:53-110) in one kernel
 * over NVLink peer memory.
 *   peer_src, peer_h, peer_signal: DEVICE arrays of `world` pointers to every
 *     rank's [rows, cols] bf16 partial, [rows, cols] bf16 h buffer and signal
 *     pad (at least 9216 bytes, zeroed once before the first call) -- peer-
 *     mapped (symmetric) memory, e.g. torch.distributed._symmetric_memory.
 *   residual: [rows, cols] bf16, identical on every rank, or NULL.
 *   h (every rank's h buffer) = residual + sum of the partials (bf16);
 *   y = RMSNorm(h) * weight, local, when weight/y are non-NULL.
 *   epoch: 1, 2, 3, ... one per call, the same on every rank.
 * Every rank calls it with the same arguments (own rank); rows % world == 0,
 * cols % 8 == 0, world <= 8.  Its waits on peers are bounded: on expiry it sets
 * tf_b200_device_status and the outputs are invalid. */
TF_API int tf_b200_allreduce_residual_rmsnorm_bf16(const void* const* peer_src, void* const* peer_h,
                                                  void* const* peer_signal, const void* residual,
                                                  const void* weight, void* y, int rank, int world,
                                                  int rows, int cols, float eps, unsigned epoch,
                                                  void* stream);

/* ---------------- flash attention, fp32, reference argument set ----------------
 * Same tensors and argument order as the reference kernels
 * flash_attn2_causal_fwd (flash_attn2.rs:61-72, plus `neg_inf`) and
 * flash_attn2_causal_bwd / flash_attn2_backward (:135-150, :209-224), with
 * the grid extents (bh) and head_dim made explicit.  head_dim <= 256.
 * dk/dv are fully written (no zero-initialisation needed). */
TF_API int tf_b200_flash_attn2_fwd_f32(const float* q, const float* k, const float* v, float* o,
                                float* l, int bh, int head_dim, int n_ctx_q, int n_ctx_k,
                                float softmax_scale, float neg_inf, int causal, void* stream);
TF_API int tf_b200_flash_attn2_bwd_f32(const float* q, const float* k, const float* v, const float* o,
                                const float* d_o, const float* l, float* dq, float* dk,
                                float* dv, int bh, int head_dim, int n_ctx_q, int n_ctx_k,
                                float softmax_scale, int causal, void* stream);

/* ---------------- RoPE ----------------
 * Replaces RopeRtOp (src/kernels/rope.rs:148-238), kernel ABI
 * entry_point(x, y, n_ctx, ln_rope_base)
 * (tests/snapshots/kernel_sources__rope_forward_source.snap:5).
 *   x, y [bh, n_ctx, head_dim]; pos = row index within n_ctx.
 *   ln_rope_base = ln(rope_base), pre-computed by the caller as in rope.rs:194.
 *   inverse != 0: the backward rotation (rope_backward, rope.rs:104-140).
 * x == y (in place) is allowed. */
TF_API int tf_b200_rope_f32(const float* x, float* y, int bh, int n_ctx, int head_dim,
                     float ln_rope_base, int style, int inverse, void* stream);
TF_API int tf_b200_rope_bf16(const void* x, void* y, int bh, int n_ctx, int head_dim,
                      float ln_rope_base, int style, int inverse, void* stream);

/* Fused transpose + RoPE (the attention layer's TransposeHeadsOp -> RopeOp,
 * src/layers/attention.rs:97-123), batched:
 *   inverse == 0: x [batch, seq_len, n_heads, head_dim] -> y [batch, n_heads, seq_len, head_dim]
 *   inverse != 0: x [batch, n_heads, seq_len, head_dim] -> y [batch, seq_len, n_heads, head_dim]
 *                 with the backward rotation (RopeOp backward then MergeHeads).
 * x and y must not overlap. */
TF_API int tf_b200_rope_transpose_bf16(const void* x, void* y, int batch, int seq_len, int n_heads,
                                int head_dim, float ln_rope_base, int style, int inverse,
                                void* stream);

/* ---------------- head transpose / merge (bit-exact copies) ----------------
 * Replace TransposeHeads / MergeHeads (src/kernels/transpose_heads.rs:100-165,
 * :207-273), kernel ABI entry_point(src, dst, seq_len, n_heads)
 * (tests/snapshots/kernel_sources__transpose_heads_source.snap:5), batched:
 *   transpose: src [batch, seq_len, n_heads * head_dim] -> dst [batch, n_heads, seq_len, head_dim]
 *   merge:     src [batch, n_heads, seq_len, head_dim] -> dst [batch, seq_len, n_heads * head_dim]
 * elem_bytes: 2 (bf16/f16) or 4 (fp32); any bit pattern is copied unchanged. */
TF_API int tf_b200_transpose_heads(const void* src, void* dst, int batch, int seq_len, int n_heads,
                            int head_dim, int elem_bytes, void* stream);
TF_API int tf_b200_merge_heads(const void* src, void* dst, int batch, int seq_len, int n_heads,
                        int head_dim, int elem_bytes, void* stream);

/* ---------------- Llama block row kernels (tensor-parallel layer support) ----------------
 * RMSNorm with optional fused residual add; replaces the reference's
 * fused_add_rmsnorm_forward (src/kernels/fused_add_rmsnorm.rs:53-110) and, with
 * residual == NULL, the teeny-core RmsNorm the layers use (src/layers/mod.rs:61-65):
 *   h = x + residual (written to h_out if non-NULL), y = h * rsqrt(mean(h^2) + eps) * weight
 *   x, residual, y, h_out [rows, cols] bf16; weight [cols] bf16; cols % 8 == 0, <= 8192. */
TF_API int tf_b200_rmsnorm_bf16(const void* x, const void* residual, const void* weight, void* y,
                                void* h_out, int rows, int cols, float eps, void* stream);
/* SwiGLU; replaces swiglu_forward (src/kernels/swiglu.rs:56-95):
 *   z [rows, 2*d_ff] = [gate || up] bf16 -> out[m, n] = silu(gate[m, n]) * up[m, n], [rows, d_ff]. */
TF_API int tf_b200_swiglu_bf16(const void* z, void* out, int rows, int d_ff, void* stream);

/* ---------------- GEMMs of the Llama block with fused epilogues (tcgen05) ----------------
 * C = A * B^T with bf16 operands and fp32 accumulation; B is an nn.Linear-style weight
 * [n, k] (row-major).  These replace the teeny-core Linear calls of the attention layer
 * and the FFN (src/layers/attention.rs:83-148, src/layers/ffn.rs:47-56), fused with the
 * kernel that follows each one in src/layers/llama_block.rs:55-65.  Shape rules:
 * k >= 1, k % 8 == 0, n % 8 == 0, 16-byte aligned pointers; m == 0 or n == 0 is a no-op.
 *
 * A operand: row-major [m, k], or, with a_seq > 0, the attention output
 * [m / a_seq, k / 128, a_seq, 128] read as the [m, k] matrix MergeHeads would build
 * (transpose_heads.rs:86-95 folded into the GEMM's loads; a_seq % 128 == 0).
 * residual: NULL, or a bf16 [m, n] added to the rounded product (c = bf16(a b^T) + residual,
 * the layer's final residual add; c may alias residual). */
TF_API int tf_b200_gemm_bf16(const void* a, const void* b, const void* residual, void* c, int m,
                             int n, int k, int a_seq, void* stream);
/* FFN gate/up projection + SwiGLU (swiglu.rs:56-95): w_gate_up is [2*d_ff, k] with gate and
 * up rows interleaved in 128-row blocks (block 2j = gate rows 128j.., block 2j+1 = up rows
 * 128j..); out [m, d_ff] = silu(a w_gate^T) * (a w_up^T).  d_ff % 128 == 0. */
TF_API int tf_b200_gemm_swiglu_bf16(const void* a, const void* w_gate_up, void* out, int m,
                                    int d_ff, int k, void* stream);
/* (cos, sin) table [seq_len, head_dim / 2] of float pairs for the QKV epilogue, with the
 * angles of tf_b200_rope_bf16 (rope.rs:86-93). */
TF_API int tf_b200_rope_table_f32(void* cs, int seq_len, int head_dim, float ln_rope_base,
                                  void* stream);
/* QKV projection + TransposeHeads + RoPE (attention.rs:89-123) in one kernel:
 * x [batch * seq_len, d_model], w_qkv = [Wq; Wk; Wv] [(n_heads_q + 2 n_heads_kv) * 128, d_model];
 * q [batch, n_heads_q, seq_len, 128], k_out / v [batch, n_heads_kv, seq_len, 128].  Q and K are
 * rotated with rope_cs (tf_b200_rope_table_f32; NULL = no rotation), style 0 = interleaved pairs,
 * 1 = rotate-half.  head_dim is 128; seq_len % 128 == 0. */
TF_API int tf_b200_gemm_qkv_rope_bf16(const void* x, const void* w_qkv, void* q, void* k_out,
                                      void* v, const void* rope_cs, int batch, int seq_len,
                                      int n_heads_q, int n_heads_kv, int d_model, int rope_style,
                                      void* stream);
/* Tensor-parallel o_proj / down_proj fused with the reduce-scatter half of the all-reduce
 * that follows it (llama_block.rs:55-65 split over `world` ranks): the partial product's rows
 * [o * m / world, (o + 1) * m / world) are stored straight into rank o's receive buffer
 * peer_recv[o] (a host array of `world` device pointers, each [world, m / world, n]) at slot
 * [rank], with NVLink peer stores as tiles finish.  The caller then runs
 * tf_b200_allreduce_residual_rmsnorm_bf16 with peer_src[p] = its own receive buffer + (p - rank)
 * * (m / world) * n elements (so global row r of slot p is at peer_src[p] + r * n), which sums
 * local memory only.
 * (m / world) % 128 == 0; world <= 8. */
TF_API int tf_b200_gemm_push_bf16(const void* a, const void* b, void* const* peer_recv, int m,
                                  int n, int k, int a_seq, int rank, int world, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TEENYFORMERS_B200_H */
