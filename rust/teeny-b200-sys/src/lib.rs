//! teeny-b200-sys -- the thin C-ABI binding through which teenyformers' Rust
//! host code reaches the B200 (sm_100a) attention kernels.
//!
//! [`ffi`] declares every entry point of `include/teenyformers_b200.h`, one to
//! one (same names, argument order and types).  [`ops`] keeps the reference's
//! op constructors (`FlashAttn2Op::new(head_dim, softmax_scale)`,
//! `RopeOp::new(head_dim, rope_base)`, `TransposeHeadsOp::new(n_heads,
//! head_dim)`, src/kernels/{flash_attn2,rope,transpose_heads}.rs) and turns
//! their launches into calls of this library on device pointers the executor
//! owns, with errors as `anyhow::Result` like the reference's host code.
//!
//! Conventions: caller-owned device pointers, a `cudaStream_t` passed as
//! `*mut c_void` (null = legacy default stream), status 0 or a negative
//! [`Status`] code; nothing here allocates device memory.

use core::ffi::{c_char, c_int, c_void};

pub mod ffi {
    use super::*;

    #[link(name = "teenyformers_b200")]
    unsafe extern "C" {
        pub fn tf_b200_version() -> c_int;
        pub fn tf_b200_status_string(status: c_int) -> *const c_char;
        pub fn tf_b200_device_status(clear: c_int) -> c_int;
        pub fn tf_b200_flash_attn2_fwd_bf16(q: *const c_void, k: *const c_void, v: *const c_void,
            o: *mut c_void, lse: *mut f32, batch: c_int, n_heads_q: c_int, n_heads_kv: c_int,
            n_ctx_q: c_int, n_ctx_k: c_int, head_dim: c_int, softmax_scale: f32, causal: c_int,
            stream: *mut c_void) -> c_int;
        pub fn tf_b200_flash_attn2_bwd_workspace_size(batch: c_int, n_heads_q: c_int,
            n_ctx_q: c_int) -> usize;
        pub fn tf_b200_flash_attn2_bwd_bf16(q: *const c_void, k: *const c_void, v: *const c_void,
            o: *const c_void, d_o: *const c_void, lse: *const f32, dq: *mut c_void,
            dk: *mut c_void, dv: *mut c_void, workspace: *mut c_void, batch: c_int,
            n_heads_q: c_int, n_heads_kv: c_int, n_ctx_q: c_int, n_ctx_k: c_int, head_dim: c_int,
            softmax_scale: f32, causal: c_int, stream: *mut c_void) -> c_int;
        pub fn tf_b200_flash_attn2_bwd_bf16_noalloc(q: *const c_void, k: *const c_void,
            v: *const c_void, o: *const c_void, d_o: *const c_void, lse: *const f32,
            dq: *mut c_void, dk: *mut c_void, dv: *mut c_void, batch: c_int, n_heads_q: c_int,
            n_heads_kv: c_int, n_ctx_q: c_int, n_ctx_k: c_int, head_dim: c_int, softmax_scale: f32,
            causal: c_int, stream: *mut c_void) -> c_int;
        pub fn tf_b200_flash_attn2_decode_workspace_size(batch: c_int, n_heads_q: c_int,
            n_heads_kv: c_int, n_q: c_int, cache_capacity: c_int, head_dim: c_int) -> usize;
        pub fn tf_b200_flash_attn2_decode_bf16(q: *const c_void, k_cache: *const c_void,
            v_cache: *const c_void, o: *mut c_void, lse: *mut f32, cache_seqlens: *const c_int,
            batch: c_int, n_heads_q: c_int, n_heads_kv: c_int, n_q: c_int, cache_capacity: c_int,
            head_dim: c_int, softmax_scale: f32, workspace: *mut c_void,
            stream: *mut c_void) -> c_int;
        pub fn tf_b200_allreduce_residual_rmsnorm_bf16(peer_src: *const *const c_void,
            peer_h: *const *mut c_void, peer_signal: *const *mut c_void, residual: *const c_void,
            weight: *const c_void, y: *mut c_void, rank: c_int, world: c_int, rows: c_int,
            cols: c_int, eps: f32, epoch: u32, stream: *mut c_void) -> c_int;
        pub fn tf_b200_flash_attn2_fwd_f32(q: *const f32, k: *const f32, v: *const f32,
            o: *mut f32, l: *mut f32, bh: c_int, head_dim: c_int, n_ctx_q: c_int, n_ctx_k: c_int,
            softmax_scale: f32, neg_inf: f32, causal: c_int, stream: *mut c_void) -> c_int;
        pub fn tf_b200_flash_attn2_bwd_f32(q: *const f32, k: *const f32, v: *const f32,
            o: *const f32, d_o: *const f32, l: *const f32, dq: *mut f32, dk: *mut f32,
            dv: *mut f32, bh: c_int, head_dim: c_int, n_ctx_q: c_int, n_ctx_k: c_int,
            softmax_scale: f32, causal: c_int, stream: *mut c_void) -> c_int;
        pub fn tf_b200_rope_f32(x: *const f32, y: *mut f32, bh: c_int, n_ctx: c_int,
            head_dim: c_int, ln_rope_base: f32, style: c_int, inverse: c_int,
            stream: *mut c_void) -> c_int;
        pub fn tf_b200_rope_bf16(x: *const c_void, y: *mut c_void, bh: c_int, n_ctx: c_int,
            head_dim: c_int, ln_rope_base: f32, style: c_int, inverse: c_int,
            stream: *mut c_void) -> c_int;
        pub fn tf_b200_rope_transpose_bf16(x: *const c_void, y: *mut c_void, batch: c_int,
            seq_len: c_int, n_heads: c_int, head_dim: c_int, ln_rope_base: f32, style: c_int,
            inverse: c_int, stream: *mut c_void) -> c_int;
        pub fn tf_b200_transpose_heads(src: *const c_void, dst: *mut c_void, batch: c_int,
            seq_len: c_int, n_heads: c_int, head_dim: c_int, elem_bytes: c_int,
            stream: *mut c_void) -> c_int;
        pub fn tf_b200_merge_heads(src: *const c_void, dst: *mut c_void, batch: c_int,
            seq_len: c_int, n_heads: c_int, head_dim: c_int, elem_bytes: c_int,
            stream: *mut c_void) -> c_int;
        pub fn tf_b200_rmsnorm_bf16(x: *const c_void, residual: *const c_void,
            weight: *const c_void, y: *mut c_void, h_out: *mut c_void, rows: c_int, cols: c_int,
            eps: f32, stream: *mut c_void) -> c_int;
        pub fn tf_b200_swiglu_bf16(z: *const c_void, out: *mut c_void, rows: c_int, d_ff: c_int,
            stream: *mut c_void) -> c_int;
        pub fn tf_b200_gemm_bf16(a: *const c_void, b: *const c_void, residual: *const c_void,
            c: *mut c_void, m: c_int, n: c_int, k: c_int, a_seq: c_int,
            stream: *mut c_void) -> c_int;
        pub fn tf_b200_gemm_swiglu_bf16(a: *const c_void, w_gate_up: *const c_void,
            out: *mut c_void, m: c_int, d_ff: c_int, k: c_int, stream: *mut c_void) -> c_int;
        pub fn tf_b200_rope_table_f32(cs: *mut c_void, seq_len: c_int, head_dim: c_int,
            ln_rope_base: f32, stream: *mut c_void) -> c_int;
        pub fn tf_b200_gemm_qkv_rope_bf16(x: *const c_void, w_qkv: *const c_void, q: *mut c_void,
            k_out: *mut c_void, v: *mut c_void, rope_cs: *const c_void, batch: c_int,
            seq_len: c_int, n_heads_q: c_int, n_heads_kv: c_int, d_model: c_int, rope_style: c_int,
            stream: *mut c_void) -> c_int;
        pub fn tf_b200_gemm_push_bf16(a: *const c_void, b: *const c_void,
            peer_recv: *const *mut c_void, m: c_int, n: c_int, k: c_int, a_seq: c_int, rank: c_int,
            world: c_int, stream: *mut c_void) -> c_int;
    }
}

/// `tf_status` of the header.
#[repr(i32)]
#[derive(Clone, Copy, Debug, PartialEq, Eq)]
pub enum Status {
    Ok = 0,
    InvalidArg = -1,
    Unsupported = -2,
    Misaligned = -3,
    Cuda = -4,
    TooLarge = -5,
    DeviceTimeout = -6,
}

/// `tf_rope_style` of the header: interleaved pairs (2k, 2k+1) are the
/// reference's RoPE (src/kernels/rope.rs); rotate-half pairs (k, k + D/2).
pub const ROPE_INTERLEAVED: c_int = 0;
pub const ROPE_ROTATE_HALF: c_int = 1;

/// Turns a status code into `anyhow::Result`, with the library's message.
pub fn check(rc: c_int) -> anyhow::Result<()> {
    if rc == 0 {
        return Ok(());
    }
    // SAFETY: tf_b200_status_string returns a static NUL-terminated string.
    let msg = unsafe { std::ffi::CStr::from_ptr(ffi::tf_b200_status_string(rc)) };
    anyhow::bail!("teenyformers_b200: {} ({rc})", msg.to_string_lossy())
}

/// Reads (and optionally clears) the device-side status word: `Ok(())`
/// unless a kernel's bounded wait expired, in which case the outputs of the
/// calls since the last clear must be discarded.
pub fn device_status(clear: bool) -> anyhow::Result<()> {
    // SAFETY: no pointers are involved.
    let code = unsafe { ffi::tf_b200_device_status(clear as c_int) };
    if code != 0 {
        anyhow::bail!("teenyformers_b200: device wait timed out at site {code}");
    }
    Ok(())
}

pub mod ops;
