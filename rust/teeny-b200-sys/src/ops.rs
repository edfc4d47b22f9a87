//! The reference's attention-path ops, launched through this library.
//!
//! Each type keeps the constructor and shape rules of its reference op
//! (`FlashAttn2Op` / `CausalFlashAttn2Op`, src/kernels/flash_attn2.rs:393-429 and
//! :539-575; `RopeOp`, src/kernels/rope.rs:246-281; `TransposeHeadsOp` /
//! `MergeHeadsOp`, src/kernels/transpose_heads.rs:168-203 and :276-312).  Where
//! the reference's `RuntimeOp` packs arguments for a generated PTX
//! `entry_point`, these take the device pointers the executor already owns and
//! a stream.  Tensors are in the reference's `[BH, S, D]` layout (batch 1 with
//! BH heads for the attention entry points) and hold bf16 bits.

use core::ffi::c_void;

use crate::{check, ffi};

/// A device pointer handed over by the executor.
pub type DevPtr = *mut c_void;
/// A `cudaStream_t`; null is the legacy default stream.
pub type Stream = *mut c_void;

fn i32_of(v: usize, what: &str) -> anyhow::Result<i32> {
    i32::try_from(v).map_err(|_| anyhow::anyhow!("{what} = {v} exceeds the 32-bit C ABI"))
}

/// Flash attention over `[BH, N, head_dim]`: causal (top-left mask) or not.
#[derive(Clone, Copy, Debug)]
pub struct FlashAttn2Op {
    pub head_dim: usize,
    pub softmax_scale: f32,
    pub causal: bool,
}

impl FlashAttn2Op {
    /// The reference's non-causal op (`FlashAttn2Op::new`).
    pub fn new(head_dim: usize, softmax_scale: f32) -> Self {
        Self { head_dim, softmax_scale, causal: false }
    }

    /// The reference's causal op (`CausalFlashAttn2Op::new`).
    pub fn causal(head_dim: usize, softmax_scale: f32) -> Self {
        Self { head_dim, softmax_scale, causal: true }
    }

    /// Output shape = Q's shape (flash_attn2.rs:411-413).
    pub fn infer_output_shape(&self, q_shape: &[usize]) -> Vec<usize> {
        q_shape.to_vec()
    }

    /// The logsumexp cache `l [BH, Nq]` the forward fills and the backward reads
    /// (flash_attn2.rs:298-307).
    pub fn param_shapes(&self, q_shape: &[usize]) -> Vec<Vec<usize>> {
        vec![vec![q_shape[0], q_shape[1]]]
    }

    /// Bytes of scratch the backward needs beside the op's own buffers.
    pub fn backward_workspace_bytes(&self, bh: usize, n_ctx_q: usize) -> anyhow::Result<usize> {
        // SAFETY: no pointers are involved.
        Ok(unsafe {
            ffi::tf_b200_flash_attn2_bwd_workspace_size(1, i32_of(bh, "bh")?,
                                                        i32_of(n_ctx_q, "n_ctx_q")?)
        })
    }

    /// O and l from Q [BH, Nq, D] and K, V [BH, Nk, D].
    ///
    /// # Safety
    /// Every pointer must address a device buffer of the stated shape that stays
    /// valid until the work queued on `stream` completes.
    #[allow(clippy::too_many_arguments)]
    pub unsafe fn forward(&self, q: DevPtr, k: DevPtr, v: DevPtr, o: DevPtr, l: *mut f32,
                          bh: usize, n_ctx_q: usize, n_ctx_k: usize,
                          stream: Stream) -> anyhow::Result<()> {
        let bh = i32_of(bh, "bh")?;
        check(unsafe {
            ffi::tf_b200_flash_attn2_fwd_bf16(q, k, v, o, l, 1, bh, bh, i32_of(n_ctx_q, "n_ctx_q")?,
                                              i32_of(n_ctx_k, "n_ctx_k")?,
                                              i32_of(self.head_dim, "head_dim")?,
                                              self.softmax_scale, self.causal as i32, stream)
        })
    }

    /// dQ, dK, dV (argument order of `pack_backward_args`, flash_attn2.rs:507-518).
    /// A null `workspace` selects the entry point that needs no scratch buffer.
    ///
    /// # Safety
    /// As for [`FlashAttn2Op::forward`]; `workspace`, if not null, holds
    /// `backward_workspace_bytes` bytes.
    #[allow(clippy::too_many_arguments)]
    pub unsafe fn backward(&self, q: DevPtr, k: DevPtr, v: DevPtr, o: DevPtr, d_o: DevPtr,
                           l: *const f32, dq: DevPtr, dk: DevPtr, dv: DevPtr, workspace: DevPtr,
                           bh: usize, n_ctx_q: usize, n_ctx_k: usize,
                           stream: Stream) -> anyhow::Result<()> {
        let bh = i32_of(bh, "bh")?;
        let (nq, nk) = (i32_of(n_ctx_q, "n_ctx_q")?, i32_of(n_ctx_k, "n_ctx_k")?);
        let d = i32_of(self.head_dim, "head_dim")?;
        let causal = self.causal as i32;
        check(unsafe {
            if workspace.is_null() {
                ffi::tf_b200_flash_attn2_bwd_bf16_noalloc(q, k, v, o, d_o, l, dq, dk, dv, 1, bh,
                                                          bh, nq, nk, d, self.softmax_scale,
                                                          causal, stream)
            } else {
                ffi::tf_b200_flash_attn2_bwd_bf16(q, k, v, o, d_o, l, dq, dk, dv, workspace, 1,
                                                  bh, bh, nq, nk, d, self.softmax_scale, causal,
                                                  stream)
            }
        })
    }
}

/// Rotary position embedding of `[BH, S, head_dim]` rows (position = row index).
#[derive(Clone, Copy, Debug)]
pub struct RopeOp {
    pub head_dim: usize,
    pub rope_base: f32,
    pub style: i32,
}

impl RopeOp {
    /// The reference's op: interleaved pairs (rope.rs:57-140).
    pub fn new(head_dim: usize, rope_base: f32) -> Self {
        Self { head_dim, rope_base, style: crate::ROPE_INTERLEAVED }
    }

    /// Output shape = input shape (rope.rs:264-266).
    pub fn infer_output_shape(&self, x_shape: &[usize]) -> Vec<usize> {
        x_shape.to_vec()
    }

    /// y = RoPE(x) (`inverse` = the backward's inverse rotation).  The library
    /// takes ln(rope_base), as `RopeRtOp::pack_args` passes it (rope.rs:194).
    ///
    /// # Safety
    /// `x` and `y` address `bh * n_ctx * head_dim` bf16 values on the device.
    pub unsafe fn launch(&self, x: DevPtr, y: DevPtr, bh: usize, n_ctx: usize, inverse: bool,
                         stream: Stream) -> anyhow::Result<()> {
        check(unsafe {
            ffi::tf_b200_rope_bf16(x, y, i32_of(bh, "bh")?, i32_of(n_ctx, "n_ctx")?,
                                   i32_of(self.head_dim, "head_dim")?, self.rope_base.ln(),
                                   self.style, inverse as i32, stream)
        })
    }
}

/// `[S, H * head_dim]` -> `[H, S, head_dim]` (and back, `MergeHeadsOp`); a
/// bit-exact copy of elements of `elem_bytes` bytes.
#[derive(Clone, Copy, Debug)]
pub struct TransposeHeadsOp {
    pub n_heads: usize,
    pub head_dim: usize,
}

impl TransposeHeadsOp {
    pub fn new(n_heads: usize, head_dim: usize) -> Self {
        Self { n_heads, head_dim }
    }

    /// `[S, D]` -> `[H, S, D / H]` (transpose_heads.rs:186-190).
    pub fn infer_output_shape(&self, x_shape: &[usize]) -> Vec<usize> {
        vec![self.n_heads, x_shape[0], self.head_dim]
    }

    /// # Safety
    /// `src`/`dst` address `seq_len * n_heads * head_dim` elements on the device.
    pub unsafe fn forward(&self, src: DevPtr, dst: DevPtr, seq_len: usize, elem_bytes: usize,
                          stream: Stream) -> anyhow::Result<()> {
        check(unsafe {
            ffi::tf_b200_transpose_heads(src, dst, 1, i32_of(seq_len, "seq_len")?,
                                         i32_of(self.n_heads, "n_heads")?,
                                         i32_of(self.head_dim, "head_dim")?,
                                         i32_of(elem_bytes, "elem_bytes")?, stream)
        })
    }

    /// The backward of a transpose is the merge (and vice versa).
    ///
    /// # Safety
    /// As for [`TransposeHeadsOp::forward`].
    pub unsafe fn merge(&self, src: DevPtr, dst: DevPtr, seq_len: usize, elem_bytes: usize,
                        stream: Stream) -> anyhow::Result<()> {
        check(unsafe {
            ffi::tf_b200_merge_heads(src, dst, 1, i32_of(seq_len, "seq_len")?,
                                     i32_of(self.n_heads, "n_heads")?,
                                     i32_of(self.head_dim, "head_dim")?,
                                     i32_of(elem_bytes, "elem_bytes")?, stream)
        })
    }
}
