"""Host-side mirror of teenyformers' attention-path custom ops, over the C ABI.

The reference defines each op as a CustomOp (graph node: name, output-shape
inference) plus a RuntimeOp (activation-input count, param-cache shapes,
forward and backward launch).  The classes here keep those names, argument
meanings and shape rules and launch the sm_100a kernels through
``include/teenyformers_b200.h``; tensors are torch CUDA tensors (torch is the
device-memory / stream plumbing only):

  FlashAttn2Op        src/kernels/flash_attn2.rs:393-429 (non-causal)
  CausalFlashAttn2Op  src/kernels/flash_attn2.rs:539-575
  RopeOp              src/kernels/rope.rs:246-281
  TransposeHeadsOp    src/kernels/transpose_heads.rs:168-203
  MergeHeadsOp        src/kernels/transpose_heads.rs:276-312

Errors: the reference asserts on bad shapes (src/layers/attention.rs:68);
here a bad call raises ValueError (shape) or TfError (status from the C ABI).
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _capi
from ._capi import TF_ROPE_INTERLEAVED, TF_ROPE_ROTATE_HALF, TfError, call

__all__ = [
    "FlashAttn2Op", "CausalFlashAttn2Op", "RopeOp", "TransposeHeadsOp", "MergeHeadsOp",
    "flash_attn2_fwd", "flash_attn2_bwd", "rope", "rope_transpose", "transpose_heads",
    "merge_heads", "bwd_workspace", "rmsnorm", "swiglu", "flash_attn2_decode",
    "decode_workspace", "linear", "linear_swiglu", "swiglu_weight_blocks", "rope_table",
    "linear_qkv_rope", "linear_push", "TF_ROPE_INTERLEAVED",
    "TF_ROPE_ROTATE_HALF", "TfError",
]


def _ptr(t: torch.Tensor | None):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _need(cond: bool, msg: str):
    if not cond:
        raise ValueError(msg)


def _as4(x: torch.Tensor) -> torch.Tensor:
    """[BH, S, D] (reference layout) -> [1, BH, S, D]; [B, H, S, D] unchanged."""
    _need(x.dim() in (3, 4), f"expected [BH,S,D] or [B,H,S,D], got {tuple(x.shape)}")
    return x.unsqueeze(0) if x.dim() == 3 else x


# ----------------------------------------------------------------- functional API
def flash_attn2_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, softmax_scale: float,
                    causal: bool, out: torch.Tensor | None = None,
                    lse: torch.Tensor | None = None):
    """O, LSE of flash attention.  q [B,Hq,Sq,D] / k,v [B,Hkv,Sk,D] (or 3-D
    [BH,S,D]); bf16 -> tcgen05 kernel, fp32 -> reference-ABI fp32 kernel."""
    q4, k4, v4 = _as4(q), _as4(k), _as4(v)
    B, Hq, Sq, D = q4.shape
    Hkv, Sk = k4.shape[1], k4.shape[2]
    _need(k4.shape == v4.shape and k4.shape[0] == B and k4.shape[3] == D, "k/v shape mismatch")
    for t in (q, k, v):
        _need(t.is_cuda and t.is_contiguous(), "inputs must be contiguous CUDA tensors")
        _need(t.dtype == q.dtype, "q, k, v dtypes differ")
    o = torch.empty_like(q) if out is None else out
    l = torch.empty(q.shape[:-1], dtype=torch.float32, device=q.device) if lse is None else lse
    if q.dtype == torch.bfloat16:
        call("tf_b200_flash_attn2_fwd_bf16", _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(l), B, Hq,
             Hkv, Sq, Sk, D, float(softmax_scale), int(bool(causal)), _stream(q))
    elif q.dtype == torch.float32:
        _need(Hq == Hkv, "the fp32 reference-ABI kernels are MHA only")
        call("tf_b200_flash_attn2_fwd_f32", _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(l), B * Hq,
             D, Sq, Sk, float(softmax_scale), float("-inf"), int(bool(causal)), _stream(q))
    else:
        raise ValueError(f"unsupported dtype {q.dtype}")
    return o, l


def bwd_workspace(q: torch.Tensor) -> torch.Tensor:
    q4 = _as4(q)
    B, Hq, Sq, _ = q4.shape
    n = _capi.raw("tf_b200_flash_attn2_bwd_workspace_size", B, Hq, Sq)
    return torch.empty(max(int(n), 16), dtype=torch.uint8, device=q.device)


def flash_attn2_bwd(q, k, v, o, lse, do, softmax_scale: float, causal: bool,
                    workspace: torch.Tensor | None = None, grads=None):
    """(dQ, dK, dV) of flash attention; same layouts as the forward."""
    q4, k4 = _as4(q), _as4(k)
    B, Hq, Sq, D = q4.shape
    Hkv, Sk = k4.shape[1], k4.shape[2]
    for t in (q, k, v, o, do, lse):
        _need(t.is_cuda and t.is_contiguous(), "inputs must be contiguous CUDA tensors")
    if grads is None:
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    else:
        dq, dk, dv = grads
    if q.dtype == torch.bfloat16:
        ws = bwd_workspace(q) if workspace is None else workspace
        call("tf_b200_flash_attn2_bwd_bf16", _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(do),
             _ptr(lse), _ptr(dq), _ptr(dk), _ptr(dv), _ptr(ws), B, Hq, Hkv, Sq, Sk, D,
             float(softmax_scale), int(bool(causal)), _stream(q))
    elif q.dtype == torch.float32:
        _need(Hq == Hkv, "the fp32 reference-ABI kernels are MHA only")
        call("tf_b200_flash_attn2_bwd_f32", _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(do),
             _ptr(lse), _ptr(dq), _ptr(dk), _ptr(dv), B * Hq, D, Sq, Sk, float(softmax_scale),
             int(bool(causal)), _stream(q))
    else:
        raise ValueError(f"unsupported dtype {q.dtype}")
    return dq, dk, dv


def decode_workspace(q: torch.Tensor, n_heads_kv: int, cache_capacity: int) -> torch.Tensor | None:
    B, Hq, n_q, D = q.shape
    n = _capi.raw("tf_b200_flash_attn2_decode_workspace_size", B, Hq, n_heads_kv, n_q,
                  cache_capacity, D)
    return torch.empty(int(n), dtype=torch.uint8, device=q.device) if n else None


def flash_attn2_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                       cache_seqlens: torch.Tensor, softmax_scale: float,
                       out: torch.Tensor | None = None, lse: torch.Tensor | None = None,
                       workspace: torch.Tensor | None = None):
    """KV-cache decode: q [B,Hq,n_q,D], caches [B,Hkv,cap,D], cache_seqlens [B] int32 (device);
    the last n_q cached keys are the new tokens'.  Returns (o, lse)."""
    for t in (q, k_cache, v_cache):
        _need(t.is_cuda and t.is_contiguous() and t.dtype == torch.bfloat16 and t.dim() == 4,
              "q and the caches must be contiguous 4-D bf16 CUDA tensors")
    _need(cache_seqlens.is_cuda and cache_seqlens.dtype == torch.int32 and
          cache_seqlens.is_contiguous(), "cache_seqlens must be a contiguous int32 CUDA tensor")
    B, Hq, n_q, D = q.shape
    _, Hkv, cap, Dk = k_cache.shape
    _need(k_cache.shape == v_cache.shape and k_cache.shape[0] == B and Dk == D,
          "cache shape mismatch")
    _need(cache_seqlens.numel() == B, "cache_seqlens must have one entry per sequence")
    o = torch.empty_like(q) if out is None else out
    l = torch.empty((B, Hq, n_q), dtype=torch.float32, device=q.device) if lse is None else lse
    ws = decode_workspace(q, Hkv, cap) if workspace is None else workspace
    call("tf_b200_flash_attn2_decode_bf16", _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(o),
         _ptr(l), _ptr(cache_seqlens), B, Hq, Hkv, n_q, cap, D, float(softmax_scale), _ptr(ws),
         _stream(q))
    return o, l


def rope(x: torch.Tensor, rope_base: float, style: int = TF_ROPE_INTERLEAVED,
         inverse: bool = False, out: torch.Tensor | None = None) -> torch.Tensor:
    """RoPE on [..., S, D] rows (pos = index along S); reference rope.rs:57-140."""
    _need(x.is_cuda and x.is_contiguous() and x.dim() >= 2, "x must be a contiguous CUDA tensor")
    S, D = x.shape[-2], x.shape[-1]
    bh = x.numel() // max(S * D, 1)
    y = torch.empty_like(x) if out is None else out
    fn = {torch.float32: "tf_b200_rope_f32", torch.bfloat16: "tf_b200_rope_bf16"}.get(x.dtype)
    _need(fn is not None, f"unsupported dtype {x.dtype}")
    call(fn, _ptr(x), _ptr(y), bh, S, D, float(math.log(rope_base)), int(style),
         int(bool(inverse)), _stream(x))
    return y


def rope_transpose(x: torch.Tensor, rope_base: float, style: int = TF_ROPE_INTERLEAVED,
                   inverse: bool = False, out: torch.Tensor | None = None) -> torch.Tensor:
    """Fused [B,S,H,D] -> RoPE -> [B,H,S,D]; inverse: [B,H,S,D] -> RoPE^-1 -> [B,S,H,D]."""
    _need(x.is_cuda and x.is_contiguous() and x.dim() == 4 and x.dtype == torch.bfloat16,
          "x must be a contiguous 4-D bf16 CUDA tensor")
    if not inverse:
        B, S, H, D = x.shape
        shape = (B, H, S, D)
    else:
        B, H, S, D = x.shape
        shape = (B, S, H, D)
    y = torch.empty(shape, dtype=x.dtype, device=x.device) if out is None else out
    call("tf_b200_rope_transpose_bf16", _ptr(x), _ptr(y), B, S, H, D,
         float(math.log(rope_base)), int(style), int(bool(inverse)), _stream(x))
    return y


def transpose_heads(x: torch.Tensor, n_heads: int) -> torch.Tensor:
    """[B?, S, H*D] -> [B?, H, S, D], bit-exact (transpose_heads.rs:49-71)."""
    _need(x.is_cuda and x.is_contiguous() and x.dim() in (2, 3), "x must be [S,D] or [B,S,D]")
    x3 = x.unsqueeze(0) if x.dim() == 2 else x
    B, S, DM = x3.shape
    _need(DM % n_heads == 0, "d_model must be divisible by n_heads")
    D = DM // n_heads
    y = torch.empty((B, n_heads, S, D), dtype=x.dtype, device=x.device)
    call("tf_b200_transpose_heads", _ptr(x), _ptr(y), B, S, n_heads, D, x.element_size(),
         _stream(x))
    return y[0] if x.dim() == 2 else y


def merge_heads(x: torch.Tensor) -> torch.Tensor:
    """[B?, H, S, D] -> [B?, S, H*D], bit-exact (transpose_heads.rs:76-96)."""
    _need(x.is_cuda and x.is_contiguous() and x.dim() in (3, 4), "x must be [H,S,D] or [B,H,S,D]")
    x4 = x.unsqueeze(0) if x.dim() == 3 else x
    B, H, S, D = x4.shape
    y = torch.empty((B, S, H * D), dtype=x.dtype, device=x.device)
    call("tf_b200_merge_heads", _ptr(x), _ptr(y), B, S, H, D, x.element_size(), _stream(x))
    return y[0] if x.dim() == 3 else y


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float,
            residual: torch.Tensor | None = None, out: torch.Tensor | None = None,
            residual_out: torch.Tensor | None = None):
    """y = h * rsqrt(mean(h^2) + eps) * weight with h = x (+ residual) over the
    last dim (fused_add_rmsnorm.rs:53-110).  With ``residual`` returns (y, h)."""
    for t in (x, weight) + ((residual,) if residual is not None else ()):
        _need(t.is_cuda and t.is_contiguous() and t.dtype == torch.bfloat16,
              "rmsnorm tensors must be contiguous bf16 CUDA tensors")
    N = x.shape[-1]
    _need(weight.numel() == N, "weight must have the last dim's size")
    rows = x.numel() // max(N, 1)
    y = torch.empty_like(x) if out is None else out
    h = None
    if residual is not None:
        _need(residual.shape == x.shape, "residual shape mismatch")
        h = torch.empty_like(x) if residual_out is None else residual_out
    call("tf_b200_rmsnorm_bf16", _ptr(x), _ptr(residual), _ptr(weight), _ptr(y), _ptr(h), rows,
         N, float(eps), _stream(x))
    return (y, h) if residual is not None else y


def swiglu(z: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """[..., 2*d_ff] = gate || up -> silu(gate) * up (swiglu.rs:56-95)."""
    _need(z.is_cuda and z.is_contiguous() and z.dtype == torch.bfloat16,
          "z must be a contiguous bf16 CUDA tensor")
    d_ff = z.shape[-1] // 2
    rows = z.numel() // max(2 * d_ff, 1)
    y = torch.empty(z.shape[:-1] + (d_ff,), dtype=z.dtype, device=z.device) if out is None else out
    call("tf_b200_swiglu_bf16", _ptr(z), _ptr(y), rows, d_ff, _stream(z))
    return y


def _bf16(*ts):
    for t in ts:
        _need(t.is_cuda and t.is_contiguous() and t.dtype == torch.bfloat16,
              "GEMM tensors must be contiguous bf16 CUDA tensors")


def linear(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor | None = None,
           heads_seq: int = 0, residual: torch.Tensor | None = None) -> torch.Tensor:
    """x @ weight.T on the tcgen05 GEMM (teeny-core Linear in the block).

    x: [..., k] row-major, or (heads_seq > 0) the attention output
    [B, H, heads_seq, 128], read as the [B * heads_seq, H * 128] matrix that
    merge_heads would build.  weight: [n, k].  Returns [..., n] (or
    [B, heads_seq, n]); with ``residual`` (same shape as the output) returns
    bf16(x @ weight.T) + residual."""
    _bf16(x, weight)
    n, k = weight.shape
    if heads_seq > 0:
        _need(x.dim() == 4 and x.shape[2] == heads_seq and x.shape[1] * x.shape[3] == k,
              "heads-layout x must be [B, H, S, 128] with H * 128 == k")
        lead = (x.shape[0], heads_seq)
        m = x.shape[0] * heads_seq
    else:
        _need(x.shape[-1] == k, "x's last dim must match weight's k")
        lead = tuple(x.shape[:-1])
        m = x.numel() // max(k, 1)
    y = torch.empty(lead + (n,), dtype=x.dtype, device=x.device) if out is None else out
    _bf16(y)
    _need(y.numel() == m * n, "out has the wrong size")
    if residual is not None:
        _bf16(residual)
        _need(residual.numel() == m * n, "residual has the wrong size")
    call("tf_b200_gemm_bf16", _ptr(x), _ptr(weight), _ptr(residual), _ptr(y), m, n, k,
         int(heads_seq), _stream(x))
    return y


def swiglu_weight_blocks(w_gate: torch.Tensor, w_up: torch.Tensor) -> torch.Tensor:
    """[d_ff, k] gate and up weights -> the [2 d_ff, k] block-interleaved weight
    linear_swiglu reads (128-row blocks: gate 0, up 0, gate 1, up 1, ...)."""
    d_ff, k = w_gate.shape
    _need(w_up.shape == w_gate.shape and d_ff % 128 == 0, "gate/up must be [d_ff, k], d_ff % 128 == 0")
    return torch.stack([w_gate.reshape(d_ff // 128, 128, k), w_up.reshape(d_ff // 128, 128, k)],
                       dim=1).reshape(2 * d_ff, k).contiguous()


def linear_swiglu(x: torch.Tensor, w_gate_up_blocks: torch.Tensor,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """silu(x @ w_gate.T) * (x @ w_up.T) in one GEMM (ffn.rs:47-56 + swiglu.rs:56-95);
    the weight comes from swiglu_weight_blocks."""
    _bf16(x, w_gate_up_blocks)
    n2, k = w_gate_up_blocks.shape
    d_ff = n2 // 2
    _need(x.shape[-1] == k, "x's last dim must match the weight's k")
    m = x.numel() // max(k, 1)
    y = torch.empty(tuple(x.shape[:-1]) + (d_ff,), dtype=x.dtype, device=x.device) if out is None else out
    _bf16(y)
    _need(y.numel() == m * d_ff, "out has the wrong size")
    call("tf_b200_gemm_swiglu_bf16", _ptr(x), _ptr(w_gate_up_blocks), _ptr(y), m, d_ff, k,
         _stream(x))
    return y


def rope_table(seq_len: int, head_dim: int, rope_base: float, device) -> torch.Tensor:
    """[seq_len, head_dim / 2, 2] fp32 (cos, sin) table for linear_qkv_rope."""
    t = torch.empty((seq_len, head_dim // 2, 2), dtype=torch.float32, device=device)
    call("tf_b200_rope_table_f32", _ptr(t), seq_len, head_dim, float(math.log(rope_base)),
         ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream))
    return t


def linear_qkv_rope(x: torch.Tensor, w_qkv: torch.Tensor, n_heads_q: int, n_heads_kv: int,
                    table: torch.Tensor | None, style: int = TF_ROPE_INTERLEAVED, outs=None):
    """x [B, S, d] @ [Wq; Wk; Wv].T -> (q [B, Hq, S, 128], k, v [B, Hkv, S, 128]) with RoPE
    on q and k (attention.rs:89-123: projections, TransposeHeads, RoPE) in one kernel."""
    _bf16(x, w_qkv)
    B, S, d = x.shape
    D = 128
    _need(w_qkv.shape == ((n_heads_q + 2 * n_heads_kv) * D, d), "w_qkv shape mismatch")
    if outs is None:
        outs = (torch.empty((B, n_heads_q, S, D), dtype=x.dtype, device=x.device),
                torch.empty((B, n_heads_kv, S, D), dtype=x.dtype, device=x.device),
                torch.empty((B, n_heads_kv, S, D), dtype=x.dtype, device=x.device))
    q, k, v = outs
    _bf16(q, k, v)
    if table is not None:
        _need(table.is_cuda and table.dtype == torch.float32 and table.is_contiguous()
              and table.shape[0] >= S and table.numel() // table.shape[0] == D,
              "table must be a contiguous fp32 [>= S, 64, 2] CUDA tensor")
    call("tf_b200_gemm_qkv_rope_bf16", _ptr(x), _ptr(w_qkv), _ptr(q), _ptr(k), _ptr(v),
         _ptr(table), B, S, n_heads_q, n_heads_kv, d, int(style), _stream(x))
    return q, k, v


def linear_push(x: torch.Tensor, weight: torch.Tensor, peer_recv_ptrs, rank: int, world: int,
                heads_seq: int = 0) -> None:
    """Tensor-parallel partial product x @ weight.T whose row slice o is stored
    into rank o's receive buffer peer_recv_ptrs[o] at slot [rank]
    ([world, m / world, n] each): the reduce-scatter half of the all-reduce that
    follows o_proj / down_proj, fused into the GEMM."""
    _bf16(x, weight)
    n, k = weight.shape
    m = (x.shape[0] * heads_seq) if heads_seq > 0 else x.numel() // max(k, 1)
    arr = (ctypes.c_void_p * world)(*[int(p) for p in peer_recv_ptrs])
    call("tf_b200_gemm_push_bf16", _ptr(x), _ptr(weight), arr, m, n, k, int(heads_seq), rank,
         world, _stream(x))


# ----------------------------------------------------------------- op classes
class FlashAttn2Op:
    """Bidirectional flash attention (reference FlashAttn2Op).

    Primary input q [BH, Nq, D] (or [B, H, Nq, D]); others k, v [BH, Nk, D].
    Output o has q's shape; param cache l [BH, Nq] (the LSE).
    ``n_kv_heads`` (GQA) is an addition: the reference is MHA only.
    """

    causal = False
    name = "flash_attn2"

    def __init__(self, head_dim: int, softmax_scale: float, n_kv_heads: int | None = None):
        self.head_dim = int(head_dim)
        self.softmax_scale = float(softmax_scale)
        self.n_kv_heads = n_kv_heads

    # CustomOp
    def infer_output_shape(self, input_shapes):
        return tuple(input_shapes[0])

    # RuntimeOp
    def n_activation_inputs(self) -> int:
        return 3

    def param_shapes(self, input_shapes, output_shape=None):
        q = tuple(input_shapes[0])
        return [list(q[:-1])]

    def has_backward(self) -> bool:
        return True

    def forward(self, q, k, v):
        _need(q.shape[-1] == self.head_dim, "head_dim mismatch")
        return flash_attn2_fwd(q, k, v, self.softmax_scale, self.causal)

    def backward(self, q, k, v, o, l, grad_output, workspace=None):
        return flash_attn2_bwd(q, k, v, o, l, grad_output, self.softmax_scale, self.causal,
                               workspace=workspace)


class CausalFlashAttn2Op(FlashAttn2Op):
    """Causal (decoder self-attention) flash attention; key k hidden from query q when k > q."""

    causal = True
    name = "causal_flash_attn2"


class RopeOp:
    """Rotary position embedding on [BH, N_CTX, HEAD_DIM] (reference RopeOp).

    ``style`` is an addition (the reference is interleaved only)."""

    name = "rope"

    def __init__(self, head_dim: int, rope_base: float, style: int = TF_ROPE_INTERLEAVED):
        self.head_dim = int(head_dim)
        self.rope_base = float(rope_base)
        self.style = int(style)

    def infer_output_shape(self, input_shapes):
        return tuple(input_shapes[0])

    def n_activation_inputs(self) -> int:
        return 1

    def param_shapes(self, input_shapes, output_shape=None):
        return []

    def has_backward(self) -> bool:
        return True

    def forward(self, x):
        _need(x.shape[-1] == self.head_dim, "head_dim mismatch")
        return rope(x, self.rope_base, self.style, inverse=False)

    def backward(self, grad_output):
        return rope(grad_output, self.rope_base, self.style, inverse=True)


class TransposeHeadsOp:
    """[S, D] -> [H, S, HEAD_DIM] (reference TransposeHeadsOp); backward = merge."""

    name = "transpose_heads"

    def __init__(self, n_heads: int, head_dim: int):
        self.n_heads = int(n_heads)
        self.head_dim = int(head_dim)

    def infer_output_shape(self, input_shapes):
        s = input_shapes[0][-2]
        lead = tuple(input_shapes[0][:-2])
        return lead + (self.n_heads, s, self.head_dim)

    def n_activation_inputs(self) -> int:
        return 1

    def param_shapes(self, input_shapes, output_shape=None):
        return []

    def has_backward(self) -> bool:
        return True

    def forward(self, x):
        return transpose_heads(x, self.n_heads)

    def backward(self, grad_output):
        return merge_heads(grad_output)


class MergeHeadsOp:
    """[H, S, HEAD_DIM] -> [S, D] (reference MergeHeadsOp); backward = transpose."""

    name = "merge_heads"

    def __init__(self, n_heads: int, head_dim: int):
        self.n_heads = int(n_heads)
        self.head_dim = int(head_dim)

    def infer_output_shape(self, input_shapes):
        shp = tuple(input_shapes[0])
        return shp[:-3] + (shp[-2], self.n_heads * self.head_dim)

    def n_activation_inputs(self) -> int:
        return 1

    def param_shapes(self, input_shapes, output_shape=None):
        return []

    def has_backward(self) -> bool:
        return True

    def forward(self, x):
        return merge_heads(x)

    def backward(self, grad_output):
        return transpose_heads(grad_output, self.n_heads)
