"""GPU parity for the tcgen05 flash-attention kernels, through the C ABI.

Oracle: oracle/oracle.c restating src/kernels/flash_attn2.rs (fp32, on the
same bf16-rounded inputs).  Tolerance (north_star): max-abs <= 2e-2 and
rel-L2 <= 1e-2 for bf16 O, LSE, dQ, dK, dV; 1e-4 abs for the fp32 kernels.
"""
import glob
import os

import numpy as np
import pytest
import torch

import oracle
import teenyformers_b200 as tfb
from tests.helpers import F32_ABS, assert_bf16_close, seeded_normal, to_np

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_device):
    yield
    assert tfb.device_status(clear=True) == 0


def make_inputs(B, Hq, Hkv, Sq, Sk, D, device, seed=0):
    q = seeded_normal((B, Hq, Sq, D), seed + 1, device=device)
    k = seeded_normal((B, Hkv, Sk, D), seed + 2, device=device)
    v = seeded_normal((B, Hkv, Sk, D), seed + 3, device=device)
    do = seeded_normal((B, Hq, Sq, D), seed + 4, device=device)
    return q, k, v, do


# (B, Hq, Hkv, Sq, Sk, D, causal)
CASES = [
    (1, 2, 2, 256, 256, 128, True),
    (1, 2, 2, 256, 256, 128, False),
    (2, 4, 2, 200, 200, 128, True),     # GQA, ragged tail
    (1, 2, 2, 77, 77, 64, True),        # D=64, single partial tile
    (1, 2, 2, 384, 130, 64, True),      # top-left causal with Sk < Sq
    (1, 3, 1, 130, 300, 128, False),    # cross attention Nq < Nk, GQA 3:1
    (1, 1, 1, 1, 1, 128, True),         # S = 1
    (1, 2, 2, 640, 640, 128, True),     # several query-tile pairs
    (2, 4, 1, 512, 512, 64, False),     # D=64, GQA 4:1, several key tiles per head
    (1, 2, 2, 1000, 1000, 64, True),    # D=64, ragged, several query-tile pairs
    (1, 8, 1, 384, 384, 128, False),    # GQA 8:1 (config #4's ratio): dK/dV over 8 query heads
    (2, 16, 2, 256, 320, 64, False),    # GQA 8:1, D=64, Sq != Sk, KV heads of two batches
]


def _id(c):
    B, Hq, Hkv, Sq, Sk, D, causal = c
    return f"b{B}h{Hq}kv{Hkv}q{Sq}k{Sk}d{D}{'c' if causal else 'n'}"


@pytest.mark.parametrize("case", CASES, ids=_id)
def test_fwd_bwd_vs_oracle(cuda_device, case):
    B, Hq, Hkv, Sq, Sk, D, causal = case
    scale = D ** -0.5
    q, k, v, do = make_inputs(B, Hq, Hkv, Sq, Sk, D, cuda_device)
    op = (tfb.CausalFlashAttn2Op if causal else tfb.FlashAttn2Op)(D, scale)
    o, lse = op.forward(q, k, v)
    dq, dk, dv = op.backward(q, k, v, o, lse, do)
    torch.cuda.synchronize()
    qn, kn, vn, don = to_np(q), to_np(k), to_np(v), to_np(do)
    o_ref, lse_ref = oracle.flash_attn2_fwd(qn, kn, vn, scale, causal)
    assert_bf16_close("O", to_np(o), o_ref)
    assert_bf16_close("LSE", to_np(lse), lse_ref)
    dq_ref, dk_ref, dv_ref = oracle.flash_attn2_bwd(qn, kn, vn, o_ref, don, lse_ref, scale, causal)
    assert_bf16_close("dQ", to_np(dq), dq_ref)
    assert_bf16_close("dK", to_np(dk), dk_ref)
    assert_bf16_close("dV", to_np(dv), dv_ref)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "attn_*.npz"))),
                         ids=lambda p: os.path.basename(p)[:-4])
def test_fp32_kernels_vs_golden(cuda_device, path):
    z = np.load(path)
    if z["q"].shape[1] != z["k"].shape[1]:
        pytest.skip("the fp32 reference-ABI kernels are MHA only, as the reference")
    scale, causal = float(z["scale"]), bool(z["causal"])
    t = {n: torch.from_numpy(z[n]).to(cuda_device) for n in ("q", "k", "v", "do")}
    o, lse = tfb.flash_attn2_fwd(t["q"], t["k"], t["v"], scale, causal)
    assert np.abs(to_np(o) - z["o"]).max() < F32_ABS
    assert np.abs(to_np(lse) - z["lse"]).max() < F32_ABS
    dq, dk, dv = tfb.flash_attn2_bwd(t["q"], t["k"], t["v"], o, lse, t["do"], scale, causal)
    for name, got in (("dq", dq), ("dk", dk), ("dv", dv)):
        assert np.abs(to_np(got) - z[name]).max() < F32_ABS, name


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "attn_*.npz"))),
                         ids=lambda p: os.path.basename(p)[:-4])
def test_bf16_kernels_vs_golden(cuda_device, path):
    z = np.load(path)
    if z["q"].shape[-1] not in (64, 128):
        pytest.skip("bf16 tcgen05 kernels are built for head_dim 64 and 128")
    scale, causal = float(z["scale"]), bool(z["causal"])
    t = {n: torch.from_numpy(z[n]).to(cuda_device).bfloat16() for n in ("q", "k", "v", "do")}
    o, lse = tfb.flash_attn2_fwd(t["q"], t["k"], t["v"], scale, causal)
    dq, dk, dv = tfb.flash_attn2_bwd(t["q"], t["k"], t["v"], o, lse, t["do"], scale, causal)
    got = {"o": o, "lse": lse, "dq": dq, "dk": dk, "dv": dv}
    # north_star criterion: vs the fp32 reference on the same (bf16-rounded) inputs
    qn, kn, vn, don = (to_np(t[n]) for n in ("q", "k", "v", "do"))
    o_ref, lse_ref = oracle.flash_attn2_fwd(qn, kn, vn, scale, causal)
    g_ref = oracle.flash_attn2_bwd(qn, kn, vn, o_ref, don, lse_ref, scale, causal)
    for name, ref in zip(("o", "lse", "dq", "dk", "dv"), (o_ref, lse_ref) + tuple(g_ref)):
        assert_bf16_close(name, to_np(got[name]), ref)
    # and vs the fp64 witness on the unrounded inputs: the gap now also holds
    # the bf16 rounding of the inputs themselves (relative 2^-9 per element)
    for name in ("o", "lse", "dq", "dk", "dv"):
        assert_bf16_close(name + " (fp64 witness)", to_np(got[name]), z[name], max_abs=6e-2,
                          rl2=1e-2)


def test_config3_full_size_sampled_parity_and_properties(cuda_device):
    """BASELINE config #3 (B=8, H=32, S=4096, D=128, causal): full-size run,
    one (b, h) slice checked against the oracle, and size-independent
    properties checked on every head:
      sum_k dV[k] == sum_q dO[q]   (rows of P sum to 1)
      sum_k dK[k] == 0             (rows of dS sum to 0)"""
    B, H, S, D = 8, 32, 4096, 128
    scale = D ** -0.5
    g = torch.Generator(device=cuda_device).manual_seed(42)
    q, k, v, do = (torch.randn((B, H, S, D), generator=g, device=cuda_device,
                               dtype=torch.bfloat16) for _ in range(4))
    o, lse = tfb.flash_attn2_fwd(q, k, v, scale, True)
    dq, dk, dv = tfb.flash_attn2_bwd(q, k, v, o, lse, do, scale, True)
    torch.cuda.synchronize()
    sum_dv = dv.float().sum(dim=2)
    sum_do = do.float().sum(dim=2)
    assert (sum_dv - sum_do).abs().max().item() < 0.05 * sum_do.abs().max().item() + 0.5
    assert dk.float().sum(dim=2).abs().max().item() < 1.0
    # one (b, h) slice in each 1/8 of the B*H heads -- the contiguous shard a
    # rank owns at N = 8 is one batch entry here -- including the first and the
    # last head of the whole tensor (shard edges at every N)
    for bsel in range(B):
        hsel = {0: 0, B - 1: H - 1}.get(bsel, (7 * bsel + 3) % H)
        sl = lambda t: to_np(t[bsel:bsel + 1, hsel:hsel + 1])
        o_ref, lse_ref = oracle.flash_attn2_fwd(sl(q), sl(k), sl(v), scale, True)
        tag = f"b{bsel}h{hsel}"
        assert_bf16_close("O " + tag, sl(o), o_ref)
        assert_bf16_close("LSE " + tag, sl(lse), lse_ref)
        dq_ref, dk_ref, dv_ref = oracle.flash_attn2_bwd(sl(q), sl(k), sl(v), o_ref, sl(do),
                                                        lse_ref, scale, True)
        assert_bf16_close("dQ " + tag, sl(dq), dq_ref)
        assert_bf16_close("dK " + tag, sl(dk), dk_ref)
        assert_bf16_close("dV " + tag, sl(dv), dv_ref)


def test_config4_gqa_full_size_sampled_parity_and_properties(cuda_device):
    """BASELINE config #4 (causal GQA forward, B=16, Hq=64, Hkv=8 -- eight query
    heads per KV head -- S=8192, D=128) at full size.  Checked against the
    oracle: one (b, KV group) slice with all eight of its query heads, on the
    first and the last 256 query rows (the oracle's kv = h / (Hq / Hkv)
    mapping is the contract; the reference layer is MHA).  On every head:
      O[b, h, 0] == V[b, h / 8, 0] bit for bit (query 0 sees key 0 only), and
      with V[k, 0] = k / S, O[q, 0] <= q / S (the causal mask)."""
    B, Hq, Hkv, S, D = 16, 64, 8, 8192, 128
    G = Hq // Hkv
    scale = D ** -0.5
    g = torch.Generator(device=cuda_device).manual_seed(4242)
    q = torch.randn((B, Hq, S, D), generator=g, device=cuda_device, dtype=torch.bfloat16)
    k = torch.randn((B, Hkv, S, D), generator=g, device=cuda_device, dtype=torch.bfloat16)
    v = torch.randn((B, Hkv, S, D), generator=g, device=cuda_device, dtype=torch.bfloat16)
    o, lse = tfb.flash_attn2_fwd(q, k, v, scale, True)
    torch.cuda.synchronize()
    kv_of = torch.arange(Hq, device=cuda_device) // G
    assert torch.equal(o[:, :, 0, :], v[:, kv_of, 0, :])
    bsel, gsel = 11, 5
    qs = to_np(q[bsel:bsel + 1, gsel * G:(gsel + 1) * G])
    ks = to_np(k[bsel:bsel + 1, gsel:gsel + 1])
    vs = to_np(v[bsel:bsel + 1, gsel:gsel + 1])
    os_, ls = to_np(o[bsel:bsel + 1, gsel * G:(gsel + 1) * G]), to_np(lse[bsel:bsel + 1, gsel * G:(gsel + 1) * G])
    for lo, hi in ((0, 256), (S - 256, S)):
        o_ref, lse_ref = oracle.flash_attn2_fwd(qs, ks, vs, scale, True, q_range=(lo, hi))
        assert_bf16_close(f"O rows {lo}:{hi}", os_[:, :, lo:hi], o_ref[:, :, lo:hi])
        assert_bf16_close(f"LSE rows {lo}:{hi}", ls[:, :, lo:hi], lse_ref[:, :, lo:hi])
    pos = torch.arange(S, device=cuda_device, dtype=torch.float32) / S
    v[..., 0] = pos.bfloat16()
    o2, _ = tfb.flash_attn2_fwd(q, k, v, scale, True, out=o, lse=lse)
    assert bool((o2[..., 0].float() <= pos.view(1, 1, S) * 1.01 + 1e-3).all())


def test_causal_mask_property_full_size(cuda_device):
    """With V[k, 0] = k / S, causal O[q, 0] is an average of visible key
    positions, so O[q, 0] <= q / S (up to bf16 rounding) for every q."""
    B, H, S, D = 2, 4, 4096, 128
    q = seeded_normal((B, H, S, D), 5, device=cuda_device)
    k = seeded_normal((B, H, S, D), 6, device=cuda_device)
    v = torch.zeros((B, H, S, D), device=cuda_device, dtype=torch.bfloat16)
    pos = torch.arange(S, device=cuda_device, dtype=torch.float32) / S
    v[..., 0] = pos.bfloat16()
    o, _ = tfb.flash_attn2_fwd(q, k, v, D ** -0.5, True)
    bound = pos.view(1, 1, S) * 1.01 + 1e-3
    assert bool((o[..., 0].float() <= bound).all())
    assert float(o[..., 0, 0].float().abs().max()) == 0.0   # query 0 sees key 0 only


def test_repeated_calls_are_deterministic(cuda_device):
    q, k, v, do = make_inputs(1, 4, 4, 512, 512, 128, cuda_device, seed=7)
    o1, l1 = tfb.flash_attn2_fwd(q, k, v, 0.088, True)
    o2, l2 = tfb.flash_attn2_fwd(q, k, v, 0.088, True)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)
    g1 = tfb.flash_attn2_bwd(q, k, v, o1, l1, do, 0.088, True)
    g2 = tfb.flash_attn2_bwd(q, k, v, o1, l1, do, 0.088, True)
    # dK/dV accumulate on chip: bitwise repeatable.  dQ is summed over key
    # tiles by fp32 reduce-adds in L2 (like the reference's atomics, in no
    # fixed order), so repeats agree to fp32 rounding before the bf16 cast.
    assert torch.equal(g1[1], g2[1]) and torch.equal(g1[2], g2[2])
    assert_bf16_close("dq repeat", to_np(g1[0]), to_np(g2[0]), max_abs=1e-2, rl2=1e-3)


def test_noalloc_path_is_bitwise_deterministic(cuda_device):
    import ctypes
    from teenyformers_b200 import _capi
    q, k, v, do = make_inputs(1, 4, 2, 384, 384, 128, cuda_device, seed=9)
    o, lse = tfb.flash_attn2_fwd(q, k, v, 0.088, True)
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    outs = []
    for _ in range(2):
        g = [torch.empty_like(t) for t in (q, k, v)]
        _capi.call("tf_b200_flash_attn2_bwd_bf16_noalloc", p(q), p(k), p(v), p(o), p(do), p(lse),
                   *(p(t) for t in g), 1, 4, 2, 384, 384, 128, 0.088, 1, stream)
        outs.append(g)
    torch.cuda.synchronize()
    for a, b in zip(*outs):
        assert torch.equal(a, b)
