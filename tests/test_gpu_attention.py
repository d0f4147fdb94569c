"""tcgen05 attention kernels vs the CPU oracles.

Tolerances (north-star parity targets): BF16 path cosine >= 0.9999 against
fp32 SDPA with max-abs error <= 2e-2 (inputs N(0,1), outputs O(1)); Sage-FP8
path cosine >= 0.999 against the quantised restatement."""
import math

import numpy as np
import pytest
import torch

from oracle import attention as oa

pytestmark = pytest.mark.gpu


def make_qkv(b, h, s, seed=0, k_bias=2.0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, h, s, 128, generator=g)
    k = torch.randn(b, h, s, 128, generator=g) + k_bias * torch.randn(1, h, 1, 128, generator=g)
    v = torch.randn(b, h, s, 128, generator=g)
    return q.bfloat16(), k.bfloat16(), v.bfloat16()


def to_np(t):
    return t.float().cpu().numpy()


def test_sage_prepare_vs_oracle(cuda_device):
    from xgen_b200.attention import sage_prepare

    q, k, v = make_qkv(1, 2, 300)
    ws = sage_prepare(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device))
    ref = oa.sage_quantize(to_np(q), to_np(k), to_np(v))
    s = 300
    nb = (s + 63) // 64
    np.testing.assert_allclose(ws.q_scale.cpu().numpy()[:, :nb], ref["q_scale"].reshape(2, nb), rtol=1e-6)
    np.testing.assert_allclose(ws.k_scale.cpu().numpy()[:, :nb], ref["k_scale"].reshape(2, nb), rtol=1e-5)
    np.testing.assert_array_equal(ws.v_scale.cpu().numpy(), ref["v_scale"].reshape(2, 128))
    q8 = ws.q8.cpu().numpy()[:, :s].reshape(1, 2, s, 128)
    np.testing.assert_array_equal(q8, ref["q8"])
    k8 = ws.k8.cpu().numpy()[:, :s].reshape(1, 2, s, 128).astype(np.int32)
    dk = np.abs(k8 - ref["k8"].astype(np.int32))
    assert dk.max() <= 1 and (dk > 0).mean() < 1e-3  # fp32 mean summation order
    v8 = ws.v8.cpu().numpy()[:, :s].reshape(1, 2, s, 128)
    np.testing.assert_array_equal(v8, ref["v8"])
    # padding rows are zero
    assert not ws.q8[:, s:].any() and not ws.k8[:, s:].any() and not ws.v8[:, s:].any()


@pytest.mark.parametrize("b,h,s,rotary,transposed", [(1, 2, 300, 96, False), (2, 3, 1000, 128, True),
                                                     (1, 1, 4097, 64, False)])
def test_sage_prepare_with_rope_equals_rope_then_prepare(cuda_device, b, h, s, rotary, transposed):
    """xgb_sage_prepare_rope (RoPE applied as Q/K are read) gives the same
    bytes as the RoPE kernel followed by xgb_sage_prepare, and the RoPE'd
    values equal the oracle's restatement of h3_partial_rope.py:9-29."""
    from oracle import elementwise as ew
    from xgen_b200.attention import SageWorkspace, sage_prepare
    from xgen_b200.h3.rope import rope_partial
    from xgen_b200.ops import try_h3_partial_rope

    q, k, v = make_qkv(b, h, s, seed=3)
    cos, sin = rope_partial(s, rotary)
    dev = cuda_device
    if transposed:  # [B, S, H, D] storage seen as [B, H, S, D] views, as sp_self_attention passes
        q, k, v = (t.transpose(1, 2).contiguous().to(dev).transpose(1, 2) for t in (q, k, v))
    else:
        q, k, v = (t.to(dev) for t in (q, k, v))
    cs = (cos.to(dev), sin.to(dev))
    fused = sage_prepare(q, k, v, ws=SageWorkspace(b, h, s, dev), rotary_emb=cs)
    with torch.no_grad():  # the try_* ops decline under autograd, as the reference's do
        q4, k4 = try_h3_partial_rope(q.transpose(1, 2).contiguous(), k.transpose(1, 2).contiguous(), *cs)
    qr, kr = q4.transpose(1, 2), k4.transpose(1, 2)
    plain = sage_prepare(qr, kr, v, ws=SageWorkspace(b, h, s, dev))
    for name in ("q8", "k8", "v8", "q_scale", "k_scale", "v_scale"):
        assert torch.equal(getattr(fused, name), getattr(plain, name)), name
    eq, ek = ew.partial_rope(to_np(q.transpose(1, 2)), to_np(k.transpose(1, 2)), cos.numpy(), sin.numpy())
    np.testing.assert_array_equal(to_np(q4), eq)
    np.testing.assert_array_equal(to_np(k4), ek)


def test_sage_backend_fuses_rope_at_sp1(cuda_device):
    """sp_self_attention at SP = 1 hands the RoPE to the Sage backend (no
    RoPE kernel of its own): same output as RoPE first, then attention."""
    from xgen_b200.attention import H3AttentionBackendB200
    from xgen_b200.h3.rope import rope_partial
    from xgen_b200.h3.sp_attention import sp_self_attention
    from xgen_b200.ops import try_h3_partial_rope

    g = torch.Generator().manual_seed(8)
    s, heads = 700, 2
    q, k, v = (torch.randn(1, s, heads * 128, generator=g).bfloat16().to(cuda_device) for _ in range(3))
    cos, sin = (t.to(cuda_device) for t in rope_partial(s, 96))
    backend = H3AttentionBackendB200("sage")
    assert backend.fuses_rope(q)
    with torch.no_grad():
        got = sp_self_attention(q, k, v, (cos, sin), backend=backend, heads=heads)
        q4, k4 = try_h3_partial_rope(q.unflatten(-1, (heads, 128)), k.unflatten(-1, (heads, 128)), cos, sin)
        expect = sp_self_attention(q4.flatten(2), k4.flatten(2), v, None, backend=backend, heads=heads)
    torch.cuda.synchronize()
    assert torch.equal(got, expect)


@pytest.mark.parametrize("b,h,s", [(1, 1, 128), (1, 2, 300), (2, 3, 1000), (1, 1, 4097)])
def test_sage_attention_vs_oracle(cuda_device, b, h, s):
    from xgen_b200.attention import kernel_errors, sage_attention

    q, k, v = make_qkv(b, h, s, seed=s)
    out = sage_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device))
    torch.cuda.synchronize()
    assert kernel_errors() == 0
    got = to_np(out)
    assert np.isfinite(got).all()
    ref = oa.sage_attention(to_np(q), to_np(k), to_np(v))
    assert oa.cosine(got, ref) >= 0.999
    exact = oa.dense_attention(to_np(q), to_np(k), to_np(v))
    assert oa.cosine(got, exact) >= 0.99


@pytest.mark.parametrize("b,h,sq,skv", [(1, 1, 128, 128), (1, 2, 257, 257), (2, 3, 1000, 1000),
                                        (1, 2, 300, 700)])
def test_dense_attention_vs_sdpa(cuda_device, b, h, sq, skv):
    from xgen_b200.attention import dense_attention, kernel_errors

    g = torch.Generator().manual_seed(sq + skv)
    q = torch.randn(b, h, sq, 128, generator=g).bfloat16()
    k = torch.randn(b, h, skv, 128, generator=g).bfloat16()
    v = torch.randn(b, h, skv, 128, generator=g).bfloat16()
    out = dense_attention(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device))
    torch.cuda.synchronize()
    assert kernel_errors() == 0
    got = to_np(out)
    ref = oa.dense_attention(to_np(q), to_np(k), to_np(v))
    assert oa.cosine(got, ref) >= 0.9999
    assert np.abs(got - ref).max() <= 2e-2


def test_dense_attention_phaa_strided_views(cuda_device):
    """q/k/v as views of a PHAA gather buffer [W_S, S, B, cs, D] ->
    (B, cs, W_S*S, D), as test_bf16_cudnn_backend_with_phaa_strides does."""
    from xgen_b200.attention import dense_attention

    ws, s_loc, b, cs = 2, 129, 1, 2
    bufs = [torch.randn(ws, s_loc, b, cs, 128, device=cuda_device).bfloat16() for _ in range(3)]
    views = [x.flatten(0, 1).permute(1, 2, 0, 3).narrow(2, 0, ws * s_loc - 1) for x in bufs]
    out = dense_attention(*views)
    ref = torch.nn.functional.scaled_dot_product_attention(*(t.float() for t in views))
    assert oa.cosine(to_np(out), to_np(ref)) >= 0.9999


def test_backend_contract(cuda_device):
    from xgen_b200.attention import H3AttentionBackendB200

    q, k, v = (t.to(cuda_device) for t in make_qkv(1, 2, 513))
    for precision in ("sage", "bf16"):
        backend = H3AttentionBackendB200(precision)
        out = backend(q, k, v, head_offset=0)
        assert out.shape == q.shape and out.dtype == q.dtype
        assert backend.calls == backend.kernel_calls == 1
        mask = torch.ones(513, 513, dtype=torch.bool, device=cuda_device)
        masked = backend(q, k, v, attn_mask=mask)
        assert backend.calls == 2 and backend.kernel_calls == 1
        assert masked.shape == q.shape


@pytest.mark.parametrize("precision", ["bf16", "sage"])
@pytest.mark.parametrize("h,s", [(1, 20000), (3, 4097), (5, 9001)])
def test_tail_split_matches_unsplit(cuda_device, precision, h, s):
    """The last partial wave's items split along the key range (merged by the
    last part to finish) give the unsplit result up to fp32 summation order
    (BF16) or to the e4m3 rounding of P, which each part takes against its own
    running max (Sage, the Sage parity bar); the workspace stays reusable
    (counters reset) and the result deterministic across launches. The
    small-shape oracle tests above run split (fewer items than SMs)."""
    from xgen_b200 import attention as A
    from xgen_b200._lib import call, i64_array

    g = torch.Generator().manual_seed(h * s)
    q, k, v = (torch.randn(1, h, s, 128, generator=g).bfloat16().to(cuda_device) for _ in range(3))
    ws = A.SageWorkspace(1, h, s, cuda_device) if precision == "sage" else None
    if ws is not None:
        A.sage_prepare(q, k, v, ws=ws)

    def run(split: bool):
        out = torch.empty_like(q)
        wsp, wsb = A._ws_args(cuda_device) if split else (None, 0)
        if precision == "sage":
            call("xgb_attention_sage", ws.q8.data_ptr(), ws.q_scale.data_ptr(), ws.k8.data_ptr(),
                 ws.k_scale.data_ptr(), ws.v8.data_ptr(), ws.v_scale.data_ptr(), 1, h, s,
                 out.data_ptr(), i64_array(out.stride()), wsp, wsb,
                 A._err_flag(cuda_device).data_ptr(), A._stream(out))
        else:
            call("xgb_attention_bf16", q.data_ptr(), i64_array(q.stride()), k.data_ptr(),
                 i64_array(k.stride()), v.data_ptr(), i64_array(v.stride()), 1, h, s, s,
                 128 ** -0.5, out.data_ptr(), i64_array(out.stride()), wsp, wsb,
                 A._err_flag(cuda_device).data_ptr(), A._stream(out))
        return out

    whole = run(False)
    parts = [run(True) for _ in range(3)]
    torch.cuda.synchronize()
    assert A.kernel_errors() == 0
    a = whole.float().cpu().numpy()
    tol = (0.99999, 1e-2) if precision == "bf16" else (0.999, 5e-2)
    for p in parts:
        b = p.float().cpu().numpy()
        assert oa.cosine(a, b) >= tol[0]
        assert np.abs(a - b).max() <= tol[1]
    assert torch.equal(parts[0], parts[1]) and torch.equal(parts[1], parts[2])


@pytest.mark.parametrize("peers,seq,batch,heads,valid,padding",
                         [(2, 150, 1, 3, 297, 0), (4, 64, 2, 2, 256, 12), (8, 1000, 1, 3, 7990, 4)])
def test_sage_prepare_from_wire_equals_decode(cuda_device, peers, seq, batch, heads, valid, padding):
    """xgb_sage_prepare_wire on a PHAA FP8 wire gives the same Sage operands
    as decoding the wire to bf16 and preparing from [batch, heads, valid,
    128] views: every code and scale equal."""
    from xgen_b200.attention import sage_prepare, sage_prepare_wire
    from xgen_b200.phaa import fp8_transport as fp8

    g = torch.Generator(device=cuda_device).manual_seed(seq + heads)
    shape = (peers, seq, batch, heads, 128)
    q, k, v = (torch.randn(shape, device=cuda_device, generator=g).bfloat16() for _ in range(3))
    k = (k.float() + 2.0).bfloat16()
    wire = fp8.encode([q, k, v], 128, peers, peer_padding=padding)
    outs = [torch.empty(shape, device=cuda_device, dtype=torch.bfloat16) for _ in range(3)]
    fp8.decode(wire, outs, 128, peers, peer_padding=padding)
    views = [x.permute(2, 3, 0, 1, 4).flatten(2, 3)[:, :, :valid] for x in outs]
    a = sage_prepare(*views)
    b = sage_prepare_wire(wire, peers=peers, seq=seq, batch=batch, heads=heads, valid_seq=valid,
                          peer_padding=padding)
    for name in ("q8", "q_scale", "k8", "k_scale", "v8", "v_scale"):
        assert torch.equal(getattr(a, name), getattr(b, name)), name
