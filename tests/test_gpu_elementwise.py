"""CUDA elementwise/FP8 operators vs the reference's own outputs (golden
fixtures) and vs the CPU oracle on larger seeded inputs — bit-exact unless a
test states otherwise."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import elementwise as ew
from oracle import fp8 as of
from oracle.numerics import bf16_bits_from_f32, f32_from_bf16_bits

pytestmark = pytest.mark.gpu


def dev_bf16(bits: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16)).view(torch.bfloat16).to(dev)


def host_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def test_partial_rope_matches_reference(cuda_device):
    from xgen_b200.ops import try_h3_partial_rope

    g = golden("partial_rope")
    with torch.no_grad():
        for i in range(int(g["ncases"])):
            b, s, h, w, r = g[f"c{i}_shape"]
            q = dev_bf16(g[f"c{i}_q"], cuda_device).reshape(b, s, h, w)
            k = dev_bf16(g[f"c{i}_k"], cuda_device).reshape(b, s, h, w)
            cos = torch.from_numpy(g[f"c{i}_cos"]).to(cuda_device)
            sin = torch.from_numpy(g[f"c{i}_sin"]).to(cuda_device)
            qo, ko = try_h3_partial_rope(q, k, cos, sin)
            assert np.array_equal(host_bits(qo).reshape(-1), g[f"c{i}_qo"].reshape(-1)), i
            assert np.array_equal(host_bits(ko).reshape(-1), g[f"c{i}_ko"].reshape(-1)), i


def test_partial_rope_large_vs_oracle(cuda_device):
    from xgen_b200.ops import try_h3_partial_rope

    gen = torch.Generator().manual_seed(5)
    b, s, h, w, r = 1, 257, 24, 128, 96
    q = torch.randn(b, s, h, w, generator=gen).bfloat16()
    k = torch.randn(b, s, h, w, generator=gen).bfloat16()
    theta = torch.arange(s, dtype=torch.float32)[:, None] * torch.rand(1, r, generator=gen)
    cos, sin = torch.cos(theta), torch.sin(theta)
    with torch.no_grad():
        qo, ko = try_h3_partial_rope(q.to(cuda_device), k.to(cuda_device), cos.to(cuda_device),
                                     sin.to(cuda_device))
    eq, ek = ew.partial_rope(q.float().numpy(), k.float().numpy(), cos.numpy(), sin.numpy())
    assert np.array_equal(host_bits(qo), bf16_bits_from_f32(eq))
    assert np.array_equal(host_bits(ko), bf16_bits_from_f32(ek))


def test_partial_rope_rejects_like_reference(cuda_device):
    from xgen_b200.ops import try_h3_partial_rope

    q = torch.randn(1, 4, 2, 128, device=cuda_device).bfloat16()
    cos = torch.randn(4, 96, device=cuda_device)
    with torch.no_grad():
        assert try_h3_partial_rope(q.float(), q.float(), cos, cos) is None  # dtype
        assert try_h3_partial_rope(q, q, cos[:, :95], cos[:, :95]) is None  # odd rotary
        assert try_h3_partial_rope(q.cpu(), q.cpu(), cos.cpu(), cos.cpu()) is None  # not CUDA


def test_qk_rms_matches_reference(cuda_device):
    from xgen_b200.ops import try_h3_qk_rms

    g = golden("qk_rms")
    with torch.no_grad():
        for i in range(int(g["ncases"])):
            b, s, h, w, r = g[f"c{i}_shape"]
            fused = dev_bf16(g[f"c{i}_fused"], cuda_device).reshape(b, s, 3 * h * w)
            q, k, _ = fused.chunk(3, dim=-1)
            q, k = q.unflatten(-1, (h, w)), k.unflatten(-1, (h, w))
            eps = g[f"c{i}_eps"]
            nq, nk = torch.nn.RMSNorm(w, eps=float(eps[0])), torch.nn.RMSNorm(w, eps=float(eps[1]))
            nq.weight.data = dev_bf16(g[f"c{i}_qw"], cuda_device)
            nk.weight.data = dev_bf16(g[f"c{i}_kw"], cuda_device)
            rot = None
            if r:
                rot = (torch.from_numpy(g[f"c{i}_cos"]).to(cuda_device),
                       torch.from_numpy(g[f"c{i}_sin"]).to(cuda_device))
            qo, ko = try_h3_qk_rms(q, k, nq, nk, rot)
            for ours, ref in ((qo, g[f"c{i}_qo"]), (ko, g[f"c{i}_ko"])):
                # one bf16 ulp allowed where the fp32 sum-of-squares order
                # (not part of the algorithm) moves a rounding boundary
                d = np.abs(host_bits(ours).astype(np.int32).reshape(-1) - ref.astype(np.int32).reshape(-1))
                assert d.max() <= 1 and (d > 0).mean() < 2e-3, (i, d.max(), (d > 0).mean())


def test_indexed_affine_matches_reference(cuda_device):
    from xgen_b200.ops import indexed_affine

    g = golden("indexed_affine")
    for i in range(int(g["ncases"])):
        b, s, w, m = g[f"c{i}_shape"]
        x = dev_bf16(g[f"c{i}_x"], cuda_device).reshape(b, s, w)
        res = dev_bf16(g[f"c{i}_residual"], cuda_device).reshape(b, s, w)
        tables = dev_bf16(g[f"c{i}_tables"], cuda_device).reshape(m, 6 * w)
        shift, scale, gate, *_ = tables.chunk(6, dim=-1)
        idx = torch.from_numpy(g[f"c{i}_idx"]).to(cuda_device)
        mod = indexed_affine(x, scale, shift, idx, modulation=True)
        gated = indexed_affine(x, gate, res, idx, modulation=False)
        assert np.array_equal(host_bits(mod).reshape(-1), g[f"c{i}_mod"].reshape(-1)), i
        assert np.array_equal(host_bits(gated).reshape(-1), g[f"c{i}_gate"].reshape(-1)), i
        # and the reference's own eager formula (test_h3_indexed_affine.py:18-21)
        eager = x * (1.0 + scale.index_select(0, idx)) + shift.index_select(0, idx)
        assert torch.equal(mod, eager)


def test_swiglu_matches_reference(cuda_device):
    from xgen_b200.ops import gate_first_swiglu

    g = golden("swiglu")
    for i in range(int(g["ncases"])):
        xb = g[f"c{i}_x"]
        x = dev_bf16(xb, cuda_device).reshape(xb.shape)
        y, amax = gate_first_swiglu(x, with_amax=True)
        d = np.abs(host_bits(y).astype(np.int32).reshape(-1) - g[f"c{i}_y"].astype(np.int32).reshape(-1))
        # CUDA expf vs IEEE exp can move a bf16 rounding boundary by one ulp
        assert d.max() <= 1 and (d > 0).mean() < 1e-2, i
        assert abs(amax.item() - float(g[f"c{i}_amax"][0])) <= 0.01 * float(g[f"c{i}_amax"][0])


def test_fp8_quant_matches_reference(cuda_device):
    from xgen_b200.ops import quantize_activation

    g = golden("fp8_quant")
    for i in range(int(g["ncases"])):
        raw = g[f"c{i}_x"]
        if int(g[f"c{i}_dtype"]) == 0:
            x = dev_bf16(raw, cuda_device).reshape(raw.shape)
        else:
            x = torch.from_numpy(raw.view(np.float16)).to(cuda_device)
        q, scale = quantize_activation(x)
        # the reference on CUDA: torch's scalar division is a reciprocal multiply
        assert scale.item() == float(g[f"c{i}_scale_cuda"][0]), i
        assert np.array_equal(q.view(torch.uint8).cpu().numpy(), g[f"c{i}_q_cuda"]), i


@pytest.mark.parametrize("shape", [(2048, 14336), (997, 5376)])
def test_fp8_quant_large_matches_torch_reference(cuda_device, shape):
    """The reference test's shapes (test_h3_cuda_precision_ops.py:49-58): our
    kernel vs quantize_per_tensor written in torch (h3_fp8.py:9-12)."""
    from xgen_b200.ops import quantize_activation

    x = torch.randn(shape, device=cuda_device, dtype=torch.bfloat16)
    for sample in (x, torch.zeros_like(x)):
        maximum = torch.finfo(torch.float8_e4m3fn).max
        scale = (sample.float().abs().amax() / maximum).clamp_min(torch.finfo(torch.float32).tiny)
        expected = (sample.float() / scale).clamp(-maximum, maximum).to(torch.float8_e4m3fn)
        actual, actual_scale = quantize_activation(sample)
        assert torch.equal(actual_scale, scale)
        assert torch.equal(actual.view(torch.uint8), expected.view(torch.uint8))


def test_per_token_quant_vs_oracle(cuda_device):
    from xgen_b200.ops import quantize_per_token

    x = (torch.randn(333, 3072) * torch.rand(333, 1) * 10).bfloat16()
    codes, scales = quantize_per_token(x.to(cuda_device))
    rc, rs = of.quantize_per_token(x.float().numpy())
    assert np.array_equal(scales.cpu().numpy(), rs)
    assert np.array_equal(codes.view(torch.uint8).cpu().numpy(), rc)


@pytest.mark.parametrize("rows,cols", [(97, 12288), (64, 100), (5, 16384)])
def test_per_token_quant_widths_vs_oracle(cuda_device, rows, cols):
    """The CTA-per-row kernel (rows up to 16,384 wide, 1-8 chunks per thread)
    and the warp-per-row fallback (unaligned widths) against the oracle."""
    from xgen_b200.ops import quantize_per_token

    g = torch.Generator().manual_seed(rows + cols)
    x = (torch.randn(rows, cols, generator=g) * torch.rand(rows, 1, generator=g) * 10).bfloat16()
    codes, scales = quantize_per_token(x.to(cuda_device))
    rc, rs = of.quantize_per_token(x.float().numpy())
    assert np.array_equal(scales.cpu().numpy(), rs)
    assert np.array_equal(codes.view(torch.uint8).cpu().numpy(), rc)


@pytest.mark.parametrize("peers,seq,batch,hpd,rotary,valid", [
    (2, 40, 1, 3, 128, None),   # 16 channels per lane, full rotary
    (4, 33, 2, 2, 96, 120),     # 16 channels per lane, partial rotary, masked tail
    (1, 50, 1, 5, 48, None),    # 8 channels per lane
    (2, 21, 1, 3, 40, 37),      # generic kernel (rotary half not a multiple of 8)
])
def test_wire_encode_fused_rope_vs_oracle(cuda_device, peers, seq, batch, hpd, rotary, valid):
    """PHAA FP8 wire encode with the pre-A2A RoPE fused in, on the
    [peer, seq, batch, head] views PHAA passes, bit-exact against the
    oracle's RoPE (h3_partial_rope.py:9-29) followed by its wire encode
    (fp8_transport.py:26-63); rows at global sequence index >= valid encode
    as zeros."""
    from xgen_b200.phaa import fp8_transport as fp8
    from xgen_b200.phaa.fp8_transport import WireView

    heads = peers * hpd
    g = torch.Generator().manual_seed(seq * 7 + rotary)
    q, k, v = (torch.randn(batch, seq, heads * 128, generator=g).bfloat16() for _ in range(3))
    ang = torch.rand(seq, rotary // 2, generator=g) * 6.0
    cos = torch.cat([ang.cos(), ang.cos()], dim=-1).float()
    sin = torch.cat([ang.sin(), ang.sin()], dim=-1).float()
    views = [t.to(cuda_device).unflatten(-1, (heads, 128)).unflatten(2, (peers, hpd)).permute(2, 1, 0, 3, 4)
             for t in (q, k, v)]
    got = fp8.encode([x for x in views], 128, peers, rotary_emb=(cos.to(cuda_device), sin.to(cuda_device)),
                     views=[WireView.of(x) for x in views], valid_seq=valid)
    # oracle: RoPE on [B, S, H, D], the same views, masked rows zeroed, encode
    q4, k4, v4 = (t.float().numpy().reshape(batch, seq, heads, 128) for t in (q, k, v))
    qr, kr = ew.partial_rope(q4, k4, cos.numpy(), sin.numpy())
    srcs = []
    for x in (qr, kr, v4):
        x5 = x.reshape(batch, seq, peers, hpd, 128).transpose(2, 1, 0, 3, 4).copy()
        if valid is not None:
            for p in range(peers):
                for s in range(seq):
                    if p * seq + s >= valid:
                        x5[p, s] = 0
        srcs.append(x5)
    want = of.wire_encode(srcs, peers)
    assert np.array_equal(got.cpu().numpy(), want)


def test_wire_encode_full_sp8_shard_vs_oracle(cuda_device):
    """The bench's encode at full size: one SP8 rank's 768P-5s shard (15,856
    tokens, 24 heads, 3 per peer, 3-D RoPE over all 128 channels), the last
    8 rows beyond the real sequence (valid_seq), bit-exact against the
    oracle's RoPE + wire encode; then decode reproduces the oracle's e4m3
    round trip."""
    from xgen_b200.h3.rope import rope_3d
    from xgen_b200.phaa import fp8_transport as fp8
    from xgen_b200.phaa.fp8_transport import WireView

    peers, seq, heads = 8, 15856, 24
    hpd = heads // peers
    g = torch.Generator().manual_seed(8)
    q, k, v = (torch.randn(1, seq, heads * 128, generator=g).bfloat16() for _ in range(3))
    cos, sin = rope_3d((31, 48, 84), 512 + 1250)
    cos, sin = cos[7 * seq:7 * seq + seq].contiguous(), sin[7 * seq:7 * seq + seq].contiguous()
    cos = torch.cat([cos, torch.ones(seq - cos.shape[0], 128)])
    sin = torch.cat([sin, torch.zeros(seq - sin.shape[0], 128)])
    valid = peers * seq - 8
    views = [t.to(cuda_device).unflatten(-1, (heads, 128)).unflatten(2, (peers, hpd)).permute(2, 1, 0, 3, 4)
             for t in (q, k, v)]
    wire = fp8.encode(views, 128, peers, rotary_emb=(cos.to(cuda_device), sin.to(cuda_device)),
                      views=[WireView.of(x) for x in views], valid_seq=valid)
    q4, k4, v4 = (t.float().numpy().reshape(1, seq, heads, 128) for t in (q, k, v))
    qr, kr = ew.partial_rope(q4, k4, cos.numpy(), sin.numpy())
    srcs = []
    for x in (qr, kr, v4):
        x5 = x.reshape(1, seq, peers, hpd, 128).transpose(2, 1, 0, 3, 4).copy()
        x5[peers - 1, seq - 8:] = 0  # global index peer*seq + s >= valid
        srcs.append(x5)
    want = of.wire_encode(srcs, peers)
    assert np.array_equal(wire.cpu().numpy(), want)
    outs = [torch.empty(peers, seq, 1, hpd, 128, device=cuda_device, dtype=torch.bfloat16) for _ in range(3)]
    fp8.decode(wire, outs, 128, peers)
    back = of.wire_decode(want, 3, peers * seq * hpd, peers, 128)
    for o, r in zip(outs, back):
        assert np.array_equal(host_bits(o).reshape(-1), bf16_bits_from_f32(r.reshape(-1)))
