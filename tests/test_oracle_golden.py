"""Pin the CPU oracle against fixtures made by the reference's own kernels."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import elementwise as ew
from oracle import fp8 as of
from oracle.numerics import (bf16_bits_from_f32, e4m3_from_f32, e4m3_to_f32,
                             f32_from_bf16_bits)


def bf(bits):
    return f32_from_bf16_bits(bits)


def test_e4m3_codec_matches_torch():
    # every finite e4m3 value and the midpoints between neighbours (ties)
    vals = e4m3_to_f32(np.arange(256, dtype=np.uint8))
    finite = np.sort(np.unique(vals[np.isfinite(vals)]))
    mids = (finite[:-1] + finite[1:]) / 2
    probe = np.concatenate([finite, mids, np.random.default_rng(0).normal(0, 50, 4096)])
    probe = np.clip(probe, -448, 448).astype(np.float32)
    ours = e4m3_from_f32(probe)
    theirs = torch.from_numpy(probe).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(ours, theirs)
    assert np.array_equal(e4m3_to_f32(ours), torch.from_numpy(theirs).view(torch.float8_e4m3fn).float().numpy())


def test_bf16_rounding_matches_torch():
    x = np.random.default_rng(1).normal(0, 3, 100000).astype(np.float32)
    x[:100] = np.float32(1.0) + np.float32(2.0 ** -8) * np.arange(100)  # exact ties
    ours = bf16_bits_from_f32(x)
    theirs = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, theirs)


def test_partial_rope_golden():
    g = golden("partial_rope")
    for i in range(int(g["ncases"])):
        q, k = bf(g[f"c{i}_q"]), bf(g[f"c{i}_k"])
        qo, ko = ew.partial_rope(q, k, g[f"c{i}_cos"], g[f"c{i}_sin"])
        assert np.array_equal(bf16_bits_from_f32(qo), g[f"c{i}_qo"]), i
        assert np.array_equal(bf16_bits_from_f32(ko), g[f"c{i}_ko"]), i


def test_qk_rms_golden():
    g = golden("qk_rms")
    for i in range(int(g["ncases"])):
        b, s, h, w, r = g[f"c{i}_shape"]
        fused = bf(g[f"c{i}_fused"]).reshape(b, s, 3 * h * w)
        q = fused[..., :h * w].reshape(b, s, h, w)
        k = fused[..., h * w:2 * h * w].reshape(b, s, h, w)
        eps = g[f"c{i}_eps"]
        cos = g[f"c{i}_cos"] if r else None
        sin = g[f"c{i}_sin"] if r else None
        qo, ko = ew.qk_rms(q, k, bf(g[f"c{i}_qw"]), bf(g[f"c{i}_kw"]), eps[0], eps[1], cos, sin)
        # The reduction order of the sum of squares is not part of the
        # algorithm; allow one bf16 ulp at a rare rounding boundary.
        for ours, ref in ((qo, g[f"c{i}_qo"]), (ko, g[f"c{i}_ko"])):
            ob = bf16_bits_from_f32(ours).astype(np.int32)
            diff = np.abs(ob - ref.astype(np.int32))
            assert diff.max() <= 1 and (diff > 0).mean() < 1e-3, i


def test_indexed_affine_golden():
    g = golden("indexed_affine")
    for i in range(int(g["ncases"])):
        b, s, w, m = g[f"c{i}_shape"]
        x, res = bf(g[f"c{i}_x"]), bf(g[f"c{i}_residual"])
        tables = bf(g[f"c{i}_tables"])
        shift, scale, gate = tables[:, :w], tables[:, w:2 * w], tables[:, 2 * w:3 * w]
        idx = g[f"c{i}_idx"]
        mod = ew.indexed_affine(x, scale, shift, idx, modulation=True)
        gated = ew.indexed_affine(x, gate, res, idx, modulation=False)
        assert np.array_equal(bf16_bits_from_f32(mod), g[f"c{i}_mod"]), i
        assert np.array_equal(bf16_bits_from_f32(gated), g[f"c{i}_gate"]), i


def test_swiglu_golden():
    g = golden("swiglu")
    for i in range(int(g["ncases"])):
        y, peak = ew.swiglu(bf(g[f"c{i}_x"]))
        assert np.array_equal(bf16_bits_from_f32(y), g[f"c{i}_y"]), i
        assert np.float32(peak) == g[f"c{i}_amax"][0]


def _wire_sources(g, i):
    streams, peers, seq, batch, heads, width, align, strided = g[f"c{i}_meta"]
    if strided:
        fused = bf(g[f"c{i}_fused"]).reshape(batch, seq, -1)
        full_heads = fused.shape[-1] // 3 // width
        chunks = np.split(fused, 3, axis=-1)
        views = []
        for t in chunks:
            t = t.reshape(batch, seq, peers, full_heads // peers, width)[:, :, :, 4:, :]
            views.append(np.transpose(t, (2, 1, 0, 3, 4)))
        return views
    return [bf(g[f"c{i}_in{s}"]) for s in range(streams)]


def test_fp8_wire_golden():
    g = golden("fp8_wire")
    for i in range(int(g["ncases"])):
        streams, peers, seq, batch, heads, width, align, strided = g[f"c{i}_meta"]
        srcs = _wire_sources(g, i)
        rows = srcs[0].size // width
        pad = of.peer_padding(rows // peers, streams, width) if align else 0
        wire = of.wire_encode(srcs, peers, pad)
        assert np.array_equal(wire, g[f"c{i}_wire"].reshape(-1)), i
        outs = of.wire_decode(wire, streams, rows, peers, width, pad)
        for s in range(streams):
            ref = g[f"c{i}_out{s}"].reshape(-1)
            assert np.array_equal(bf16_bits_from_f32(outs[s]).reshape(-1), ref), (i, s)


def test_fp8_quant_golden():
    g = golden("fp8_quant")
    for i in range(int(g["ncases"])):
        raw = g[f"c{i}_x"]
        x = bf(raw) if int(g[f"c{i}_dtype"]) == 0 else raw.view(np.float16).astype(np.float32)
        codes, scale = of.quantize_per_tensor(x, scalar_div="ieee")  # the CPU run
        assert np.float32(scale) == g[f"c{i}_scale"][0], i
        assert np.array_equal(codes, g[f"c{i}_q"]), i
        codes, scale = of.quantize_per_tensor(x, scalar_div="cuda")  # CUDA semantics
        assert np.float32(scale) == g[f"c{i}_scale_cuda"][0], i
        assert np.array_equal(codes, g[f"c{i}_q_cuda"]), i


def test_e4m3_decode_table_finite():
    vals = e4m3_to_f32(np.arange(256, dtype=np.uint8))
    assert np.nanmax(vals) == 448.0 and np.isnan(vals[0x7F]) and np.isnan(vals[0xFF])


@pytest.mark.parametrize("scale", [1e-3, 1.0, 300.0])
def test_scaled_mm_oracle_close_to_fp32(scale):
    rng = np.random.default_rng(0)
    a = rng.normal(0, scale, (33, 64)).astype(np.float32)
    w = rng.normal(0, 0.02, (48, 64)).astype(np.float32)
    qa, sa = of.quantize_per_tensor(a)
    qw, sw = of.quantize_per_tensor(w)
    out = of.scaled_mm(qa, qw, sa, sw)
    ref = a @ w.T
    rel = np.sqrt(((out - ref) ** 2).mean()) / np.sqrt((ref ** 2).mean())
    assert rel < 0.08
