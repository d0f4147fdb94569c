"""The H3 DiT block on B200 kernels (FP8 linears, Sage/BF16 attention,
fused AdaLN) vs the fp32 restatement of the reference block math.

Tolerance: FP8 e4m3 projections carry ~3-5 % relative error each (the
reference's own FP8-vs-BF16 bound is rel-RMSE < 0.08 per projection,
x_base/tests/test_h3_cuda_precision_ops.py:19-32). The block's branch
output (y - x) must keep cosine >= 0.99 with the fp32 branch, and the fused
prologue must agree with the unfused kernels it replaces."""
import numpy as np
import pytest
import torch

from oracle import block as ob
from oracle.attention import cosine

pytestmark = pytest.mark.gpu


def _setup(cfg, s, seed=0):
    from xgen_b200.h3.block import H3DiTBlockB200
    from xgen_b200.h3.rope import rope_partial

    g = torch.Generator().manual_seed(seed)
    x = torch.randn(1, s, cfg.hidden, generator=g).bfloat16()
    table = (0.5 * torch.randn(3, 6 * cfg.hidden, generator=g)).bfloat16()
    idx = torch.randint(3, (s,), generator=g)
    cos, sin = rope_partial(s, 96)
    w = H3DiTBlockB200.random_weights(cfg, seed)
    return x, table, idx, cos, sin, w


@pytest.mark.parametrize("variant", ["baseline", "reference_model"])
@pytest.mark.parametrize("precision", ["sage", "bf16"])
def test_block_vs_fp32_restatement(cuda_device, variant, precision):
    from xgen_b200.h3.block import H3BlockConfig, H3DiTBlockB200

    if variant == "baseline":  # LayerNorm + GELU
        cfg = H3BlockConfig(hidden=1536, heads=12, ffn=6144, precision=precision)
    else:  # the reference model: RMSNorm, Q/K RMSNorm, SwiGLU
        cfg = H3BlockConfig(hidden=1536, heads=12, ffn=4096, activation="swiglu", norm="rmsnorm",
                            qk_norm=True, precision=precision)
    s = 640
    x, table, idx, cos, sin, w = _setup(cfg, s)
    blk = H3DiTBlockB200(w, cfg, cuda_device)
    dev = cuda_device
    y = blk.forward(x.to(dev), table.to(dev), idx.to(dev), (cos.to(dev), sin.to(dev)))
    torch.cuda.synchronize()
    ref = ob.block_forward(x.float(), w, table, idx, cos, sin, cfg)
    got = y.float().cpu()
    assert torch.isfinite(got).all()
    assert cosine((got - x.float()).numpy(), (ref - x.float()).numpy()) >= 0.99


def test_norm_modulate_quant_matches_unfused(cuda_device):
    """Fused prologue vs torch LayerNorm + the bit-exact indexed-affine kernel
    + per-token quantisation."""
    from xgen_b200.ops import indexed_affine, norm_modulate_quant, quantize_per_token

    g = torch.Generator().manual_seed(4)
    b, s, h = 2, 300, 3072
    x = (3 * torch.randn(b, s, h, generator=g)).bfloat16().to(cuda_device)
    table = torch.randn(5, 6 * h, generator=g).bfloat16().to(cuda_device)
    shift, scale = table[:, :h], table[:, h:2 * h]
    idx = torch.randint(5, (s,), generator=g).to(cuda_device)
    codes, scales, mod = norm_modulate_quant(x, "layernorm", None, 1e-6, scale, shift, idx,
                                             return_bf16=True)
    n = torch.nn.functional.layer_norm(x.float(), (h,), eps=1e-6).bfloat16()
    ref_mod = indexed_affine(n, scale, shift, idx, modulation=True)
    d = (mod.float() - ref_mod.float()).abs()
    # The fp32 LayerNorm statistics may round n differently by one bf16 ulp;
    # that ulp is scaled by (1 + scale) and the shift can cancel the result,
    # so the bound is relative to |n * (1 + scale)| plus one output ulp.
    f = (1.0 + scale.index_select(0, idx).float()).bfloat16().float()
    bound = (n.float() * f).abs() * 2 ** -7 + ref_mod.float().abs() * 2 ** -7 + 1e-6
    assert (mod == ref_mod).float().mean() > 0.99
    assert (d <= bound).all()
    rc, rs = quantize_per_token(mod.reshape(b * s, h))
    assert torch.equal(scales, rs) and torch.equal(codes.view(torch.uint8), rc.view(torch.uint8))


def test_output_adaln_matches_layernorm_then_indexed_affine(cuda_device):
    """Final-layer norm_out (minimax_h3.py:672-696): the default path is
    bitwise the reference's (torch LayerNorm + the bit-exact indexed affine,
    as test_h3_output_adaln.py:29-45 pins, including strided table chunks);
    the one-pass kernel equals the bf16 copy of the quantising prologue and
    stays within its one-ulp bound."""
    from xgen_b200.ops import norm_modulate_quant, output_adaln

    g = torch.Generator().manual_seed(5)
    for b, s, h in ((1, 2003, 5376), (2, 137, 512)):
        x = torch.randn(b, s, h, generator=g).bfloat16().to(cuda_device)
        modulation = torch.randn(3, 2 * h, generator=g).bfloat16().to(cuda_device)
        shift, scale = modulation.chunk(2, dim=-1)  # row stride 2h, as the cached table
        idx = (torch.arange(s) % 3).to(cuda_device)
        n = torch.nn.functional.layer_norm(x, (h,), eps=1e-6)
        eager = n * (1.0 + scale.index_select(0, idx)) + shift.index_select(0, idx)
        got = output_adaln(x, scale, shift, idx)
        assert torch.equal(got.view(torch.int16), eager.view(torch.int16))
        fused = output_adaln(x, scale, shift, idx, fused=True)
        _, _, mod = norm_modulate_quant(x, "layernorm", None, 1e-6, scale, shift, idx, return_bf16=True)
        assert torch.equal(fused, mod)
        f = (1.0 + scale.index_select(0, idx).float()).bfloat16().float()
        bound = (n.float() * f).abs() * 2 ** -7 + eager.float().abs() * 2 ** -7 + 1e-6
        assert (fused == eager).float().mean() > 0.99
        assert ((fused.float() - eager.float()).abs() <= bound).all()


@pytest.mark.parametrize("norm,h", [("rmsnorm", 1536), ("rmsnorm", 5376), ("layernorm", 4096),
                                    ("layernorm", 512), ("rmsnorm", 1004)])
def test_norm_modulate_quant_widths(cuda_device, norm, h):
    """The fused prologue for RMSNorm x weight and LayerNorm at widths that
    take each vector variant (1-6 chunks per thread) and the scalar kernel
    (h % 8 != 0): within one bf16 ulp of torch's norm + the bit-exact
    indexed affine, and its e4m3 codes equal per-token quantisation of its
    own bf16 output."""
    from xgen_b200.ops import indexed_affine, norm_modulate_quant, quantize_per_token

    g = torch.Generator().manual_seed(h)
    b, s = 1, 96
    x = (2 * torch.randn(b, s, h, generator=g)).bfloat16().to(cuda_device)
    table = torch.randn(3, 2 * h, generator=g).bfloat16().to(cuda_device)
    shift, scale = table[:, :h], table[:, h:]
    idx = torch.randint(3, (s,), generator=g).to(cuda_device)
    w = (1 + 0.1 * torch.randn(h, generator=g)).bfloat16().to(cuda_device) if norm == "rmsnorm" else None
    codes, scales, mod = norm_modulate_quant(x, norm, w, 1e-6, scale, shift, idx, return_bf16=True)
    if norm == "rmsnorm":
        n = torch.nn.functional.rms_norm(x.float(), (h,), w.float(), eps=1e-6).bfloat16()
    else:
        n = torch.nn.functional.layer_norm(x.float(), (h,), eps=1e-6).bfloat16()
    ref_mod = indexed_affine(n, scale, shift, idx, modulation=True)
    f = (1.0 + scale.index_select(0, idx).float()).bfloat16().float()
    bound = (n.float() * f).abs() * 2 ** -7 + ref_mod.float().abs() * 2 ** -7 + 1e-6
    assert (mod == ref_mod).float().mean() > 0.99
    assert ((mod.float() - ref_mod.float()).abs() <= bound).all()
    rc, rs = quantize_per_token(mod.reshape(b * s, h))
    assert torch.equal(scales, rs) and torch.equal(codes.view(torch.uint8), rc.view(torch.uint8))


@pytest.mark.parametrize("precision", ["sage", "bf16"])
def test_config1_block_at_stated_shape(cuda_device, precision):
    """BASELINE config 1 at its stated shape: 4,096 video tokens of a
    4x32x32 latent grid + 256 text tokens, hidden 1536, 12 x 128 heads, 3-D
    RoPE (theta 10000, head dims 32/48/48 over t/h/w), AdaLN LayerNorm from
    one random 6 x 1536 row, GELU FFN 6144, activations N(0, 1), weights
    N(0, 0.02), seed 0; the B200 block (FP8 per-token projections, Sage or
    BF16 attention) against the unquantised fp32 restatement of the
    reference block (h3_npu_fusion.py:339-356).

    Tolerance on the branch output d = y - x (FP8 error compounds over the
    four projections; the reference's own FP8-vs-BF16 gate is rel-RMSE < 0.08
    per projection): cosine >= 0.995, rel-RMSE <= 0.08, the 99.9th
    percentile of |y - ref| <= 5 % of max |d_ref|, and max |y - ref| <= 15 %
    of max |d_ref| (with N(0, 1) AdaLN rows the gates and (1 + scale) reach
    +-3, so the branch output spans several units and its largest elements
    carry the largest absolute FP8 error)."""
    from xgen_b200.h3.block import H3BlockConfig, H3DiTBlockB200
    from xgen_b200.h3.rope import rope_3d

    cfg = H3BlockConfig(hidden=1536, heads=12, head_dim=128, ffn=6144, activation="gelu",
                        norm="layernorm", precision=precision)
    cos, sin = rope_3d((4, 32, 32), 256, split=(32, 48, 48), theta=10000.0)
    s = cos.shape[0]
    assert s == 4352
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1, s, cfg.hidden, generator=g).bfloat16()
    table = torch.randn(1, 6 * cfg.hidden, generator=g).bfloat16()
    idx = torch.zeros(s, dtype=torch.int64)
    w = H3DiTBlockB200.random_weights(cfg, seed=0)
    blk = H3DiTBlockB200(w, cfg, cuda_device)
    dev = cuda_device
    y = blk.forward(x.to(dev), table.to(dev), idx.to(dev), (cos.to(dev), sin.to(dev)))
    torch.cuda.synchronize()
    ref = ob.block_forward(x.float(), w, table, idx, cos, sin, cfg)
    got = y.float().cpu()
    assert torch.isfinite(got).all()
    d_got, d_ref = got - x.float(), ref - x.float()
    cos_sim = cosine(d_got.numpy(), d_ref.numpy())
    rel_rmse = float((d_got - d_ref).pow(2).mean().sqrt() / d_ref.pow(2).mean().sqrt())
    err = (got - ref).abs()
    max_abs, p999 = float(err.max()), float(torch.quantile(err.flatten()[::7], 0.999))
    peak = float(d_ref.abs().max())
    print(f"config1 {precision}: cosine {cos_sim:.6f} rel-RMSE {rel_rmse:.4f} max-abs {max_abs:.4f} "
          f"p99.9 {p999:.4f} branch peak {peak:.3f}")
    assert cos_sim >= 0.995 and rel_rmse <= 0.08, (cos_sim, rel_rmse)
    assert p999 <= 0.05 * peak and max_abs <= 0.15 * peak, (p999, max_abs, peak)
