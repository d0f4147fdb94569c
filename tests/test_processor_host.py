"""install() and H3AttnProcessorB200 host logic on CPU: the reference's
validation errors (x_diffusers/x_diffusers/adaptor/h3_cuda_precision.py:
229-236, h3_cuda.py:126-129), the module swap, and how the processor maps a
module's SP/PHAA attributes onto the SP attention call (no kernel runs)."""
from types import SimpleNamespace

import pytest
import torch
from torch import nn

from h3_fakes import fake_h3
from xgen_b200.fp8_linear import H3FP8Linear
from xgen_b200.h3 import processor as proc
from xgen_b200.h3.block import H3BlockConfig, H3DiTBlockB200

CFG = H3BlockConfig(hidden=256, heads=2, head_dim=128, ffn=512, qk_norm=True)


def _model(blocks=2):
    weights = H3DiTBlockB200.random_weights(CFG, seed=1)
    table = torch.zeros(3, 6 * CFG.hidden, dtype=torch.bfloat16)
    return fake_h3(weights, CFG, table, blocks=blocks)


def test_install_swaps_modules_and_sets_flags():
    model = _model()
    backend = proc.install(model, "fp8-bf16", device="cpu")
    assert backend.precision == "bf16" and model._h3_dense_cuda is backend
    assert model._h3_cuda_precision == "fp8-bf16"
    for block in model.transformer_blocks:
        attn = block.attn
        assert attn.fused_projections and attn.to_q is None and attn.to_k is None and attn.to_v is None
        assert isinstance(attn.to_qkv, H3FP8Linear) and attn.to_qkv.out_features == 3 * CFG.hidden
        assert isinstance(attn.to_out[0], H3FP8Linear) and isinstance(attn.to_out[1], nn.Dropout)
        assert isinstance(block.ff.net[0].proj, H3FP8Linear) and isinstance(block.ff.net[2], H3FP8Linear)
        assert attn._h3_attention_backend is backend and isinstance(attn.processor, proc.H3AttnProcessorB200)
        assert attn._h3_fused_qk_rms and attn._h3_fused_partial_rope and not attn._h3_phaa_fp8
        assert block._h3_b200_block is not None and block._h3_b200_block.to_qkv is attn.to_qkv
        assert block.forward.__func__ is proc.h3_block_forward_b200


def test_install_concatenates_qkv_in_order():
    model = _model(1)
    attn = model.transformer_blocks[0].attn
    w = torch.cat([attn.to_q.weight, attn.to_k.weight, attn.to_v.weight]).detach()
    proc.install(model, "fp8-sage", device="cpu")
    expect = H3FP8Linear(w, None, scaling="per_token")
    assert torch.equal(attn.to_qkv.weight.view(torch.uint8), expect.weight.view(torch.uint8))
    assert torch.equal(attn.to_qkv.weight_scale, expect.weight_scale)


def test_install_rejects_like_the_reference(monkeypatch):
    with pytest.raises(ValueError, match="precision"):
        proc.install(_model(), "fp4", device="cpu")
    model = _model()
    model.transformer_blocks[1].attn.fused_projections = True
    with pytest.raises(ValueError, match="unfused BF16"):
        proc.install(model, device="cpu")
    assert model.transformer_blocks[0].attn.to_q is not None  # nothing converted
    model = _model()
    a = model.transformer_blocks[0].attn
    a.to_q = nn.Linear(CFG.hidden, CFG.hidden, bias=True).bfloat16()
    with pytest.raises(ValueError, match="biases"):
        proc.install(model, device="cpu")
    with pytest.raises(ValueError, match="XGEN_PHAA_FP8"):
        proc.install(_model(), fp8_transport=True, phaa_num=1, device="cpu")  # SP = 1
    monkeypatch.setenv("XGEN_PHAA_FP8", "1")
    manager = SimpleNamespace(sp_group=None, sp_size=2)
    with pytest.raises(ValueError, match="XGEN_PHAA_FP8"):
        proc.install(_model(), parallel_manager=manager, phaa_num=2, device="cpu")  # 1 local head
    proc.install(_model(), parallel_manager=manager, phaa_num=1, device="cpu")


class _Recorder:
    def __init__(self):
        self.calls = []

    def __call__(self, q, k, v, rotary_emb, **kw):
        self.calls.append(kw)
        return torch.zeros_like(q)


@pytest.mark.parametrize("sp,phaa,fp8,tp_cp,expect", [
    (1, 0, False, False, dict(sp_size=1, use_phaa=False, pad_key="pad")),
    (4, 0, False, False, dict(sp_size=4, use_phaa=False, pad_key="pad")),
    (4, 0, False, True, dict(sp_size=4, use_phaa=False, pad_key="mmh3_seq")),
    (4, 2, True, False, dict(sp_size=4, use_phaa=True, pad_key="mmh3_seq", phaa_num=2, fp8_transport=True)),
])
def test_processor_maps_module_attributes(monkeypatch, sp, phaa, fp8, tp_cp, expect):
    rec = _Recorder()
    monkeypatch.setattr(proc, "sp_self_attention", rec)
    monkeypatch.setattr(proc, "try_h3_qk_rms", lambda *a, **k: None)
    monkeypatch.setattr(proc.H3AttnProcessorB200, "comm_stream", lambda self, device: "stream")
    attn = SimpleNamespace(
        heads=8, fused_projections=True, to_qkv=nn.Linear(1024, 3 * 1024, bias=False),
        norm_q=nn.RMSNorm(128), norm_k=nn.RMSNorm(128), to_out=[nn.Identity(), nn.Identity()],
        parallel_manager=SimpleNamespace(sp_group="group", sp_size=sp), _h3_attention_backend="backend",
        _h3_phaa_num=phaa, _h3_phaa_fp8=fp8, _h3_tp_cp=tp_cp, _h3_fused_qk_rms=True)
    mask = torch.ones(1, dtype=torch.bool)
    out = proc.H3AttnProcessorB200()(attn, torch.randn(1, 16, 1024), rotary_emb=("c", "s"), attention_mask=mask)
    assert out.shape == (1, 16, 1024)
    kw = rec.calls[0]
    for key, value in expect.items():
        assert kw[key] == value, key
    assert kw["backend"] == "backend" and kw["heads"] == 8 and kw["head_dim"] == 128
    assert kw["attention_mask"] is mask
    assert (kw["comm_stream"] == "stream") == (sp > 1)
