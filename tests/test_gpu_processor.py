"""The drop-in H3 attention processor and recipe installer on a stand-in H3
transformer with the reference's module layout (tests/h3_fakes.py).

After install(): the processor's attention branch equals the same kernels
called directly, bit for bit; the installed block forward equals
H3DiTBlockB200 built from the same weights, bit for bit; the module-by-module
fallback (the reference's fused_h3_block_forward composition) agrees with it
to the rounding of the unfused norm (cosine >= 0.9999); a masked call takes
the backend's masked path."""
import pytest
import torch

from h3_fakes import fake_h3

pytestmark = pytest.mark.gpu

HID, HEADS, FFN, S = 512, 4, 2048, 1000


def _setup(cuda_device, precision="sage"):
    from xgen_b200.h3.block import H3BlockConfig, H3DiTBlockB200
    from xgen_b200.h3.rope import rope_partial

    cfg = H3BlockConfig(hidden=HID, heads=HEADS, head_dim=128, ffn=FFN, activation="gelu",
                        norm="layernorm", qk_norm=True, precision=precision)
    weights = H3DiTBlockB200.random_weights(cfg, seed=4)
    g = torch.Generator().manual_seed(9)
    table = (0.1 * torch.randn(3, 6 * HID, generator=g)).bfloat16()
    model = fake_h3(weights, cfg, table).to(cuda_device)
    reference = H3DiTBlockB200(weights, cfg, cuda_device)
    x = torch.randn(1, S, HID, generator=g).bfloat16().to(cuda_device)
    idx = torch.randint(0, 3, (S,), generator=g).to(cuda_device)
    cos, sin = rope_partial(S, 96)
    return model, reference, x, table.to(cuda_device), idx, (cos.to(cuda_device), sin.to(cuda_device))


@pytest.mark.parametrize("precision", ["fp8-sage", "fp8-bf16"])
def test_installed_block_matches_b200_block(cuda_device, precision):
    from xgen_b200.fp8_linear import H3FP8Linear
    from xgen_b200.h3.processor import H3AttnProcessorB200, install

    model, reference, x, table, idx, rot = _setup(cuda_device, {"fp8-sage": "sage", "fp8-bf16": "bf16"}[precision])
    backend = install(model, precision)
    block = model.transformer_blocks[0]
    attn = block.attn
    assert attn.fused_projections and attn.to_q is None and isinstance(attn.to_qkv, H3FP8Linear)
    assert isinstance(attn.to_out[0], H3FP8Linear) and isinstance(block.ff.net[2], H3FP8Linear)
    assert isinstance(block.ff.net[0].proj, H3FP8Linear)
    assert isinstance(attn.processor, H3AttnProcessorB200) and attn._h3_attention_backend is backend
    assert block._h3_b200_block is not None
    with torch.no_grad():
        got = block(x, None, idx, rot)
        expect = reference.forward(x, table, idx, rot)
    torch.cuda.synchronize()
    assert torch.equal(got, expect)
    assert backend.kernel_calls == 1


def test_processor_branch_matches_kernels(cuda_device):
    """attn(hidden, rotary) == to_out(sp_self_attention(qk_rms(to_qkv(hidden))))."""
    from xgen_b200.h3.processor import install
    from xgen_b200.h3.sp_attention import sp_self_attention
    from xgen_b200.ops import try_h3_qk_rms

    model, reference, x, table, idx, rot = _setup(cuda_device)
    install(model, "fp8-sage")
    attn = model.transformer_blocks[0].attn
    with torch.no_grad():
        got = attn(x, rot)
        q, k, v = reference.to_qkv(x).chunk(3, dim=-1)
        q4, k4 = try_h3_qk_rms(q.unflatten(-1, (HEADS, 128)), k.unflatten(-1, (HEADS, 128)),
                               reference.norm_q, reference.norm_k)
        att = sp_self_attention(q4.flatten(2), k4.flatten(2), v, rot, backend=reference.attention,
                                heads=HEADS, head_dim=128)
        expect = reference.to_out(att)
    torch.cuda.synchronize()
    assert torch.equal(got, expect)


def test_module_by_module_fallback_agrees(cuda_device):
    """Without the fused block (e.g. a layout it does not cover), the
    installed forward composes norm -> indexed affine -> processor -> gated
    residual -> FFN, as fused_h3_block_forward does."""
    from xgen_b200.h3.processor import install

    model, reference, x, table, idx, rot = _setup(cuda_device)
    install(model, "fp8-sage")
    block = model.transformer_blocks[0]
    with torch.no_grad():
        fused = block(x, None, idx, rot)
        block._h3_b200_block = None
        composed = block(x, None, idx, rot)
    a, b = fused.double().flatten(), composed.double().flatten()
    cos = float(a @ b / (a.norm() * b.norm()))
    assert cos >= 0.9999, cos
    assert float((fused - composed).abs().max()) <= 0.05


def test_masked_call_takes_the_masked_path(cuda_device):
    """With a mask the backend runs PyTorch SDPA (the reference backends'
    masked fallback): the processor output equals that composition."""
    import torch.nn.functional as F

    from xgen_b200.h3.processor import install
    from xgen_b200.ops import try_h3_partial_rope, try_h3_qk_rms

    model, reference, x, table, idx, rot = _setup(cuda_device)
    backend = install(model, "fp8-sage")
    attn = model.transformer_blocks[0].attn
    g = torch.Generator(device=cuda_device).manual_seed(3)
    mask = torch.rand(1, 1, S, S, device=cuda_device, generator=g) > 0.1
    with torch.no_grad():
        before = backend.kernel_calls
        masked = attn(x, rot, mask)
        assert backend.kernel_calls == before  # SDPA, not the Sage kernel
        q, k, v = reference.to_qkv(x).chunk(3, dim=-1)
        q4, k4 = try_h3_qk_rms(q.unflatten(-1, (HEADS, 128)), k.unflatten(-1, (HEADS, 128)),
                               reference.norm_q, reference.norm_k)
        q4, k4 = try_h3_partial_rope(q4.contiguous(), k4.contiguous(), *rot)
        v4 = v.unflatten(-1, (HEADS, 128))
        att = F.scaled_dot_product_attention(q4.transpose(1, 2), k4.transpose(1, 2), v4.transpose(1, 2),
                                             attn_mask=mask)
        expect = reference.to_out(att.transpose(1, 2).flatten(2))
    torch.cuda.synchronize()
    assert torch.equal(masked, expect)
