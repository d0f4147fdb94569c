"""tcgen05 FP8 GEMM / H3FP8Linear vs torch._scaled_mm, the CPU oracle and
the reference's own accuracy bound.

Tolerance: the GEMM's fp32 accumulation order differs from cuBLASLt's and
from the oracle's exact sum. Where an output cancels towards zero, that
fp32 difference (about K * 2^-24 * |terms|) can be a few ulps of the small
bf16 result, so the bound is relative to the output scale: >= 99.5 % of
elements bit-identical and |difference| <= 2^-10 * rms(reference) everywhere."""
import numpy as np
import pytest
import torch

from oracle import fp8 as of

pytestmark = pytest.mark.gpu


def assert_gemm_close(got: torch.Tensor, ref) -> None:
    """Per element: |got - ref| <= one bf16 ulp of |ref| + 2^-10 * rms(ref)
    (the cancellation allowance), and >= 99.5 % of elements identical."""
    g = got.float().cpu().numpy().astype(np.float64)
    r = ref.float().cpu().numpy() if isinstance(ref, torch.Tensor) else np.asarray(ref, np.float32)
    r = r.astype(np.float64)
    rms = np.sqrt((r ** 2).mean())
    ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(r), 1e-30))) - 7)
    bound = ulp + 2.0 ** -10 * rms
    worst = (np.abs(g - r) / bound).max()
    same = (g == r).mean()
    assert same >= 0.995 and worst <= 1.0, (same, worst)


def test_fp8_projection_bias_and_unaligned_rows(cuda_device):
    """x_base/tests/test_h3_cuda_precision_ops.py:19-32 on our module."""
    from xgen_b200.fp8_linear import H3FP8Linear

    torch.manual_seed(42)
    weight = torch.randn(256, 128, dtype=torch.bfloat16)
    bias = torch.randn(256, dtype=torch.bfloat16)
    layer = H3FP8Linear(weight, bias).cuda()
    x = torch.randn(2, 19, 128, device=cuda_device, dtype=torch.bfloat16)
    result = layer(x)
    reference = torch.nn.functional.linear(x, weight.cuda(), bias.cuda())
    assert result.shape == reference.shape and result.dtype == reference.dtype
    assert layer.weight.dtype == torch.float8_e4m3fn and layer.calls == 1
    assert torch.isfinite(result).all()
    rel = (result.float() - reference.float()).square().mean().sqrt() / reference.float().square().mean().sqrt()
    assert rel.item() < 0.08


def test_projection_rejects_unaligned_dimensions():
    from xgen_b200.fp8_linear import H3FP8Linear

    with pytest.raises(ValueError, match="divisible by 16"):
        H3FP8Linear(torch.randn(17, 32))


@pytest.mark.parametrize("m,n,k", [(19, 256, 128), (1000, 3072, 3072), (333, 9216, 3072),
                                   (64, 12288, 3072), (130, 3072, 12288)])
def test_per_tensor_gemm_matches_scaled_mm(cuda_device, m, n, k):
    from xgen_b200.fp8_linear import H3FP8Linear

    g = torch.Generator().manual_seed(m + n)
    w = (torch.randn(n, k, generator=g) * 0.02).bfloat16()
    bias = torch.randn(n, generator=g).bfloat16()
    layer = H3FP8Linear(w, bias).to(cuda_device)
    x = torch.randn(m, k, generator=g).bfloat16().to(cuda_device)
    got = layer(x)
    from xgen_b200.ops import quantize_activation

    qa, sa = quantize_activation(x)
    ref = torch._scaled_mm(qa, layer.weight.t(), scale_a=sa, scale_b=layer.weight_scale.reshape(()),
                           bias=layer.bias, out_dtype=torch.bfloat16)
    assert_gemm_close(got, ref)


def test_per_token_gemm_matches_oracle(cuda_device):
    from xgen_b200.fp8_linear import H3FP8Linear

    g = torch.Generator().manual_seed(3)
    m, n, k = 200, 1024, 3072
    w = (torch.randn(n, k, generator=g) * 0.02).bfloat16()
    layer = H3FP8Linear(w, None, scaling="per_token").to(cuda_device)
    x = (torch.randn(m, k, generator=g) * torch.rand(m, 1, generator=g) * 5).bfloat16().to(cuda_device)
    got = layer(x)
    qa, sa = of.quantize_per_token(x.float().cpu().numpy())
    qw = layer.weight.view(torch.uint8).cpu().numpy()
    sw = layer.weight_scale.cpu().numpy()
    ref = of.scaled_mm(qa, qw, sa, sw)
    assert_gemm_close(got, ref)


@pytest.mark.parametrize("offset", [1, 4])
def test_per_token_quantize_misaligned_output(cuda_device, offset):
    """A C-ABI caller may hand xgb_fp8_quantize_per_token an output that is
    not 8-byte aligned: it must take the byte-store path and give the same
    codes and scales as the aligned call and the oracle."""
    from xgen_b200 import _lib
    from xgen_b200.ops import quantize_per_token

    g = torch.Generator().manual_seed(5)
    rows, cols = 37, 3072
    x = (torch.randn(rows, cols, generator=g) * 3).bfloat16().to(cuda_device)
    codes, scales = quantize_per_token(x)
    buf = torch.zeros(rows * cols + 16, dtype=torch.uint8, device=cuda_device)
    sc = torch.empty(rows, dtype=torch.float32, device=cuda_device)
    _lib.call("xgb_fp8_quantize_per_token", x.data_ptr(), _lib.XGB_BF16, rows, cols, x.stride(0),
              buf.data_ptr() + offset, sc.data_ptr(), torch.cuda.current_stream().cuda_stream)
    got = buf[offset:offset + rows * cols].view(rows, cols)
    assert torch.equal(got, codes.view(torch.uint8)) and torch.equal(sc, scales)
    qa, sa = of.quantize_per_token(x.float().cpu().numpy())
    assert np.array_equal(got.cpu().numpy(), qa) and np.array_equal(sc.cpu().numpy(), sa)
    assert int(buf[:offset].sum()) == 0 and int(buf[offset + rows * cols:].sum()) == 0


def test_gated_epilogue_matches_gemm_then_indexed_affine(cuda_device):
    """attn_out -> x + gate[idx] * attn_out with the reference's rounding,
    fused vs GEMM followed by the (bit-exact) indexed-affine kernel."""
    from xgen_b200.fp8_linear import H3FP8Linear
    from xgen_b200.ops import indexed_affine

    g = torch.Generator().manual_seed(9)
    b, s, hid = 1, 333, 3072
    w = (torch.randn(hid, hid, generator=g) * 0.02).bfloat16()
    layer = H3FP8Linear(w, torch.randn(hid, generator=g).bfloat16(), scaling="per_token").to(cuda_device)
    x = torch.randn(b, s, hid, generator=g).bfloat16().to(cuda_device)
    res = torch.randn(b, s, hid, generator=g).bfloat16().to(cuda_device)
    tables = torch.randn(3, 6 * hid, generator=g).bfloat16().to(cuda_device)
    gate = tables[:, 2 * hid:3 * hid]
    idx = torch.randint(3, (s,), generator=g).to(cuda_device)
    fused = layer.forward_gated(x, gate, idx, res)
    plain = layer(x)
    two_step = indexed_affine(plain, gate, res, idx, modulation=False)
    assert torch.equal(fused, two_step)


@pytest.mark.parametrize("scaling", ["per_tensor", "per_token"])
def test_swiglu_epilogue_matches_gemm_then_swiglu(cuda_device, scaling):
    """FFN up projection + gate-first SwiGLU (h3_swiglu.py:15-41) fused in
    the GEMM epilogue vs the plain GEMM followed by the bit-exact SwiGLU
    kernel: identical bits (same bf16 GEMM results, same SwiGLU rounding)."""
    from xgen_b200.fp8_linear import H3FP8Linear
    from xgen_b200.ops import gate_first_swiglu, quantize_per_token

    g = torch.Generator().manual_seed(11)
    m, hid, f = 389, 1024, 1536
    w = (torch.randn(2 * f, hid, generator=g) * 0.03).bfloat16()
    bias = torch.randn(2 * f, generator=g).bfloat16()
    plain = H3FP8Linear(w, bias, scaling=scaling).to(cuda_device)
    fused = plain.swiglu_interleaved()
    x = torch.randn(m, hid, generator=g).bfloat16().to(cuda_device)
    expect = gate_first_swiglu(plain(x))
    got = fused(x)
    assert got.shape == (m, f)
    assert torch.equal(got, expect)
    q, s = quantize_per_token(x)
    assert torch.equal(fused.forward_quantized(q, s, activation=3),
                       gate_first_swiglu(plain.forward_quantized(q, s)))
    with pytest.raises(ValueError):
        plain.forward_quantized(q, s, activation=3)


@pytest.mark.parametrize("m,n,k", [(129, 256, 208), (257, 272, 3072), (1000, 3072, 256),
                                   (15845, 512, 3072)])
def test_cta_pair_gemm_matches_single_cta(cuda_device, monkeypatch, m, n, k):
    """The CTA-pair kernel (cta_group::2, M > 128) gives the same bits as the
    1-CTA kernel for every epilogue, including M, N and K tails: both
    accumulate each output over K in the same order."""
    from xgen_b200.fp8_linear import H3FP8Linear
    from xgen_b200.ops import quantize_per_token

    g = torch.Generator().manual_seed(m + n + k)
    w = (torch.randn(n, k, generator=g) * 0.03).bfloat16()
    bias = torch.randn(n, generator=g).bfloat16()
    layer = H3FP8Linear(w, bias, scaling="per_token").to(cuda_device)
    x = torch.randn(m, k, generator=g).bfloat16().to(cuda_device)
    q, s = quantize_per_token(x)
    res = torch.randn(1, m, n, generator=g).bfloat16().to(cuda_device)
    gate = torch.randn(3, n, generator=g).bfloat16().to(cuda_device)
    idx = torch.randint(3, (m,), generator=g).to(cuda_device)

    def run():
        out = [layer.forward_quantized(q, s), layer.forward_quantized(q, s, activation=1),
               layer.forward_gated(x.unsqueeze(0), gate, idx, res)]
        if n % 256 == 0:
            out.append(layer.swiglu_interleaved().forward_quantized(q, s, activation=3))
        torch.cuda.synchronize()
        return out

    monkeypatch.setenv("XGB_GEMM_CTA_PAIRS", "0")
    single = run()
    monkeypatch.setenv("XGB_GEMM_CTA_PAIRS", "1")
    pair = run()
    from xgen_b200.attention import kernel_errors
    assert kernel_errors() == 0
    for a, b in zip(single, pair):
        assert torch.equal(a, b)
