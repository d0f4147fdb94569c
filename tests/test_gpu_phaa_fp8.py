"""PHAA layouts and CUDA streams on one GPU with a simulated 2-rank SP
collective, as the reference's own tests do it
(x_base/tests/test_phaa_fp8.py:11-143): the collective is a local copy, so
every exchange variant must reproduce the same bytes and the same output.
The wire codec, the direct layouts and the attention are this library's
CUDA kernels."""
from unittest.mock import patch

import pytest
import torch
import torch.distributed as dist
import torch.nn.functional as F

from xgen_b200.sp.padding import get_pad_manager

pytestmark = pytest.mark.gpu


@pytest.fixture
def pad_one():
    # phaa_attention.get_pad patched to 1 in the reference tests.
    get_pad_manager()._pads["pad"] = 1
    yield
    get_pad_manager().clear()


def _local_copy(output, tensor, **kwargs):
    output.copy_(tensor)


class _Async:
    """all_to_all_single stand-in: sync calls copy in place, async calls copy
    on a collective stream and return a work whose block_current_stream
    makes the caller's stream wait (test_phaa_fp8.py:85-104)."""

    def __init__(self):
        self.stream = torch.cuda.Stream()

    def __call__(self, output, tensor, **kwargs):
        if not kwargs.get("async_op"):
            output.copy_(tensor)
            return None
        self.stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):
            output.copy_(tensor)
            done = self.stream.record_event()

        class Work:
            def block_current_stream(self_inner):
                torch.cuda.current_stream().wait_event(done)

        return Work()


@pytest.mark.parametrize("batch_size", [1, 2])
def test_fp8_phaa_uneven_heads_and_padding(cuda_device, pad_one, batch_size):
    from xgen_b200.phaa import phaa_attention

    g = torch.Generator(device=cuda_device).manual_seed(42)
    qkv = [torch.randn((batch_size, 32, 14 * 64), dtype=torch.bfloat16, device=cuda_device,
                       generator=g) for _ in range(3)]

    def attention(q, k, v, **kwargs):
        return F.scaled_dot_product_attention(q, k, v)

    options = dict(comm_stream=torch.cuda.Stream(), sp_group=None, sp_size=2,
                   heads=14, phaa_split_num=2, head_dim=64, attention_fn=attention)
    with patch.object(dist, "get_world_size", return_value=2), \
         patch.object(dist, "all_to_all_single", side_effect=_local_copy) as exchange:
        dense = phaa_attention.run_phaa_attention(*qkv, **options)
        assert exchange.call_count == 8
        exchange.reset_mock()
        fp8 = phaa_attention.run_phaa_attention(*qkv, **options, fp8_transport=True)
        assert exchange.call_count == 4
        exchange.reset_mock()
        gather_first = phaa_attention.run_phaa_attention(*qkv, **options, fp8_transport=True,
                                                         gather_priority=True)
        assert exchange.call_count == 4
        exchange.reset_mock()
        scatter_group = object()
        dual = phaa_attention.run_phaa_attention(*qkv, **options, fp8_transport=True,
                                                 scatter_group=scatter_group,
                                                 scatter_stream=torch.cuda.Stream())
        assert [c.kwargs["group"] for c in exchange.call_args_list] == [
            None, None, scatter_group, scatter_group]
    for c in exchange.call_args_list[-2:]:
        received, sent = c.args
        assert received.dtype == sent.dtype == torch.uint8
        assert received.shape == sent.shape
        assert sent.shape[-1] == 64 + 4  # e4m3 row and fp32 scale
    torch.cuda.synchronize()
    assert dense.shape == fp8.shape == qkv[0].shape
    assert dense.dtype == fp8.dtype == qkv[0].dtype
    assert torch.isfinite(fp8).all()
    assert torch.equal(fp8, gather_first)
    assert torch.equal(fp8, dual)
    assert F.cosine_similarity(dense.float().flatten(), fp8.float().flatten(), dim=0) > 0.99


def _run_variants(qkv, attention, head_dim, heads, device):
    from xgen_b200.phaa import phaa_attention
    from xgen_b200.phaa.fp8_async_transport import AsyncFP8Options

    offsets = []

    def recording(q, k, v, *, head_offset, attn_mask, **kw):
        offsets.append(head_offset)
        return attention(q, k, v, head_offset=head_offset, attn_mask=attn_mask, **kw)

    recording.writes_into = getattr(attention, "writes_into", False)
    options = dict(comm_stream=torch.cuda.Stream(), sp_group=None, sp_size=2, heads=heads,
                   phaa_split_num=4, head_dim=head_dim, attention_fn=recording,
                   fp8_transport=True, gather_priority=True)
    fake = _Async()
    results = {}
    with patch.object(dist, "get_world_size", return_value=2), \
         patch.object(dist, "all_to_all_single", side_effect=fake) as exchange:
        results["natural"] = phaa_attention.run_phaa_attention(*qkv, **options)
        natural_shapes = [c.args[0].shape for c in exchange.call_args_list]
        results["natural_offsets"] = list(offsets)
        offsets.clear()
        results["tail"] = phaa_attention.run_phaa_attention(*qkv, **options, tail_first=True)
        results["tail_offsets"] = list(offsets)
        offsets.clear()
        exchange.reset_mock()
        results["async"] = phaa_attention.run_phaa_attention(
            *qkv, **options, device_join=True, async_options=AsyncFP8Options())
        results["async_offsets"] = list(offsets)
        assert [c.args[0].shape for c in exchange.call_args_list] == natural_shapes
        assert all(c.kwargs.get("async_op") is True for c in exchange.call_args_list)
        for name, opts in (
                ("direct", AsyncFP8Options(direct_return=True)),
                ("tiled", AsyncFP8Options(direct_return=True, row_tiling=True)),
                ("packed", AsyncFP8Options(direct_return=True, row_tiling=True,
                                           fused_return_pack=True)),
                ("direct_qkv", AsyncFP8Options(direct_return=True, row_tiling=True,
                                               direct_gather=True)),
                ("all_direct", AsyncFP8Options(direct_return=True, fused_return_pack=True,
                                               direct_gather=True))):
            results[name] = phaa_attention.run_phaa_attention(
                *qkv, **options, tail_first=True, device_join=True, async_options=opts)
    torch.cuda.synchronize()
    return results


def test_fp8_phaa_c4_tail_first_preserves_head_order(cuda_device, pad_one):
    g = torch.Generator(device=cuda_device).manual_seed(42)
    qkv = [torch.randn((1, 32, 14 * 64), dtype=torch.bfloat16, device=cuda_device, generator=g)
           for _ in range(3)]

    def attention(q, k, v, *, head_offset, attn_mask):
        return F.scaled_dot_product_attention(q, k, v, attn_mask=attn_mask)

    r = _run_variants(qkv, attention, 64, 14, cuda_device)
    assert r["natural_offsets"] == [0, 2, 4, 6]
    assert r["tail_offsets"] == [6, 0, 2, 4]
    assert r["async_offsets"] == [0, 2, 4, 6]
    for name in ("tail", "async", "direct", "tiled", "packed", "direct_qkv", "all_direct"):
        assert torch.equal(r["natural"], r[name]), name


def test_async_variants_with_b200_attention(cuda_device):
    """The same variants through this library's attention backend (D=128,
    its writes-into fast path for the natural order), sequence 301 per rank
    (pad 1 at SP2) so every KV tile edge and the pad row are exercised."""
    from xgen_b200.attention import H3AttentionBackendB200

    get_pad_manager()._pads["pad"] = 1
    try:
        g = torch.Generator(device=cuda_device).manual_seed(7)
        qkv = [torch.randn((1, 301, 8 * 128), dtype=torch.bfloat16, device=cuda_device,
                           generator=g) for _ in range(3)]
        backend = H3AttentionBackendB200("bf16")
        r = _run_variants(qkv, backend, 128, 8, cuda_device)
    finally:
        get_pad_manager().clear()
    for name in ("tail", "async", "direct", "tiled", "packed", "direct_qkv", "all_direct"):
        assert torch.equal(r["natural"], r[name]), name
    assert backend.kernel_calls > 0


@pytest.mark.parametrize("fuse_rope", [False, True])
def test_sage_from_wire_matches_decode_path(cuda_device, fuse_rope):
    """With a Sage backend, PHAA prepares Q/K/V straight from the received
    FP8 wire (sage_prepare_wire): bit-identical to decoding the wire into
    bf16 gather buffers and calling the same backend on them, with the SP
    pad row and (optionally) the fused pre-A2A RoPE."""
    from xgen_b200.attention import H3AttentionBackendB200
    from xgen_b200.phaa import phaa_attention

    backend = H3AttentionBackendB200("sage")

    class ViaDecode:  # hides `precision`: PHAA decodes into gather buffers
        writes_into = True

        def __call__(self, q, k, v, **kw):
            return backend(q, k, v, **kw)

    g = torch.Generator(device=cuda_device).manual_seed(21)
    qkv = [torch.randn((1, 301, 8 * 128), dtype=torch.bfloat16, device=cuda_device, generator=g)
           for _ in range(3)]
    ang = torch.rand(301, 48, device=cuda_device, generator=g) * 3
    rot = (torch.cat([ang.cos(), ang.cos()], -1).float().contiguous(),
           torch.cat([ang.sin(), ang.sin()], -1).float().contiguous())
    options = dict(comm_stream=torch.cuda.Stream(), sp_group=None, sp_size=2, heads=8,
                   phaa_split_num=2, head_dim=128, fp8_transport=True,
                   rotary_emb=rot if fuse_rope else None, fuse_rope=fuse_rope)
    get_pad_manager()._pads["pad"] = 1
    try:
        with patch.object(dist, "get_world_size", return_value=2), \
             patch.object(dist, "all_to_all_single", side_effect=_Async()):
            before = backend.kernel_calls
            wire = phaa_attention.run_phaa_attention(*qkv, attention_fn=backend, **options)
            assert backend.kernel_calls - before == 2
            decoded = phaa_attention.run_phaa_attention(*qkv, attention_fn=ViaDecode(), **options)
        torch.cuda.synchronize()
    finally:
        get_pad_manager().clear()
    assert torch.equal(wire, decoded)


def test_sage_fp16_activations_take_the_decode_path(cuda_device):
    """fp16 activations with the FP8 wire and a Sage backend: the wire
    decode rounds to fp16 (the reference's _decode writes the destination
    dtype), so PHAA must not hand the wire to the bf16-only wire preparation;
    it decodes into fp16 gather buffers and calls the backend on them."""
    from xgen_b200.attention import H3AttentionBackendB200
    from xgen_b200.phaa import phaa_attention

    backend = H3AttentionBackendB200("sage")

    class ViaDecode:
        writes_into = True

        def __call__(self, q, k, v, **kw):
            return backend(q, k, v, **kw)

    g = torch.Generator(device=cuda_device).manual_seed(23)
    qkv = [torch.randn((1, 256, 4 * 128), device=cuda_device, generator=g).half() for _ in range(3)]
    options = dict(comm_stream=torch.cuda.Stream(), sp_group=None, sp_size=2, heads=4,
                   phaa_split_num=1, head_dim=128, fp8_transport=True)

    def refuse(*args, **kwargs):
        raise AssertionError("the wire preparation must not see fp16 activations")

    with patch.object(dist, "get_world_size", return_value=2), \
         patch.object(dist, "all_to_all_single", side_effect=_local_copy), \
         patch.object(backend, "attend_fp8_wire", side_effect=refuse):
        got = phaa_attention.run_phaa_attention(*qkv, attention_fn=backend, **options)
        expect = phaa_attention.run_phaa_attention(*qkv, attention_fn=ViaDecode(), **options)
    torch.cuda.synchronize()
    assert got.dtype == torch.float16 and torch.isfinite(got.float()).all()
    assert torch.equal(got, expect)
