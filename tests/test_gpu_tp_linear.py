"""FP8 Linear under tensor parallelism (x_base/x_base/operator/h3_fp8.py
:71-108, h3_fp8_quant.py:18-25) on one GPU: the collectives are stand-ins
that supply the other rank's contribution, so each rank's arithmetic is
checked exactly against the composition it must equal."""
from types import SimpleNamespace
from unittest.mock import patch

import pytest
import torch
import torch.distributed as dist

pytestmark = pytest.mark.gpu

_GROUP = object()  # an explicit TP group; every collective on it is patched below


def test_group_scale_quantisation(cuda_device):
    from xgen_b200.ops import quantize_activation

    g = torch.Generator().manual_seed(3)
    x = torch.randn(257, 96, generator=g).bfloat16().to(cuda_device)
    peer_scale = torch.tensor(10.0 / 448.0, device=cuda_device)  # the other rank's larger peak

    def max_reduce(t, op=None, group=None):
        assert op == dist.ReduceOp.MAX
        t.copy_(torch.maximum(t, peer_scale))

    with patch.object(dist, "all_reduce", side_effect=max_reduce) as ar:
        q, s = quantize_activation(x, group=object())
        assert ar.call_count == 1
    assert torch.equal(s, peer_scale)
    expect = (x.float().cpu() / s.cpu()).clamp(-448, 448).to(torch.float8_e4m3fn)
    assert torch.equal(q.cpu().view(torch.uint8), expect.view(torch.uint8))
    # without a group it is the ordinary per-tensor quantiser
    q1, s1 = quantize_activation(x)
    q2, s2 = quantize_activation(x, group=None)
    assert torch.equal(q1.view(torch.uint8), q2.view(torch.uint8)) and torch.equal(s1, s2)


def _shards(cuda_device, n=256, k=512, seed=7):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(n, k, generator=g) * 0.05).bfloat16()
    b = torch.randn(n, generator=g).bfloat16()
    x = torch.randn(3, 40, k, generator=g).bfloat16().to(cuda_device)
    return w, b, x


def test_column_parallel_gather(cuda_device):
    from xgen_b200.fp8_linear import H3FP8Linear, H3FP8TPLinear

    w, b, x = _shards(cuda_device)
    w0, w1 = w.chunk(2, dim=0)
    b0, b1 = b.chunk(2)
    ref1 = H3FP8Linear(w1, b1).to(cuda_device)(x)  # rank 1's local output
    layer = H3FP8TPLinear(SimpleNamespace(weight=w0, bias=b0, column_parallel=True,
                                          gather_output=True, tp_group=_GROUP)).to(cuda_device)

    def gather(values, output, group=None):
        values[0].copy_(output)
        values[1].copy_(ref1)

    with patch.object(dist, "is_initialized", return_value=True), \
         patch.object(dist, "get_world_size", return_value=2), \
         patch.object(dist, "get_rank", return_value=0), \
         patch.object(dist, "all_gather", side_effect=gather):
        out = layer(x)
    ref0 = H3FP8Linear(w0, b0).to(cuda_device)(x)
    assert torch.equal(out, torch.cat([ref0, ref1], dim=-1))


def test_row_parallel_slices_reduces_and_adds_bias_after(cuda_device):
    from xgen_b200.fp8_linear import H3FP8Linear, H3FP8TPLinear
    from xgen_b200.ops import quantize_activation

    w, b, x = _shards(cuda_device, seed=9)
    w0, w1 = w.chunk(2, dim=1)
    x0, x1 = x.chunk(2, dim=-1)
    # the group scale: MAX over the two input shards
    _, s0 = quantize_activation(x0.reshape(-1, x0.shape[-1]))
    _, s1 = quantize_activation(x1.reshape(-1, x1.shape[-1]))
    shared = torch.maximum(s0, s1)
    # rank 1's partial product with the shared scale
    other = H3FP8Linear(w1).to(cuda_device)
    other.activation_group = object()
    with patch.object(dist, "all_reduce", side_effect=lambda t, op=None, group=None: t.copy_(shared)):
        part1 = other(x1)

    layer = H3FP8TPLinear(SimpleNamespace(weight=w0, bias=b, column_parallel=False,
                                          input_is_parallel=False, tp_group=_GROUP)).to(cuda_device)
    layer.activation_group = object()
    calls = []

    def reduce(t, op=dist.ReduceOp.SUM, group=None):
        calls.append(op)
        if op == dist.ReduceOp.MAX:
            t.copy_(shared)
        else:  # the output sum
            t.add_(part1)

    with patch.object(dist, "is_initialized", return_value=True), \
         patch.object(dist, "get_world_size", return_value=2), \
         patch.object(dist, "get_rank", return_value=0), \
         patch.object(dist, "all_reduce", side_effect=reduce):
        out = layer(x)
    assert calls == [dist.ReduceOp.MAX, dist.ReduceOp.SUM]
    own = H3FP8Linear(w0).to(cuda_device)
    own.activation_group = object()
    with patch.object(dist, "all_reduce", side_effect=lambda t, op=None, group=None: t.copy_(shared)):
        part0 = own(x0)
    assert torch.equal(out, (part0 + part1) + b.to(cuda_device))


def test_group_falls_back_to_registered_tp_state(cuda_device):
    """tp_group None: the layer uses the group ParallelManager registered, and
    with none registered it runs unsharded without a collective
    (x_base/x_base/tensor_parallelism/layers.py:17-27)."""
    from xgen_b200 import tp_state
    from xgen_b200.fp8_linear import H3FP8Linear, H3FP8TPLinear

    w, b, x = _shards(cuda_device, seed=5)
    w0, w1 = w.chunk(2, dim=0)
    b0, b1 = b.chunk(2)
    ref0 = H3FP8Linear(w0, b0).to(cuda_device)(x)
    ref1 = H3FP8Linear(w1, b1).to(cuda_device)(x)
    layer = H3FP8TPLinear(SimpleNamespace(weight=w0, bias=b0, column_parallel=True,
                                          gather_output=True, tp_group=None)).to(cuda_device)
    seen = []

    def gather(values, output, group=None):
        seen.append(group)
        values[0].copy_(output)
        values[1].copy_(ref1)

    with patch.object(dist, "all_gather", side_effect=gather):
        assert torch.equal(layer(x), ref0) and not seen  # nothing registered
        tp_state.set_tp_group(_GROUP, 2, 0)
        try:
            out = layer(x)
        finally:
            tp_state.clear_tp_group()
    assert seen == [_GROUP]
    assert torch.equal(out, torch.cat([ref0, ref1], dim=-1))
