"""FP8 Linear on the B200 tcgen05 GEMM.

Mirror of H3FP8Linear (x_base/x_base/operator/h3_fp8.py:15-68): e4m3
weights with an fp32 scale, dynamic e4m3 activations, bf16 output with an
optional bias, the same construction checks (dimensions divisible by 16)
and forward checks (CUDA bf16/fp16 input of the right width). Two scaling
schemes:

  "per_tensor"  the reference's: one weight scale, one activation scale per
                call (abs-peak / 448, evaluated with CUDA semantics)
  "per_token"   B200 target: per-output-channel weight scales and per-token
                activation scales

`forward_gated` fuses the AdaLN gated residual that follows the attention and
FFN output projections (h3_indexed_affine.py:52-61) into the GEMM epilogue.
`swiglu_interleaved()` returns a copy of a gate-first SwiGLU up projection
whose rows are regrouped so that the GEMM epilogue applies the SwiGLU
(h3_swiglu.py:15-41) and writes only the [M, out/2] activation.
"""
from __future__ import annotations

import torch
from torch import nn

from . import _lib
from ._lib import call
from .ops import quantize_activation, quantize_per_token


def quantize_per_tensor(value: torch.Tensor):
    """(e4m3 tensor, fp32 scale) with scale = max(amax/448, FLT_MIN), as
    x_base/x_base/operator/h3_fp8.py:9-12 on the tensor's own device."""
    maximum = torch.finfo(torch.float8_e4m3fn).max
    scale = (value.float().abs().amax() / maximum).clamp_min(torch.finfo(torch.float32).tiny)
    return (value.float() / scale).clamp(-maximum, maximum).to(torch.float8_e4m3fn), scale


def quantize_per_channel(value: torch.Tensor):
    """Per-row (output channel) e4m3 of a [out, in] weight. The scale is an
    IEEE division by a tensor 448 (a Python-scalar divisor becomes a
    reciprocal multiply on CUDA tensors only), so the codes do not depend on
    the device the weight is quantised on."""
    maximum = torch.finfo(torch.float8_e4m3fn).max
    amax = value.float().abs().amax(dim=1)
    scale = (amax / torch.full_like(amax, maximum)).clamp_min(torch.finfo(torch.float32).tiny)
    return (value.float() / scale[:, None]).clamp(-maximum, maximum).to(torch.float8_e4m3fn), scale


class H3FP8Linear(nn.Module):
    """Keep FP8 weights; quantise activations to e4m3 on every call."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None = None,
                 scaling: str = "per_tensor"):
        super().__init__()
        if weight.ndim != 2 or weight.shape[0] % 16 or weight.shape[1] % 16:
            raise ValueError("H3 FP8 requires projection dimensions divisible by 16")
        if scaling not in ("per_tensor", "per_token"):
            raise ValueError(f"Unknown FP8 scaling: {scaling}")
        self.scaling = scaling
        self.out_features, self.in_features = weight.shape
        packed, scale = (quantize_per_tensor if scaling == "per_tensor" else quantize_per_channel)(
            weight.detach())
        self.register_buffer("weight", packed.contiguous())
        self.register_buffer("weight_scale", scale.reshape(-1).float())
        self.register_buffer("bias", bias.detach().clone().to(torch.bfloat16) if bias is not None else None)
        self.calls = 0
        self.swiglu = False

    @classmethod
    def from_packed(cls, weight, scale, bias=None):
        """Reuse quantised bytes and their scale (h3_fp8.py:26-39)."""
        if weight.dtype != torch.float8_e4m3fn or weight.ndim != 2 or any(n % 16 for n in weight.shape):
            raise ValueError("Packed H3 FP8 projection requires an aligned E4M3 matrix")
        if scale.numel() != 1 or scale.dtype != torch.float32:
            raise ValueError("Packed H3 FP8 projection requires one FP32 weight scale")
        result = cls.__new__(cls)
        nn.Module.__init__(result)
        result.scaling = "per_tensor"
        result.out_features, result.in_features = weight.shape
        result.register_buffer("weight", weight.contiguous())
        result.register_buffer("weight_scale", scale.detach().clone().reshape(1))
        result.register_buffer("bias", bias.detach().clone().to(torch.bfloat16) if bias is not None else None)
        result.calls = 0
        result.swiglu = False
        return result

    def swiglu_interleaved(self) -> "H3FP8Linear":
        """The same projection with rows regrouped per 128 as [gate j..j+127 |
        value j..j+127] (gate = the first out/2 rows), for the fused SwiGLU
        epilogue; its forward_quantized(..., activation=3) returns
        silu(gate) * value with the reference's bf16 rounding."""
        half = self.out_features // 2
        if self.out_features % 256:
            raise ValueError("fused SwiGLU needs out_features divisible by 256")
        order = torch.arange(self.out_features, device=self.weight.device).view(2, half // 128, 128)
        order = order.permute(1, 0, 2).reshape(-1)
        result = self.__class__.__new__(self.__class__)
        nn.Module.__init__(result)
        result.scaling = self.scaling
        result.out_features, result.in_features = self.out_features, self.in_features
        result.register_buffer("weight", self.weight.index_select(0, order).contiguous())
        scale = self.weight_scale
        result.register_buffer("weight_scale", scale.index_select(0, order) if scale.numel() > 1
                               else scale.clone())
        result.register_buffer("bias", self.bias.index_select(0, order)
                               if self.bias is not None else None)
        result.calls = 0
        result.swiglu = True
        return result

    def _check(self, x):
        if not x.is_cuda or x.dtype not in (torch.bfloat16, torch.float16):
            raise ValueError("H3 FP8 Linear requires CUDA BF16/FP16 input")
        if x.shape[-1] != self.in_features:
            raise ValueError("H3 FP8 Linear input width does not match its weight")

    def _quantize(self, matrix):
        if self.scaling == "per_tensor":
            q, s = quantize_activation(matrix, group=getattr(self, "activation_group", None))
            return q, s.reshape(1), 0
        q, s = quantize_per_token(matrix)
        return q, s, 1

    def forward(self, x):
        return self._forward(x, None)

    def forward_gated(self, x, gate_table, gate_index, residual):
        """residual + gate_table[gate_index] * self(x), each eager op rounded
        to bf16 (the block's `_apply(..., modulation=False)`), in one GEMM."""
        if (gate_table.dtype != torch.bfloat16 or gate_table.stride(-1) != 1
                or gate_table.shape[-1] != self.out_features or residual.dtype != torch.bfloat16
                or residual.shape[-1] != self.out_features or residual.stride(-1) != 1):
            raise ValueError("gated FP8 Linear needs bf16 gate rows [.., out] and a bf16 residual")
        return self._forward(x, (gate_table, gate_index, residual))

    def forward_quantized(self, q, scale, activation: int = 0, gated=None, out_shape=None):
        """GEMM on activations already quantised to e4m3 (q [M, in], scale
        [M] per token or [1] per tensor), e.g. by the fused norm/modulate/
        quant prologue. activation: 0 none, 1 GELU (erf), 2 GELU (tanh),
        3 gate-first SwiGLU (only on a `swiglu_interleaved()` projection;
        the result has out_features/2 columns)."""
        if q.dtype != torch.float8_e4m3fn or q.ndim != 2 or q.shape[1] != self.in_features:
            raise ValueError("pre-quantised FP8 Linear input must be e4m3 [M, in]")
        if (activation == 3) != self.swiglu:
            raise ValueError("the fused SwiGLU needs (and only fits) a swiglu_interleaved projection")
        m = q.shape[0]
        width = self.out_features // 2 if activation == 3 else self.out_features
        return self._gemm(q.contiguous(), scale.reshape(-1), 1 if scale.numel() > 1 else 0, m,
                          q.device, activation, gated, out_shape or (m, width))

    def _forward(self, x, gated):
        self._check(x)
        matrix = x.reshape(-1, self.in_features)
        m = matrix.shape[0]
        # A swiglu_interleaved projection always applies its SwiGLU.
        activation, width = (3, self.out_features // 2) if self.swiglu else (0, self.out_features)
        if gated is not None and self.swiglu:
            raise ValueError("the gated epilogue does not combine with the fused SwiGLU")
        if not m:
            return x.new_empty((*x.shape[:-1], width))
        matrix = matrix.contiguous()
        q, sa, sa_stride = self._quantize(matrix)
        out = self._gemm(q, sa, sa_stride, m, x.device, activation, gated, (*x.shape[:-1], width))
        return out if x.dtype == torch.bfloat16 else out.to(x.dtype)

    def _gemm(self, q, sa, sa_stride, m, device, activation, gated, out_shape):
        width = self.out_features // 2 if activation == 3 else self.out_features
        out = torch.empty((m, width), device=device, dtype=torch.bfloat16)
        gate = idx = res = None
        ldg = ldr = 0
        if gated is not None:
            gate, idx, res = gated
            res = res.reshape(-1, self.out_features)
            idx = idx.reshape(-1)
            if idx.numel() != m:  # indices over the sequence, broadcast over batch
                idx = idx.repeat(m // idx.numel())
            idx = idx.to(torch.int64).contiguous()
            ldg, ldr = gate.stride(0), res.stride(0)
        from .attention import _err_flag

        call("xgb_fp8_gemm", q.data_ptr(), self.weight.data_ptr(), m, self.out_features,
             self.in_features, sa.data_ptr(), sa_stride, self.weight_scale.data_ptr(),
             0 if self.weight_scale.numel() == 1 else 1,
             self.bias.data_ptr() if self.bias is not None else None, activation, out.data_ptr(),
             width, gate.data_ptr() if gate is not None else None, ldg,
             idx.data_ptr() if idx is not None else None,
             res.data_ptr() if res is not None else None, ldr, _err_flag(device).data_ptr(),
             torch.cuda.current_stream(device).cuda_stream)
        self.calls += 1
        return out.reshape(out_shape)


class H3FP8TPLinear(H3FP8Linear):
    """H3FP8Linear inside tensor parallelism, keeping the communication of
    the TP layer it replaces (x_base/x_base/operator/h3_fp8.py:71-108).

    A column-parallel layer holds a slice of the output features: it adds
    its bias locally and, with `gather_output`, all-gathers the slices along
    the feature axis. A row-parallel layer holds a slice of the input
    features: it takes its slice of a full input (when `input_is_parallel`
    is false), and its partial products are summed over the group (all-reduce,
    or the layer's `reduce_fn(output, group)`) before the bias is added once.

    The TP attributes are read from the replaced layer: `column_parallel`
    (else: is it a ColumnParallelLinear), `gather_output`,
    `input_is_parallel`, `tp_group`, `reduce_fn`. Without a `tp_group` the
    group registered by ParallelManager (xgen_b200.tp_state) is used, and
    the layer runs unsharded when none is. Set `activation_group` to share
    one activation scale over a group (MAX all-reduce before packing)."""

    _TP_ATTRIBUTES = (("gather_output", False), ("input_is_parallel", True), ("tp_group", None),
                      ("reduce_fn", None))

    def __init__(self, original, scaling: str = "per_tensor"):
        super().__init__(original.weight, getattr(original, "bias", None), scaling=scaling)
        declared = getattr(original, "column_parallel", None)
        self.column_parallel = (bool(declared) if declared is not None
                                else type(original).__name__ == "ColumnParallelLinear")
        for name, default in self._TP_ATTRIBUTES:
            setattr(self, name, getattr(original, name, default))

    def _gather_columns(self, output, group, world):
        import torch.distributed as dist

        slices = [torch.empty_like(output) for _ in range(world)]
        dist.all_gather(slices, output, group=group)
        return torch.cat(slices, dim=-1)

    def _reduce_rows(self, output, group):
        import torch.distributed as dist

        if self.reduce_fn is not None:
            return self.reduce_fn(output, group)
        dist.all_reduce(output, group=group)
        return output

    def forward(self, x):
        from . import tp_state

        group, world, rank = tp_state.resolve(self.tp_group)
        sharded = world > 1
        if self.column_parallel:
            output = self._forward(x, None)
            return self._gather_columns(output, group, world) if sharded and self.gather_output else output
        if sharded and not self.input_is_parallel:
            x = x.chunk(world, dim=-1)[rank]
        bias, self.bias = self.bias, None  # the row bias is added once, after the sum
        try:
            partial = self._forward(x, None)
        finally:
            self.bias = bias
        total = self._reduce_rows(partial, group) if sharded else partial
        return total if bias is None else total + bias
