"""Attention on the B200 tcgen05 kernels and the reference-facing backend.

`H3AttentionBackendB200` is the drop-in for the model-local attention
backends the reference installs on each H3 attention module
(`attn._h3_attention_backend`, x_diffusers/x_diffusers/adaptor/
h3_cuda_precision.py:231-236): `H3SageCUDA` (x_base/x_base/operator/
h3_sage_cuda.py:6-25) for the Sage-FP8 recipe and `H3DenseCUDA`
(h3_dense_cuda.py:7-15) for BF16. Same call signature, same `calls` /
`kernel_calls` counters, same masked-call behaviour (a mask, dropout or an
unsupported head dim goes to PyTorch SDPA, as AttentionManager.attention
does at x_base/x_base/operator/attention.py:357-362).
"""
from __future__ import annotations

import math
import os

import torch
import torch.nn.functional as F

from . import _lib, trace
from ._lib import call, i64_array

HEAD_DIM = 128
_err_flags: dict[int, torch.Tensor] = {}


def _err_flag(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    flag = _err_flags.get(idx)
    if flag is None:
        flag = torch.zeros(1, dtype=torch.int32, device=device)
        _err_flags[idx] = flag
    return flag


_split_workspaces: dict[int, torch.Tensor] = {}


def _split_ws(device: torch.device) -> torch.Tensor:
    """Per-device workspace for the attention kernels' tail split (zeroed
    once; the kernels leave it reusable; launches on one device are
    stream-ordered through the caller's stream)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _split_workspaces.get(idx)
    if ws is None:
        ws = torch.zeros(_lib.lib().xgb_attention_split_workspace_bytes(), dtype=torch.uint8,
                         device=device)
        _split_workspaces[idx] = ws
    return ws


def kernel_errors(device: torch.device | None = None) -> int:
    """Non-zero if a tcgen05 kernel on `device` gave up on a bounded wait
    (synchronises the device)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    return int(_err_flag(device).item())


def _ws_args(device: torch.device):
    """Tail-split workspace arguments. XGB_ATTN_TAIL_SPLIT=0 passes none,
    which turns the split off: the Sage result then no longer depends on how
    many (batch, head) items a launch holds (split parts quantise P against
    their own running max), e.g. for bit-identical results across SP degrees."""
    if os.environ.get("XGB_ATTN_TAIL_SPLIT", "1") == "0":
        return None, 0
    ws = _split_ws(device)
    return ws.data_ptr(), ws.numel()


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _check_qkv(q, k, v, what: str):
    for t in (q, k, v):
        if not t.is_cuda:
            raise ValueError(f"{what} requires CUDA tensors")
        if t.ndim != 4 or t.shape[-1] != HEAD_DIM or t.stride(-1) != 1:
            raise ValueError(f"{what} requires [B, H, S, {HEAD_DIM}] views with unit channel stride")
    if q.shape[:2] != k.shape[:2] or k.shape != v.shape:
        raise ValueError(f"{what}: q/k/v batch, heads and k/v shapes must match")


class SageWorkspace:
    """Device buffers of one Sage quantisation (int8 Q/K, e4m3 V, scales)."""

    def __init__(self, batch: int, heads: int, seq: int, device: torch.device):
        self.shape = (batch, heads, seq)
        s_pad = (seq + 127) // 128 * 128
        bh = batch * heads
        self.s_pad = s_pad
        self.q8 = torch.empty((bh, s_pad, HEAD_DIM), dtype=torch.int8, device=device)
        self.k8 = torch.empty_like(self.q8)
        self.v8 = torch.empty((bh, s_pad, HEAD_DIM), dtype=torch.uint8, device=device)
        self.q_scale = torch.empty((bh, s_pad // 64), dtype=torch.float32, device=device)
        self.k_scale = torch.empty_like(self.q_scale)
        self.v_scale = torch.empty((bh, HEAD_DIM), dtype=torch.float32, device=device)
        nbytes = _lib.lib().xgb_sage_prepare_workspace(batch, heads, seq)
        self.scratch = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=device)
        self.scratch_bytes = nbytes


def sage_prepare(q, k, v, sm_scale: float | None = None, ws: SageWorkspace | None = None,
                 rotary_emb=None):
    """Sage quantisation of bf16/fp16 [B, H, S, 128] views: K mean-smoothing,
    per-64-token INT8 Q (sm_scale*log2e folded in) and K, per-channel e4m3 V.
    rotary_emb=(cos, sin) (fp32 [S, R], bf16 inputs): the rotate-half RoPE
    of Q and K is applied inside the same kernels (xgb_sage_prepare_rope)."""
    _check_qkv(q, k, v, "Sage attention")
    if q.shape != k.shape:
        raise ValueError("Sage attention expects self-attention shapes (Sq == Skv)")
    b, h, s, d = q.shape
    sm_scale = float(sm_scale) if sm_scale is not None else 1.0 / math.sqrt(d)
    if ws is None or ws.shape != (b, h, s):
        ws = SageWorkspace(b, h, s, q.device)
    dtype = {torch.bfloat16: _lib.XGB_BF16, torch.float16: _lib.XGB_F16}.get(q.dtype)
    if dtype is None or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("Sage attention requires bf16/fp16 inputs of one dtype")
    if rotary_emb is not None:
        cos, sin = rotary_emb
        if (q.dtype != torch.bfloat16 or cos.dtype != torch.float32 or sin.dtype != torch.float32
                or cos.shape != sin.shape or cos.ndim != 2 or cos.shape[0] != s or not cos.is_cuda
                or not cos.is_contiguous() or not sin.is_contiguous()):
            raise ValueError("fused Sage RoPE needs bf16 Q/K/V and contiguous fp32 cos/sin [S, R] on the GPU")
        call("xgb_sage_prepare_rope", q.data_ptr(), i64_array(q.stride()), k.data_ptr(),
             i64_array(k.stride()), v.data_ptr(), i64_array(v.stride()), b, h, s, d, sm_scale,
             cos.data_ptr(), sin.data_ptr(), cos.shape[1], ws.q8.data_ptr(), ws.q_scale.data_ptr(),
             ws.k8.data_ptr(), ws.k_scale.data_ptr(), ws.v8.data_ptr(), ws.v_scale.data_ptr(),
             ws.scratch.data_ptr(), ws.scratch_bytes, _err_flag(q.device).data_ptr(), _stream(q))
        return ws
    call("xgb_sage_prepare", q.data_ptr(), i64_array(q.stride()), k.data_ptr(),
         i64_array(k.stride()), v.data_ptr(), i64_array(v.stride()), dtype, b, h, s, d, sm_scale,
         ws.q8.data_ptr(), ws.q_scale.data_ptr(), ws.k8.data_ptr(), ws.k_scale.data_ptr(),
         ws.v8.data_ptr(), ws.v_scale.data_ptr(), ws.scratch.data_ptr(), ws.scratch_bytes,
         _err_flag(q.device).data_ptr(), _stream(q))
    return ws


def sage_prepare_wire(wire: torch.Tensor, *, peers: int, seq: int, batch: int, heads: int,
                      valid_seq: int, peer_padding: int = 0, sm_scale: float | None = None,
                      ws: SageWorkspace | None = None) -> SageWorkspace:
    """sage_prepare on Q/K/V read straight from a received PHAA FP8 wire
    (uint8, peer-major [Q|K|V] sections of rows [seq, batch, heads] per
    peer): the same outputs as decoding the wire into bf16 [batch, heads,
    valid_seq, 128] and calling sage_prepare, without the decode pass."""
    if wire.dtype != torch.uint8 or not wire.is_cuda or not wire.is_contiguous():
        raise ValueError("Sage wire preparation needs a contiguous CUDA uint8 wire")
    expect = peers * (3 * seq * batch * heads * (HEAD_DIM + 4) + peer_padding)
    if wire.numel() != expect:
        raise ValueError("PHAA FP8 wire size does not match its layout")
    sm_scale = float(sm_scale) if sm_scale is not None else 1.0 / math.sqrt(HEAD_DIM)
    if ws is None or ws.shape != (batch, heads, valid_seq):
        ws = SageWorkspace(batch, heads, valid_seq, wire.device)
    call("xgb_sage_prepare_wire", wire.data_ptr(), peers, seq, batch, heads, valid_seq, peer_padding,
         sm_scale, ws.q8.data_ptr(), ws.q_scale.data_ptr(), ws.k8.data_ptr(), ws.k_scale.data_ptr(),
         ws.v8.data_ptr(), ws.v_scale.data_ptr(), ws.scratch.data_ptr(), ws.scratch_bytes,
         _err_flag(wire.device).data_ptr(), torch.cuda.current_stream(wire.device).cuda_stream)
    return ws


def sage_attention_prepared(ws: SageWorkspace, out: torch.Tensor | None = None) -> torch.Tensor:
    """The tcgen05 INT8-QK / FP8-PV attention over a prepared workspace."""
    b, h, s = ws.shape
    if out is None:
        out = torch.empty((b, h, s, HEAD_DIM), dtype=torch.bfloat16, device=ws.q8.device)
    if out.shape != (b, h, s, HEAD_DIM) or out.dtype != torch.bfloat16 or out.stride(-1) != 1:
        raise ValueError("Sage attention output must be a bf16 [B, H, S, 128] view")
    call("xgb_attention_sage", ws.q8.data_ptr(), ws.q_scale.data_ptr(), ws.k8.data_ptr(),
         ws.k_scale.data_ptr(), ws.v8.data_ptr(), ws.v_scale.data_ptr(), b, h, s, out.data_ptr(),
         i64_array(out.stride()), *_ws_args(out.device), _err_flag(out.device).data_ptr(),
         _stream(out))
    return out


def sage_attention(q, k, v, sm_scale: float | None = None, out=None,
                   ws: SageWorkspace | None = None, rotary_emb=None) -> torch.Tensor:
    """Sage-style quantised attention of bf16 [B, H, S, 128] views (HND);
    rotary_emb: RoPE fused into the preparation (see sage_prepare)."""
    ws = sage_prepare(q, k, v, sm_scale, ws, rotary_emb=rotary_emb)
    return sage_attention_prepared(ws, out)


def dense_attention(q, k, v, sm_scale: float | None = None, out=None) -> torch.Tensor:
    """BF16 tcgen05 flash attention of [B, H, S, 128] views (any 16-byte
    aligned strides; TMA reads the views in place)."""
    _check_qkv(q, k, v, "BF16 attention")
    if q.dtype != torch.bfloat16 or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("BF16 attention requires bf16 inputs")
    b, h, sq, d = q.shape
    skv = k.shape[2]
    sm_scale = float(sm_scale) if sm_scale is not None else 1.0 / math.sqrt(d)
    if out is None:
        out = torch.empty((b, h, sq, d), dtype=torch.bfloat16, device=q.device)
    call("xgb_attention_bf16", q.data_ptr(), i64_array(q.stride()), k.data_ptr(),
         i64_array(k.stride()), v.data_ptr(), i64_array(v.stride()), b, h, sq, skv, sm_scale,
         out.data_ptr(), i64_array(out.stride()), *_ws_args(q.device), _err_flag(q.device).data_ptr(),
         _stream(q))
    return out


class H3AttentionBackendB200:
    """Model-local attention backend: `precision="sage"` (INT8 QK / FP8 PV,
    the H3SageCUDA slot) or `"bf16"` (the H3DenseCUDA slot)."""

    # run_phaa_attention may pass `out=` (a bf16 view of its send buffer)
    writes_into = True

    def __init__(self, precision: str = "sage"):
        if precision not in ("sage", "bf16"):
            raise ValueError(f"Unsupported H3 attention precision: {precision}")
        self.precision = precision
        self.calls = 0
        self.kernel_calls = 0
        self._ws = None

    def _kernel_eligible(self, query, key, value, attn_mask) -> bool:
        return (attn_mask is None and query.is_cuda and query.shape[-1] == HEAD_DIM
                and query.dtype in (torch.bfloat16, torch.float16)
                and (self.precision == "sage" or query.dtype == torch.bfloat16)
                and key.dtype == query.dtype and value.dtype == query.dtype
                and all(t.stride(-1) == 1 for t in (query, key, value))
                and (self.precision == "bf16" or query.shape == key.shape))

    def attend_fp8_wire(self, wire, *, peers, seq, batch, heads, valid_seq, peer_padding=0, out):
        """Sage attention on Q/K/V read straight from a received PHAA FP8
        wire (sage_prepare_wire): the same result as decoding the wire and
        calling this backend on [batch, heads, valid_seq, 128] views. out is
        a bf16 (batch, heads, valid_seq, 128) view."""
        if self.precision != "sage":
            raise ValueError("attention from the FP8 wire is the Sage path")
        key_ = ("wire", batch, heads, valid_seq, wire.device)
        if self._ws is None:
            self._ws = {}
        ws = sage_prepare_wire(wire, peers=peers, seq=seq, batch=batch, heads=heads, valid_seq=valid_seq,
                               peer_padding=peer_padding, ws=self._ws.get(key_))
        self._ws[key_] = ws
        trace.mark("prepared")
        sage_attention_prepared(ws, out)
        trace.mark("attended")
        self.kernel_calls += 1
        self.calls += 1
        return out

    def fuses_rope(self, query) -> bool:
        """Whether a call with `rotary_emb` applies the RoPE inside the Sage
        preparation (bf16 Sage) rather than as a pass of its own."""
        return self.precision == "sage" and query.dtype == torch.bfloat16

    def __call__(self, query, key, value, *, attn_mask=None, head_offset=0, out=None, rotary_emb=None):
        """B200 extension: `rotary_emb=(cos, sin)` (fp32 [S, R] over the
        sequence positions) rotates Q and K first, fused into the Sage
        preparation when `fuses_rope(query)`."""
        eligible = self._kernel_eligible(query, key, value, attn_mask) and (
            out is None or query.dtype == torch.bfloat16)
        if rotary_emb is not None and not (eligible and self.fuses_rope(query)):
            query, key = _rope_heads_major(query, key, rotary_emb)
        if eligible:
            if self.precision == "sage":
                b, h, s, _ = query.shape
                key_ = (b, h, s, query.device)
                if self._ws is None:
                    self._ws = {}
                if key_ not in self._ws:
                    self._ws[key_] = SageWorkspace(b, h, s, query.device)
                output = sage_attention(query, key, value, out=out, ws=self._ws[key_],
                                        rotary_emb=rotary_emb)
            else:
                output = dense_attention(query, key, value, out=out)
            self.kernel_calls += 1
            output = output.to(query.dtype) if output.dtype != query.dtype else output
        else:
            output = F.scaled_dot_product_attention(query, key, value, attn_mask=attn_mask)
            if out is not None:
                out.copy_(output)
                output = out
        self.calls += 1
        return output


def _rope_heads_major(query, key, rotary_emb):
    """Rotate-half RoPE of [B, H, S, D] Q/K views with the B200 kernel
    (which takes [B, S, H, D] rows)."""
    from .ops import try_h3_partial_rope

    q4 = query.transpose(1, 2).contiguous()
    k4 = key.transpose(1, 2).contiguous()
    with torch.no_grad():  # the kernels carry no autograd
        rotated = try_h3_partial_rope(q4, k4, *rotary_emb)
    if rotated is None:
        raise ValueError("H3 RoPE tables must be fp32 [S, R] with even R <= head_dim")
    return rotated[0].transpose(1, 2), rotated[1].transpose(1, 2)
