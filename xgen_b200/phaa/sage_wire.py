"""INT8 on the wire: Sage quantisation before the SP exchange, attention on
the exchanged bytes in place.

The reference moves bf16 (or its FP8 wire, per row e4m3 + fp32 scale) and
quantises for SageAttention after the A2A
(x_base/x_base/phaa/fp8_transport.py:85-144, attention.py:363-375). Here
every rank quantises its own rows once, as the attention kernel consumes
them, and the attention reads the received buffers without a decode or a
second quantisation pass:

1. `xgb_sage_wire_stats`: per (peer, batch, head) channel sums of RoPE'd K and
   abs-maxima of V over the local rows; all-reduced (SUM, MAX) over the SP
   group, which gives every rank the sequence-wide K mean and V scale.
2. `xgb_sage_wire_encode`: RoPE (bit-exact with the reference's partial
   RoPE), int8 Q/K per group of 16 tokens (S_loc is a multiple of 16, so
   groups never straddle ranks), e4m3 V per channel.
3. Four `all_to_all_single` calls (Q, K, V codes and the Q/K scales).
4. `xgb_attention_sage_strided` on the received [peer, S_loc, batch, head]
   rows, which for one (batch, head) are rows of one uniform stride.

Wire bytes per token and head: 3 x 128 + 8/16 (Q/K scales) = 384.5, against
3 x 132 for the FP8 wire. B200 extension; `run_phaa_attention(...,
int8_transport=True)` uses it for the gather.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from .. import _lib
from .._lib import call, i64_array

D = 128


def _views(t: torch.Tensor, heads: int, peers: int):
    """(B, S, heads*D) -> [peer, S, B, local head, D] view."""
    hl = heads // peers
    return t.unflatten(-1, (heads, D)).unflatten(2, (peers, hl)).permute(2, 1, 0, 3, 4)


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


class SageWire:
    """Send/receive buffers of one exchange shape, reusable across layers."""

    def __init__(self, peers: int, seq: int, batch: int, heads_local: int, device):
        shape = (peers, seq, batch, heads_local, D)
        self.shape = shape
        mk = lambda dt: torch.empty(shape, dtype=dt, device=device)  # noqa: E731
        self.q8, self.k8, self.v8 = mk(torch.int8), mk(torch.int8), mk(torch.uint8)
        self.q8r, self.k8r, self.v8r = mk(torch.int8), mk(torch.int8), mk(torch.uint8)
        sshape = (peers, seq // 16, batch, heads_local, 2)
        self.scales = torch.empty(sshape, dtype=torch.float32, device=device)
        self.scales_r = torch.empty(sshape, dtype=torch.float32, device=device)
        self.ksum = torch.empty((peers, batch, heads_local, D), dtype=torch.float32, device=device)
        self.vmax = torch.empty_like(self.ksum)
        self.v_scale = torch.empty_like(self.ksum)
        nbytes = _lib.lib().xgb_sage_wire_stats_workspace(peers, seq, batch, heads_local)
        self.stats_ws = torch.empty(max(nbytes, 4), dtype=torch.uint8, device=device)


def sage_wire_exchange(query, key, value, *, heads: int, group, peers: int, rotary_emb,
                       seq_real: int, sm_scale: float | None = None, bufs: SageWire | None = None,
                       exchange=None) -> SageWire:
    """Quantise this rank's (B, S_loc, heads*D) Q/K/V and exchange them:
    afterwards bufs.q8r/k8r/v8r/scales_r hold [source peer, S_loc, B, local
    head, ...] and bufs.v_scale[rank] the V scales of this rank's heads."""
    b, s, width = query.shape
    if width != heads * D or heads % peers or s % 16:
        raise ValueError("INT8 wire needs 128-wide heads divisible by SP and S_loc % 16 == 0")
    if any(t.dtype != torch.bfloat16 or not t.is_cuda for t in (query, key, value)):
        raise ValueError("INT8 wire needs CUDA bf16 Q/K/V")
    hl = heads // peers
    bufs = bufs or SageWire(peers, s, b, hl, query.device)
    if bufs.shape != (peers, s, b, hl, D):
        raise ValueError("INT8 wire buffers do not match the exchange shape")
    qv, kv, vv = (_views(t, heads, peers) for t in (query, key, value))
    cos = sin = None
    rotary = 0
    if rotary_emb is not None:
        cos, sin = rotary_emb
        rotary = cos.shape[-1]
    st = _stream(query)
    strides = lambda t: i64_array(t.stride()[:4])  # noqa: E731
    call("xgb_sage_wire_stats", kv.data_ptr(), strides(kv), vv.data_ptr(), strides(vv), peers, s, b,
         hl, cos.data_ptr() if cos is not None else None,
         sin.data_ptr() if sin is not None else None, rotary, bufs.ksum.data_ptr(),
         bufs.vmax.data_ptr(), bufs.stats_ws.data_ptr(), bufs.stats_ws.numel(), st)
    if peers > 1 or group is not None:
        dist.all_reduce(bufs.ksum, op=dist.ReduceOp.SUM, group=group)
        dist.all_reduce(bufs.vmax, op=dist.ReduceOp.MAX, group=group)
    scale = float(sm_scale) if sm_scale is not None else 1.0 / math.sqrt(D)
    call("xgb_sage_wire_encode", qv.data_ptr(), strides(qv), kv.data_ptr(), strides(kv),
         vv.data_ptr(), strides(vv), peers, s, b, hl,
         cos.data_ptr() if cos is not None else None,
         sin.data_ptr() if sin is not None else None, rotary, scale, bufs.ksum.data_ptr(),
         bufs.vmax.data_ptr(), seq_real, bufs.q8.data_ptr(), bufs.k8.data_ptr(),
         bufs.v8.data_ptr(), bufs.scales.data_ptr(), bufs.v_scale.data_ptr(), st)
    exchange = exchange or dist.all_to_all_single
    for recv, send in ((bufs.q8r, bufs.q8), (bufs.k8r, bufs.k8), (bufs.v8r, bufs.v8),
                       (bufs.scales_r, bufs.scales)):
        exchange(recv, send, group=group)
    return bufs


def sage_wire_attention(bufs: SageWire, out: torch.Tensor, seq_real: int, rank: int) -> torch.Tensor:
    """Attention over the received buffers; out is a (B, local heads,
    seq_real, D) bf16 view (e.g. of the return-A2A send buffer)."""
    from ..attention import _err_flag, _ws_args

    peers, s, b, hl, _ = bufs.shape
    if tuple(out.shape) != (b, hl, seq_real, D) or out.dtype != torch.bfloat16 or out.stride(-1) != 1:
        raise ValueError("INT8 wire attention output must be a (B, heads, S, 128) bf16 view")
    row = b * hl * D  # bytes between consecutive sequence rows of one (batch, head)
    qkv_strides = i64_array([hl * D, D, row])
    g = b * hl * 2   # scale elements between consecutive 16-row groups
    vs = bufs.v_scale[rank]
    call("xgb_attention_sage_strided", bufs.q8r.data_ptr(), qkv_strides, bufs.scales_r.data_ptr(),
         i64_array([hl * 2, 2, g]), bufs.k8r.data_ptr(), qkv_strides,
         bufs.scales_r.data_ptr() + 4, i64_array([hl * 2, 2, g]), bufs.v8r.data_ptr(), qkv_strides,
         vs.data_ptr(), i64_array([hl * D, D]), b, hl, seq_real, peers * s, out.data_ptr(),
         i64_array(out.stride()), *_ws_args(out.device), _err_flag(out.device).data_ptr(),
         _stream(out))
    return out
