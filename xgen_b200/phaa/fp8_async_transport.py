"""Asynchronous PHAA FP8 exchange with direct layouts, on the B200 codec.

Same public surface as x_base/x_base/phaa/fp8_async_transport.py:84-193
(`AsyncFP8Options`, `PendingFP8Exchange`, `submit_fp8_exchange`,
`finish_fp8_exchange`): one tensor or a Q/K/V triple goes over the FP8 byte
wire (per row: e4m3 payload + fp32 scale, streams interleaved per peer, no
per-peer padding) with an async NCCL `all_to_all_single` enqueued on the
current stream; finishing makes the consuming stream wait for it and
decodes.

Every request is first turned into an `_ExchangePlan`: its kind, the
[peer, seq, batch, head] row layout the encoder reads, and how the decoder
addresses the destination. The kinds:

  gather         Q/K/V head shards -> same-shaped gather buffers
  direct_gather  Q/K/V head shards -> the attention input [B, heads, valid_seq, D]
                 (pad rows of the last peer dropped)
  return         one attention result -> a same-shaped buffer, or (with a
                 `return_layout` at finish) the final [B, seq, heads*D] output
                 at the chunk's head offset
  fused_return   the attention output [B, heads, valid_seq, D] read as it is
                 (pad rows sent as zeros), decoded like `return`

`row_tiling` only changes the reference Triton kernels' rows per program;
the CUDA codec has one launch shape, so it is accepted and has no effect.
B200 extension: `rotary_emb=(cos, sin)` applies the pre-A2A partial RoPE to
Q and K inside the encode of a gather.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import NamedTuple

import torch
import torch.distributed as dist

from .fp8_transport import WireView, _DTYPE, _rows_view, decode_view, encode


@dataclass(frozen=True)
class AsyncFP8Options:
    direct_return: bool = False
    row_tiling: bool = False
    fused_return_pack: bool = False
    direct_gather: bool = False

    def __post_init__(self):
        if self.fused_return_pack and not self.direct_return:
            raise ValueError("PHAA fused return pack requires direct return")


class PendingFP8Exchange(NamedTuple):
    work: object
    send: torch.Tensor
    recv: torch.Tensor
    outputs: tuple | None
    decode_args: "_ExchangePlan"


@dataclass
class _ExchangePlan:
    kind: str
    streams: int
    head_dim: int
    peers: int
    rows: int            # wire rows per stream
    layout: tuple        # [peer, seq, batch, head] of the rows on the wire
    valid_seq: int       # global sequence rows that carry data (direct gather)

    @property
    def wire_shape(self):
        return (self.streams * self.rows, self.head_dim + 4)


def _fail(message: str):
    raise ValueError(message)


def _plan(outputs, tensors, head_dim, peers, return_shard_seq, direct_gather) -> _ExchangePlan:
    streams = len(tensors)
    if streams not in (1, 3) or (outputs is None and streams == 3):
        _fail("PHAA FP8 transport expects one tensor or a QKV triple")
    if outputs is not None and len(outputs) != streams:
        _fail("PHAA FP8 transport requires one output per input")
    shape = tuple(tensors[0].shape)
    if head_dim % 4 or any(tuple(t.shape) != shape for t in tensors):
        _fail("PHAA FP8 transport requires matching shapes and head dim divisible by four")
    if any(t.device.type != "cuda" for t in tensors):
        _fail("PHAA FP8 transport requires CUDA tensors")
    if any(t.dtype not in _DTYPE for t in tensors):
        _fail("PHAA FP8 transport requires bf16/fp16 tensors")
    if outputs is not None and not all(o.is_contiguous() for o in outputs):
        _fail("PHAA FP8 transport requires contiguous outputs")

    if return_shard_seq:
        # the attention output [batch, heads, valid_seq, D], read in place
        if outputs is not None or streams != 1 or len(shape) != 4 or shape[-1] != head_dim:
            _fail("PHAA return pack expects an attention output and direct return")
        batch, heads, valid_seq, _ = shape
        if not 0 < valid_seq <= peers * return_shard_seq:
            _fail("PHAA return pack received an invalid sequence length")
        layout = (peers, return_shard_seq, batch, heads)
        return _ExchangePlan("fused_return", 1, head_dim, peers, peers * return_shard_seq * batch * heads,
                             layout, valid_seq)

    rows, ragged = divmod(tensors[0].numel(), head_dim)
    if ragged or rows % peers:
        _fail("PHAA FP8 rows must divide evenly among peers")
    if direct_gather:
        if streams != 3 or len(shape) != 5 or shape[-1] != head_dim:
            _fail("PHAA direct gather expects QKV head shards")
        _, shard_seq, batch, heads, _ = shape
        valid_seq = outputs[0].shape[-2]
        if not 0 < valid_seq <= peers * shard_seq or any(
                tuple(o.shape) != (batch, heads, valid_seq, head_dim) for o in outputs):
            _fail("PHAA direct gather requires matching attention output shapes")
        return _ExchangePlan("direct_gather", 3, head_dim, peers, rows, shape[:4], valid_seq)
    if outputs is not None and any(tuple(o.shape) != shape for o in outputs):
        _fail("PHAA FP8 transport requires matching input and output shapes")
    return _ExchangePlan("gather" if streams == 3 else "return", streams, head_dim, peers, rows, (), 0)


def submit_fp8_exchange(outputs, tensors, head_dim, group, *, row_tiling=False, return_shard_seq=0,
                        direct_gather=False, rotary_emb=None):
    """Encode on the active CUDA stream and enqueue the async all-to-all."""
    del row_tiling  # one launch shape on B200
    plan = _plan(outputs, tensors, head_dim, dist.get_world_size(group), return_shard_seq, direct_gather)
    if rotary_emb is not None and plan.kind not in ("gather", "direct_gather"):
        _fail("fused PHAA RoPE applies to a QKV gather only")
    device = tensors[0].device
    send = torch.empty(plan.wire_shape, dtype=torch.uint8, device=device)
    if plan.kind == "fused_return":
        t = tensors[0]
        sb, sh, ss, _ = t.stride()
        view = WireView(t.data_ptr(), plan.layout, (plan.layout[1] * ss, ss, sb, sh), t.dtype)
        encode((t,), head_dim, plan.peers, out=send, views=[view], valid_seq=plan.valid_seq)
    else:
        shaped = [_rows_view(t, plan.peers, head_dim) for t in tensors]  # kept alive past the launch
        views = [WireView.of(t) for t in shaped]
        plan.layout = views[0].shape
        encode(tensors, head_dim, plan.peers, out=send, views=views, rotary_emb=rotary_emb)
    recv = torch.empty_like(send)
    work = dist.all_to_all_single(recv, send, group=group, async_op=True)
    return PendingFP8Exchange(work, send, recv, outputs, plan)


def finish_fp8_exchange(pending, *, output=None, return_layout=()):
    """Make the consuming stream wait for the exchange, then decode.

    `return_layout` = (seq, batch, peers, heads_per_peer, chunk_heads,
    head_start) decodes a returned attention chunk into `output`
    [batch, seq, peers*heads_per_peer*D] at head `head_start`."""
    stream = torch.cuda.current_stream(pending.recv.device)
    pending.work.block_current_stream()
    for buf in (pending.send, pending.recv):
        buf.record_stream(stream)
    plan = pending.decode_args
    d = plan.head_dim
    if return_layout:
        seq, batch, peers, heads_per_peer, chunk_heads, head_start = return_layout
        if output.stride(-1) != 1 or not output.is_contiguous():
            _fail("PHAA direct return requires a contiguous output")
        hidden = output.shape[-1]
        base = output.data_ptr() + head_start * d * output.element_size()
        # wire rows [source peer, seq, batch, chunk head] -> output[b, s, peer, head]
        views = [WireView(base, (peers, seq, batch, chunk_heads),
                          (heads_per_peer * d, hidden, seq * hidden, d), output.dtype)]
        decode_view(pending.recv, views, d)
        return
    outputs = pending.outputs
    if plan.kind == "direct_gather":
        _, shard_seq, batch, heads = plan.layout
        valid = plan.valid_seq
        # wire rows [source peer, shard seq, batch, head] -> out[b, head, peer*shard_seq + s]
        views = [WireView(o.data_ptr(), (plan.peers, shard_seq, batch, heads),
                          (shard_seq * d, d, heads * valid * d, valid * d), o.dtype) for o in outputs]
        decode_view(pending.recv, views, d, valid_seq=valid)
        return
    per_peer = plan.rows // plan.peers
    views = [WireView(o.data_ptr(), (plan.peers, per_peer, 1, 1), (per_peer * d, d, 0, 0), o.dtype)
             for o in outputs]
    decode_view(pending.recv, views, d)
