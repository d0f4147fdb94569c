"""Asynchronous PHAA FP8 exchange with direct layouts, on the B200 codec.

Mirror of x_base/x_base/phaa/fp8_async_transport.py:84-193:
`submit_fp8_exchange` packs one tensor or a Q/K/V triple into the FP8 byte
wire (per row: e4m3 payload + fp32 scale, streams interleaved per peer, no
per-peer padding) on the current stream and enqueues an async NCCL
`all_to_all_single`; `finish_fp8_exchange` makes the consuming stream wait
for it and decodes. The direct layouts write and read the attention tensors
in place:

- direct gather: the decode writes Q/K/V straight into the attention input
  [batch, chunk_heads, valid_seq, D], dropping the sequence pad;
- fused return pack: the encode reads the attention output
  [batch, chunk_heads, valid_seq, D] and emits zero rows for the pad;
- direct return: the decode writes the returned chunk straight into the
  final [batch, seq, heads*D] output at the chunk's head offset.

`row_tiling` only changes the reference Triton kernels' rows per program;
the CUDA codec has one launch shape, so it is accepted and has no effect.
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
    decode_args: tuple


def submit_fp8_exchange(outputs, tensors, head_dim, group, *, row_tiling=False, return_shard_seq=0,
                        direct_gather=False, rotary_emb=None):
    """Pack and enqueue a collective on the active CUDA stream.

    B200 extension: `rotary_emb=(cos, sin)` applies the pre-A2A partial RoPE
    to Q and K inside the encode (QKV triples only)."""
    send, recv, decode_args = _pack_exchange(
        outputs, tensors, head_dim, group, row_tiling=row_tiling,
        return_shard_seq=return_shard_seq, direct_gather=direct_gather, rotary_emb=rotary_emb,
    )
    work = dist.all_to_all_single(recv, send, group=group, async_op=True)
    return PendingFP8Exchange(work, send, recv, outputs, decode_args)


def finish_fp8_exchange(pending, *, output=None, return_layout=()):
    """Wait on the consuming CUDA stream and unpack the received bytes.

    `return_layout` = (seq, batch, peers, heads_per_peer, chunk_heads,
    head_start) decodes a returned attention chunk into `output`
    [batch, seq, peers*heads_per_peer*D]."""
    stream = torch.cuda.current_stream(pending.recv.device)
    pending.work.block_current_stream()
    pending.send.record_stream(stream)
    pending.recv.record_stream(stream)
    outputs = (output,) if return_layout else pending.outputs
    _unpack_exchange(pending.recv, outputs, pending.decode_args, return_layout)


def _pack_exchange(outputs, tensors, head_dim, group, *, row_tiling=False, return_shard_seq=0,
                   direct_gather=False, rotary_emb=None):
    del row_tiling  # one launch shape on B200 (see module docstring)
    streams = len(tensors)
    if streams not in (1, 3) or (outputs is None and streams != 1):
        raise ValueError("PHAA FP8 transport expects one tensor or a QKV triple")
    if outputs is not None and len(outputs) != streams:
        raise ValueError("PHAA FP8 transport requires one output per input")
    shape = tensors[0].shape
    if head_dim % 4 or any(x.shape != shape for x in tensors):
        raise ValueError("PHAA FP8 transport requires matching shapes and head dim divisible by four")
    if direct_gather:
        if streams != 3 or len(shape) != 5 or shape[-1] != head_dim:
            raise ValueError("PHAA direct gather expects QKV head shards")
        peers, shard_seq, batches, chunk_heads, _ = shape
        valid_seq = outputs[0].shape[-2]
        expected = (batches, chunk_heads, valid_seq, head_dim)
        if not 0 < valid_seq <= peers * shard_seq or any(tuple(out.shape) != expected for out in outputs):
            raise ValueError("PHAA direct gather requires matching attention output shapes")
    elif outputs is not None and any(out.shape != shape for out in outputs):
        raise ValueError("PHAA FP8 transport requires matching input and output shapes")
    if outputs is not None and any(not out.is_contiguous() for out in outputs):
        raise ValueError("PHAA FP8 transport requires contiguous outputs")
    if any(t.device.type != "cuda" for t in tensors):
        raise ValueError("PHAA FP8 transport requires CUDA tensors")
    if any(t.dtype not in _DTYPE for t in tensors):
        raise ValueError("PHAA FP8 transport requires bf16/fp16 tensors")
    if rotary_emb is not None and (streams != 3 or return_shard_seq):
        raise ValueError("fused PHAA RoPE applies to a QKV gather only")
    peers = dist.get_world_size(group)
    rows = tensors[0].numel() // head_dim
    return_seq = 0
    if return_shard_seq:
        if outputs is not None or streams != 1 or len(shape) != 4 or shape[-1] != head_dim:
            raise ValueError("PHAA return pack expects an attention output and direct return")
        batches, chunk_heads, return_seq, _ = shape
        if not 0 < return_seq <= peers * return_shard_seq:
            raise ValueError("PHAA return pack received an invalid sequence length")
        rows = peers * return_shard_seq * batches * chunk_heads
    if rows % peers or tensors[0].numel() % head_dim:
        raise ValueError("PHAA FP8 rows must divide evenly among peers")
    peer_rows = rows // peers
    device = tensors[0].device
    send = torch.empty((streams * rows, head_dim + 4), dtype=torch.uint8, device=device)
    recv = torch.empty_like(send)
    if return_seq:
        # Attention output [batch, head, seq, D] read as [peer, shard_seq,
        # batch, head]: global sequence = peer * shard_seq + s.
        t = tensors[0]
        if t.stride(-1) != 1:
            t = t.contiguous()
        sb, sh, ss, _ = t.stride()
        views = [WireView(t.data_ptr(), (peers, return_shard_seq, batches, chunk_heads),
                          (return_shard_seq * ss, ss, sb, sh), t.dtype)]
        encode((t,), head_dim, peers, out=send, views=views, valid_seq=return_seq)
    else:
        sources = [_rows_view(t, peers, head_dim) for t in tensors]  # alive past the launch
        views = [WireView.of(t) for t in sources]
        encode(tensors, head_dim, peers, out=send, views=views, rotary_emb=rotary_emb)
    layout = views[0].shape
    return send, recv, (rows, streams, head_dim, peer_rows, layout, direct_gather)


def _unpack_exchange(recv, outputs, decode_args, return_layout=()):
    rows, streams, head_dim, peer_rows, layout, direct_gather = decode_args
    peers = rows // peer_rows
    dtype = outputs[0].dtype
    if return_layout:
        # Received rows: [source peer, seq, batch, chunk head] -> output
        # [batch, seq, peer, heads_per_peer, D] at head_start.
        seq, batches, peers_, heads_per_peer, chunk_heads, head_start = return_layout
        out = outputs[0]
        if out.stride(-1) != 1 or not out.is_contiguous():
            raise ValueError("PHAA direct return requires a contiguous output")
        hidden = out.shape[-1]
        elem = out.element_size()
        views = [WireView(out.data_ptr() + head_start * head_dim * elem,
                          (peers_, seq, batches, chunk_heads),
                          (heads_per_peer * head_dim, hidden, seq * hidden, head_dim), dtype)]
        decode_view(recv, views, head_dim)
    elif direct_gather:
        # Received rows: [source peer, shard seq, batch, chunk head] ->
        # attention input [batch, head, valid_seq, D], pad rows dropped.
        batches, chunk_heads, valid_seq, _ = outputs[0].shape
        shard_seq = layout[1]
        views = [WireView(o.data_ptr(), (peers, shard_seq, batches, chunk_heads),
                          (shard_seq * head_dim, head_dim, chunk_heads * valid_seq * head_dim,
                           valid_seq * head_dim), dtype) for o in outputs]
        decode_view(recv, views, head_dim, valid_seq=valid_seq)
    else:
        views = [WireView(o.data_ptr(), (peers, peer_rows, 1, 1),
                          (peer_rows * head_dim, head_dim, 0, 0), dtype) for o in outputs]
        decode_view(recv, views, head_dim)
