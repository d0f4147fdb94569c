"""PHAA FP8 wire transport on the B200 kernels.

Mirrors x_base/x_base/phaa/fp8_transport.py: `fp8_all_to_all_many(outputs,
tensors, head_dim, group)` encodes one tensor or a Q/K/V triple into one byte
buffer (per row of `head_dim` channels: e4m3 payload + fp32 scale, streams
interleaved per peer, optional Align16 per-peer padding), exchanges it with a
single NCCL `all_to_all_single`, and decodes into the outputs. The encode
kernel reads any [peer, seq, batch, head, head_dim] view with unit channel
stride directly (the reference needs XGEN_PHAA_FP8_MIXED_STRIDES=1 for mixed
strides and otherwise copies), and can fuse the pre-A2A partial RoPE of
Q and K (`rotary_emb`), which the reference runs as a separate kernel.
"""
from __future__ import annotations

import logging
import os
from typing import NamedTuple

import torch
import torch.distributed as dist

from .. import _lib
from .._lib import call, i64_array, ptr_array

_mixed_stride_metrics = dict(calls=0, avoided_contiguous_bytes=0)
_peer_alignment_metrics = dict(calls=0, padded_calls=0, padding_bytes=0)
_DTYPE = {torch.bfloat16: _lib.XGB_BF16, torch.float16: _lib.XGB_F16}


def mixed_stride_metrics():
    """Scalar diagnostics, as the reference's (fp8_transport.py:16-18)."""
    return dict(_mixed_stride_metrics)


def peer_alignment_metrics():
    """Align16 counters, as the reference's (fp8_transport.py:21-23)."""
    return dict(_peer_alignment_metrics)


class WireView(NamedTuple):
    """Rows of `head_dim` channels of one tensor addressed as
    [peer, seq, batch, head] with element strides (unit channel stride).
    Unlike a torch view it may describe rows beyond the tensor (global
    sequence index >= valid_seq), which the codec never touches."""
    ptr: int
    shape: tuple
    strides: tuple
    dtype: torch.dtype

    @staticmethod
    def of(t: torch.Tensor) -> "WireView":
        """From a 5-D [peer, seq, batch, head, head_dim] tensor view."""
        if t.ndim != 5 or t.stride(-1) != 1:
            raise ValueError("PHAA FP8 wire views are 5-D with unit channel stride")
        return WireView(t.data_ptr(), tuple(t.shape[:4]), tuple(t.stride()[:4]), t.dtype)


def _rows_view(t: torch.Tensor, peers: int, head_dim: int) -> torch.Tensor:
    """A [peer, seq, batch, head, head_dim] view of `t` whose lexicographic
    row order equals the reference's flattened row order."""
    if t.ndim == 5 and t.shape[0] == peers and t.shape[-1] == head_dim and t.stride(-1) == 1:
        return t
    if t.ndim >= 2 and t.stride(-1) == 1 and t.shape[-1] % head_dim == 0 and t.ndim <= 4:
        v = t.unflatten(-1, (t.shape[-1] // head_dim, head_dim))
        while v.ndim < 5:
            v = v.unsqueeze(1)
        if v.shape[0] == peers:
            return v
    return t.contiguous().reshape(peers, -1, 1, 1, head_dim)


def encode(tensors, head_dim: int, peers: int, *, peer_padding: int = 0, rotary_emb=None,
           out: torch.Tensor | None = None, views=None, valid_seq: int | None = None
           ) -> torch.Tensor:
    """Encode 1 or 3 tensors into the PHAA byte wire (a flat uint8 tensor).

    `views`, when given, are `WireView`s of the sources (any strides, unit
    channel stride); rows whose global sequence index peer*seq + s reaches
    `valid_seq` encode as zeros without being read."""
    streams = len(tensors)
    if views is None:
        # `rows` keeps any contiguous copies alive until the kernel is queued.
        rows = [_rows_view(t, peers, head_dim) for t in tensors]
        views = [WireView.of(r) for r in rows]
    shape = views[0].shape
    if any(v.shape != shape for v in views):
        raise ValueError("PHAA FP8 transport requires matching shapes")
    peer_rows = shape[1] * shape[2] * shape[3]
    nbytes = peers * (peer_rows * streams * (head_dim + 4) + peer_padding)
    wire = out if out is not None else torch.empty(nbytes, dtype=torch.uint8,
                                                    device=tensors[0].device)
    strides = [s for v in views for s in v.strides]
    cos = sin = None
    rotary = 0
    if rotary_emb is not None:
        cos, sin = rotary_emb
        rotary = cos.shape[-1]
    call("xgb_fp8_wire_encode_view", ptr_array(v.ptr for v in views), i64_array(strides),
         streams, shape[0], shape[1], shape[2], shape[3], head_dim, _DTYPE[tensors[0].dtype],
         cos.data_ptr() if cos is not None else None, sin.data_ptr() if sin is not None else None,
         rotary, shape[0] * shape[1] if valid_seq is None else valid_seq, peer_padding,
         wire.data_ptr(), torch.cuda.current_stream(tensors[0].device).cuda_stream)
    return wire


def decode(wire: torch.Tensor, outputs, head_dim: int, peers: int, *, peer_padding: int = 0):
    """Decode the wire into contiguous outputs (rows = numel / head_dim)."""
    streams = len(outputs)
    rows = outputs[0].numel() // head_dim
    call("xgb_fp8_wire_decode", wire.data_ptr(), ptr_array(o.data_ptr() for o in outputs),
         streams, rows, peers, head_dim, peer_padding, _DTYPE[outputs[0].dtype],
         torch.cuda.current_stream(wire.device).cuda_stream)


def decode_view(wire: torch.Tensor, views, head_dim: int, *, valid_seq: int | None = None,
                peer_padding: int = 0):
    """Decode the wire into `WireView` destinations, skipping rows whose
    global sequence index peer*seq + s reaches `valid_seq`."""
    shape = views[0].shape
    if any(v.shape != shape for v in views):
        raise ValueError("PHAA FP8 decode views must match")
    strides = [s for v in views for s in v.strides]
    call("xgb_fp8_wire_decode_view", wire.data_ptr(), ptr_array(v.ptr for v in views),
         i64_array(strides), len(views), shape[0], shape[1], shape[2], shape[3], head_dim,
         shape[0] * shape[1] if valid_seq is None else valid_seq, peer_padding,
         _DTYPE[views[0].dtype], torch.cuda.current_stream(wire.device).cuda_stream)


def fp8_all_to_all(output, tensor, head_dim, group):
    fp8_all_to_all_many((output,), (tensor,), head_dim, group)


def fp8_all_to_all_many(outputs, tensors, head_dim, group, *, rotary_emb=None):
    """Exchange equal-shaped tensors and their row scales in one byte
    collective (x_base/x_base/phaa/fp8_transport.py:85-144)."""
    streams = len(tensors)
    if streams not in (1, 3) or len(outputs) != streams:
        raise ValueError("PHAA FP8 transport expects one tensor or a QKV triple")
    if any(t.device.type != "cuda" for t in outputs):
        raise ValueError("PHAA FP8 transport requires CUDA tensors")
    if any(x.shape != tensors[0].shape for x in outputs):
        raise ValueError("PHAA FP8 transport requires matching shapes and head dim divisible by four")
    if any(not out.is_contiguous() for out in outputs):
        raise ValueError("PHAA FP8 transport requires contiguous outputs")
    if any(t.dtype not in _DTYPE for t in outputs):
        raise ValueError("PHAA FP8 transport requires bf16/fp16 tensors")
    recv, peers, peer_padding = fp8_exchange_wire(tensors, head_dim, group, rotary_emb=rotary_emb)
    decode(recv, outputs, head_dim, peers, peer_padding=peer_padding)


def fp8_exchange_wire(tensors, head_dim, group, *, rotary_emb=None):
    """Encode and exchange, without the decode: returns (received wire as
    uint8 [bytes], peers, peer_padding) for a consumer that reads the wire
    itself (sage_prepare_wire). The received wire is allocated on the
    current stream."""
    streams = len(tensors)
    if streams not in (1, 3):
        raise ValueError("PHAA FP8 transport expects one tensor or a QKV triple")
    if any(t.device.type != "cuda" for t in tensors):
        raise ValueError("PHAA FP8 transport requires CUDA tensors")
    shape = tensors[0].shape
    if head_dim % 4 or any(x.shape != shape for x in tensors):
        raise ValueError("PHAA FP8 transport requires matching shapes and head dim divisible by four")
    if any(t.dtype not in _DTYPE for t in tensors):
        raise ValueError("PHAA FP8 transport requires bf16/fp16 tensors")
    rows = tensors[0].numel() // head_dim
    peers = dist.get_world_size(group)
    if rows % peers or tensors[0].numel() % head_dim:
        raise ValueError("PHAA FP8 rows must divide evenly among peers")
    peer_rows = rows // peers
    peer_bytes = peer_rows * streams * (head_dim + 4)
    align_peers = os.environ.get("XGEN_PHAA_FP8_ALIGN16", "0") == "1"
    peer_padding = (-peer_bytes) % 16 if align_peers else 0
    if align_peers:
        if _peer_alignment_metrics["calls"] == 0:
            logging.getLogger(__name__).info("PHAA FP8 per-peer 16-byte alignment enabled")
        _peer_alignment_metrics["calls"] += 1
        _peer_alignment_metrics["padded_calls"] += int(peer_padding > 0)
        _peer_alignment_metrics["padding_bytes"] += peers * peer_padding
    if (streams == 3 and len(shape) == 5 and shape[0] == peers
            and len({x.stride() for x in tensors}) > 1 and all(x.stride(-1) == 1 for x in tensors)):
        _mixed_stride_metrics["calls"] += 1
        _mixed_stride_metrics["avoided_contiguous_bytes"] += sum(
            x.numel() * x.element_size() for x in tensors if not x.is_contiguous())
    send = encode(tensors, head_dim, peers, peer_padding=peer_padding, rotary_emb=rotary_emb)
    wire_shape = (peers, peer_bytes + peer_padding) if peer_padding else (streams * rows, head_dim + 4)
    send = send.view(wire_shape)
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return recv.view(-1), peers, peer_padding
