"""The SP exchanges as one kernel each over NVLink (B200 extension of PHAA).

`fp8_transport.fp8_exchange_wire` / `fp8_all_to_all` encode Q/K/V (the
gather) or the attention output (the return) into a local send buffer and
move it with NCCL `all_to_all_single` (x_base/x_base/phaa/fp8_transport.py
:85-144). Here the encode kernel (`xgb_fp8_wire_encode_peers`) stores each
peer's rows straight into that peer's receive buffer, at the offset the
all-to-all would have delivered them to, so the received wire is byte for
byte the NCCL path's: `sage_prepare_wire` reads the gathered one unchanged
and the wire decode reads the returned one.

The receive buffers live in symmetric memory (`torch.distributed.
_symmetric_memory`: every rank maps every other rank's buffer), two slots
per group and shape, used in turn. Each exchange e (slot e % 2) is ordered
by epoch flags at the end of the buffers, all waits bounded:

  1. wait until every peer has signalled it finished reading this slot at
     exchange e - 2 ("freed"),
  2. encode into the peers' slots,
  3. signal every peer "arrived" = e, then wait until every peer's arrived
     flag in this rank's buffer reaches e,
  4. the consumer reads the slot; `release` then signals "freed" = e.

A rank never waits on its own flags: its own section of a slot is ordered
by a CUDA event that `release` records on the reading stream and the next
exchange into that slot waits for on its own stream.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from .._lib import call, i64_array, ptr_array
from .fp8_transport import WireView, _rows_view

_ROW_BYTES = 132          # 128 e4m3 codes + fp32 scale
_MAX_PEERS = 8
_MAX_HEADS = 12
_LIMIT_NS = 5_000_000_000
_ARRIVED, _FREED = 0, 1
_wires: dict = {}


def enabled() -> bool:
    """XGB_SP_PEER_WIRE=1 routes the eligible FP8-wire exchanges of PHAA (the
    Sage gather read straight from the wire, and the return) through this
    path."""
    return os.environ.get("XGB_SP_PEER_WIRE", "0") == "1"


def eligible(tensors, head_dim: int, group) -> bool:
    """Q/K/V chunk views, or one returned attention output, [peers, seq,
    batch, heads, 128] in bf16 on the GPU, at most 8 peers and 12 heads per
    peer, seq*batch a multiple of 4."""
    if len(tensors) not in (1, 3) or head_dim != 128 or group is None:
        return False
    t = tensors[0]
    if t.ndim != 5 or not t.is_cuda or any(x.dtype != torch.bfloat16 or x.shape != t.shape for x in tensors):
        return False
    peers, seq, batch, heads, _ = t.shape
    if peers != dist.get_world_size(group) or not 1 < peers <= _MAX_PEERS:
        return False
    return heads <= _MAX_HEADS and (seq * batch) % 4 == 0 and all(
        x.stride(-1) == 1 and x.data_ptr() % 16 == 0 and all(s % 8 == 0 for s in x.stride()[:4])
        for x in tensors)


class PeerWire:
    """Two receive slots of `slot_bytes` (peers x section) plus the epoch
    flags, in symmetric memory over `group`. Creating one is collective."""

    def __init__(self, group, slot_bytes: int, device: torch.device):
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group
        self.peers = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if slot_bytes % (16 * self.peers):
            raise ValueError("peer wire sections must be multiples of 16 bytes")
        self.slot_bytes = slot_bytes
        self.section = slot_bytes // self.peers
        self.flag_off = 2 * slot_bytes
        flag_bytes = (2 * 2 * self.peers * 4 + 15) // 16 * 16
        self.buf = symm_mem.empty(self.flag_off + flag_bytes, dtype=torch.uint8, device=device)
        # Flags start at 0 on every rank before any rank can signal (the
        # rendezvous below is collective).
        self.buf[self.flag_off:].zero_()
        torch.cuda.synchronize(device)
        self.handle = symm_mem.rendezvous(self.buf, group)
        self.ptrs = [int(p) for p in self.handle.buffer_ptrs]
        self.others = [p for p in range(self.peers) if p != self.rank]
        self.freed = [None, None]  # per slot: event after this rank's own reads
        self.epoch = 0

    def _flag(self, owner: int, kind: int, slot: int, src: int) -> int:
        return self.ptrs[owner] + self.flag_off + ((kind * 2 + slot) * self.peers + src) * 4

    def _wait(self, kind: int, slot: int, value: int, stream: int, err: int) -> None:
        flags = [self._flag(self.rank, kind, slot, p) for p in self.others]
        call("xgb_peer_wait", ptr_array(flags), len(flags), value, _LIMIT_NS, err, stream)

    def _signal(self, kind: int, slot: int, value: int, stream: int) -> None:
        flags = [self._flag(p, kind, slot, self.rank) for p in self.others]
        call("xgb_peer_signal", ptr_array(flags), len(flags), value, stream)

    def exchange(self, tensors, rotary_emb=None, valid_seq: int | None = None):
        """Encode 1 or 3 views [peers, seq, batch, heads, 128] into every
        peer's next slot; returns (received wire uint8 [slot_bytes], ticket)
        on the current stream."""
        from ..attention import _err_flag

        device = tensors[0].device
        stream = torch.cuda.current_stream(device).cuda_stream
        err = _err_flag(device).data_ptr()
        e = self.epoch + 1
        slot = e % 2
        if self.freed[slot] is not None:
            torch.cuda.current_stream(device).wait_event(self.freed[slot])
        if e > 2:
            self._wait(_FREED, slot, e - 2, stream, err)
        views = [WireView.of(t) for t in tensors]
        peers, seq, batch, heads = views[0].shape
        dst = [self.ptrs[p] + slot * self.slot_bytes + self.rank * self.section for p in range(peers)]
        cos = sin = None
        rotary = 0
        if rotary_emb is not None:
            cos, sin = rotary_emb
            rotary = cos.shape[-1]
        call("xgb_fp8_wire_encode_peers", ptr_array(v.ptr for v in views),
             i64_array(s for v in views for s in v.strides), len(views), peers, seq, batch, heads,
             cos.data_ptr() if cos is not None else None, sin.data_ptr() if sin is not None else None,
             rotary, peers * seq if valid_seq is None else valid_seq, ptr_array(dst), stream)
        self._signal(_ARRIVED, slot, e, stream)
        self._wait(_ARRIVED, slot, e, stream, err)
        self.epoch = e
        wire = self.buf.narrow(0, slot * self.slot_bytes, self.slot_bytes)
        return wire, (self, e, slot)


def exchange_wire(tensors, head_dim: int, group, *, rotary_emb=None):
    """fp8_exchange_wire over peer memory: (received wire, peers,
    peer_padding = 0, ticket); pass the ticket to `release` on the stream
    that reads the wire, after its reads."""
    rows = [_rows_view(t, dist.get_world_size(group), head_dim) for t in tensors]
    peers, seq, batch, heads, _ = rows[0].shape
    slot_bytes = peers * len(rows) * seq * batch * heads * _ROW_BYTES
    key = (id(group), len(rows), slot_bytes, tensors[0].device.index)
    pw = _wires.get(key)
    if pw is None:
        pw = _wires[key] = PeerWire(group, slot_bytes, tensors[0].device)
    wire, ticket = pw.exchange(rows, rotary_emb=rotary_emb)
    return wire, peers, 0, ticket


def release(ticket) -> None:
    """Tell every peer this rank has finished reading the ticket's slot."""
    pw, e, slot = ticket
    cur = torch.cuda.current_stream(pw.buf.device)
    pw._signal(_FREED, slot, e, cur.cuda_stream)
    ev = torch.cuda.Event()
    ev.record(cur)
    pw.freed[slot] = ev
