"""PHAA: head-chunked Ulysses attention with the A2A overlapped on a side stream.

Mirror of `run_phaa_attention` (x_base/x_base/phaa/phaa_attention.py:38-366)
for the options the H3 CUDA recipes use: bf16 or FP8 wire exchange, natural
or tail-first chunk order, gather priority, a separate scatter stream/group,
device or host join. The local heads are split into `phaa_split_num` chunks
(remainder to the first chunks); chunk i+1's gather A2A runs on
`comm_stream` while chunk i's attention runs on the compute stream, and each
chunk's output returns by its own A2A.

With `async_options` (an `AsyncFP8Options`; requires FP8 transport and
device join) every exchange is an async NCCL collective submitted on
`comm_stream` and joined on the consuming stream (`submit_fp8_exchange` /
`finish_fp8_exchange`), optionally with the direct gather, fused return pack
and direct return layouts (phaa_attention.py:84-107, :150-327).

B200 extensions:
- `fuse_rope=True` with `rotary_emb=(cos, sin)` applies the partial RoPE to Q
  and K inside the FP8 wire encode (the reference applies it in a separate
  pass before PHAA; the bytes on the wire are identical).
- `int8_transport=True` (one head chunk, the B200 Sage backend) sends Q/K/V
  already Sage-quantised (`sage_wire`: RoPE, int8 Q/K per 16 tokens, e4m3 V
  per channel, sequence-wide K mean and V scale from an all-reduce) and runs
  the attention on the received bytes in place; the output returns over the
  FP8 wire (`fp8_transport=True`) or bf16.
"""
from __future__ import annotations

from contextlib import nullcontext

import torch
import torch.distributed as dist

from ..sp.padding import get_pad_manager
from .. import trace
from . import fp8_transport as fp8
from . import peer_wire


class _HostStreams:
    """Stream/event stand-ins for CPU tensors (gloo tests): ops are synchronous."""

    class Event:
        def record(self, *a):
            pass

    @staticmethod
    def current_stream():
        return _HostStreams._Stream()

    class _Stream:
        def wait_stream(self, *a):
            pass

        def wait_event(self, *a):
            pass

        def synchronize(self):
            pass

        def record_event(self):
            return _HostStreams.Event()

    @staticmethod
    def stream(s):
        return nullcontext()


def chunk_sizes(heads_per_device: int, split: int) -> list[int]:
    base, rem = divmod(heads_per_device, split)
    return [base + (1 if i < rem else 0) for i in range(split)]


def run_phaa_attention(query, key, value, *, comm_stream, sp_group, sp_size, heads,
                       phaa_split_num, head_dim, rope_fn=None, rotary_emb=None,
                       attention_mask=None, pad_key="pad", attention_fn=None,
                       fp8_transport=False, gather_priority=False, scatter_stream=None,
                       scatter_group=None, tail_first=False, device_join=False,
                       async_options=None, fuse_rope=False, int8_transport=False):
    """query/key/value (B, S_loc, heads*head_dim) -> (B, S_loc, heads*head_dim)."""
    W_S = sp_size
    B, Sq, H = query.shape
    D = head_dim
    if attention_fn is None:
        raise ValueError("PHAA on B200 requires a model-local attention_fn")
    if fuse_rope and (not fp8_transport or rotary_emb is None):
        raise ValueError("fused PHAA RoPE requires FP8 transport and rotary_emb")
    if gather_priority and not fp8_transport:
        raise ValueError("PHAA gather priority requires FP8 transport")
    if device_join and (not fp8_transport or scatter_stream is not None):
        raise ValueError("PHAA device join requires single-stream FP8 transport")
    async_exchange = async_options is not None
    direct_gather = async_exchange and async_options.direct_gather
    direct_return = async_exchange and async_options.direct_return
    fused_return_pack = async_exchange and async_options.fused_return_pack
    if async_exchange and not device_join:
        raise ValueError("PHAA async exchange requires device join")
    if (scatter_stream is None) != (scatter_group is None) or (
            scatter_stream is not None and not fp8_transport):
        raise ValueError("Separate PHAA scatter requires FP8, a stream and a process group")
    if fp8_transport and query.device.type != "cuda":
        raise ValueError("PHAA FP8 transport requires CUDA")
    if int8_transport:
        return _int8_wire(query, key, value, comm_stream=comm_stream, sp_group=sp_group,
                          sp_size=sp_size, heads=heads, phaa_split_num=phaa_split_num,
                          head_dim=head_dim, rotary_emb=rotary_emb, attention_mask=attention_mask,
                          pad_key=pad_key, attention_fn=attention_fn, fp8_transport=fp8_transport,
                          device_join=device_join)

    hpd = heads // W_S
    sizes = chunk_sizes(hpd, phaa_split_num)
    offsets = [sum(sizes[:i]) for i in range(phaa_split_num)]
    order = list(range(phaa_split_num))
    if tail_first:
        if not fp8_transport or phaa_split_num != 4:
            raise ValueError("PHAA tail-first requires FP8 transport and four chunks")
        order = [3, 0, 1, 2]
    pad = get_pad_manager().get_or_default(pad_key, 0)
    acc = torch.cuda if query.device.type == "cuda" else _HostStreams
    output_stream = scatter_stream if scatter_stream is not None else comm_stream
    output_group = scatter_group if scatter_group is not None else sp_group

    def exchange_one(out, inp, group):
        if fp8_transport:
            fp8.fp8_all_to_all(out, inp, D, group)
        else:
            dist.all_to_all_single(out, inp.contiguous(), group=group)

    q5 = query.unflatten(-1, (heads, D)).unflatten(2, (W_S, hpd))
    k5 = key.unflatten(-1, (heads, D)).unflatten(2, (W_S, hpd))
    v5 = value.unflatten(-1, (heads, D)).unflatten(2, (W_S, hpd))
    chunks = []
    for c in range(phaa_split_num):
        o, cs = offsets[c], sizes[c]
        chunks.append(tuple(t[:, :, :, o:o + cs, :].permute(2, 1, 0, 3, 4) for t in (q5, k5, v5)))
    def gather_shape(cs):
        if direct_gather:
            return (B, cs, W_S * Sq - pad, D)
        return (W_S, Sq, B, cs, D)

    # Sage backends take the received FP8 wire as it is: the Sage
    # preparation reads Q/K/V from it (bf16(e4m3 * scale), the decode's
    # values), so there is no decode pass and no bf16 gather buffer. Only
    # for bf16 activations: the wire decode rounds to the activation dtype,
    # and the wire-reading preparation produces bf16 values.
    from_wire = (fp8_transport and not async_exchange and attention_mask is None
                 and query.dtype == torch.bfloat16
                 and (rope_fn is None or rotary_emb is None or fuse_rope) and D == 128
                 and getattr(attention_fn, "precision", None) == "sage"
                 and hasattr(attention_fn, "attend_fp8_wire"))
    wires = [None] * phaa_split_num
    gather = [None if from_wire else
              tuple(torch.empty(gather_shape(cs), device=query.device, dtype=query.dtype) for _ in range(3))
              for cs in sizes]
    if direct_return:
        final = torch.empty((B, Sq, H), device=query.device, dtype=query.dtype)
        returned = None
    else:
        # The layer's output [B, Sq, H]: head peer*hpd + offsets[i] + j of
        # chunk i. The peer return decodes straight into it; the other paths
        # receive into `returned` and are copied in at the end.
        final = torch.empty((B, Sq, H), device=query.device, dtype=query.dtype)
        returned = [torch.empty((W_S, Sq, B, cs * D), device=query.device, dtype=query.dtype)
                    for cs in sizes]
    decoded_in_place = set()

    def final_chunk(i):
        """Chunk i's heads of `final` as a [W_S, Sq, B, cs, D] view."""
        return final.view(B, Sq, W_S, hpd, D).narrow(3, offsets[i], sizes[i]).permute(2, 1, 0, 3, 4)
    pending_gathers, pending_returns = {}, []
    if async_exchange:
        from .fp8_async_transport import finish_fp8_exchange, submit_fp8_exchange
    gathered = [acc.Event() for _ in sizes]
    attended = [acc.Event() for _ in sizes]
    results = [None] * phaa_split_num

    def gather_chunk(i):
        if async_exchange:
            pending_gathers[i] = submit_fp8_exchange(
                gather[i], chunks[i], D, sp_group, row_tiling=async_options.row_tiling,
                direct_gather=direct_gather, rotary_emb=rotary_emb if fuse_rope else None)
            for t in chunks[i]:
                t.record_stream(comm_stream)
            return
        if from_wire and peer_wire.enabled() and peer_wire.eligible(chunks[i], D, sp_group):
            # B200: encode straight into the peers' receive buffers (no NCCL step)
            wires[i] = peer_wire.exchange_wire(chunks[i], D, sp_group,
                                               rotary_emb=rotary_emb if fuse_rope else None)
        elif from_wire:
            wires[i] = fp8.fp8_exchange_wire(chunks[i], D, sp_group,
                                             rotary_emb=rotary_emb if fuse_rope else None) + (None,)
        elif fp8_transport:
            fp8.fp8_all_to_all_many(gather[i], chunks[i], D, sp_group,
                                    rotary_emb=rotary_emb if fuse_rope else None)
        else:
            for out, inp in zip(gather[i], chunks[i]):
                exchange_one(out, inp, sp_group)
        gathered[i].record(comm_stream)

    trace.mark("start")
    comm_stream.wait_stream(acc.current_stream())
    if scatter_stream is not None:
        scatter_stream.wait_stream(acc.current_stream())
    with acc.stream(comm_stream):
        for i in (order if gather_priority else order[:1]):
            gather_chunk(i)
            trace.mark("gathered", comm_stream)

    for pos, step in enumerate(order):
        if async_exchange:
            finish_fp8_exchange(pending_gathers.pop(step))
        else:
            acc.current_stream().wait_event(gathered[step])
        cs = sizes[step]
        if from_wire:
            wire, peers, peer_padding, ticket = wires[step]
            wires[step] = None
            send = torch.empty((W_S, Sq, B, cs, D), device=query.device, dtype=query.dtype)
            if pad > 0:
                send[-1, Sq - pad:].zero_()
            view = send.flatten(0, 1).permute(1, 2, 0, 3)
            attention_fn.attend_fp8_wire(wire, peers=peers, seq=Sq, batch=B, heads=cs,
                                         valid_seq=W_S * Sq - pad, peer_padding=peer_padding,
                                         out=view.narrow(2, 0, W_S * Sq - pad))
            if ticket is None:
                wire.record_stream(acc.current_stream())  # allocated on the comm stream
            else:
                peer_wire.release(ticket)  # the Sage preparation has read it
            results[step] = send.flatten(-2, -1)
        else:
            if direct_gather:
                qv, kv, vv = gather[step]
            else:
                qv, kv, vv = (x.flatten(0, 1).permute(1, 2, 0, 3) for x in gather[step])
                if pad > 0:
                    qv, kv, vv = (x.narrow(2, 0, x.shape[2] - pad) for x in (qv, kv, vv))
            if rope_fn is not None and rotary_emb is not None and not fuse_rope:
                qv, kv = rope_fn(qv, kv, *rotary_emb)
            if fused_return_pack:
                # The return encode reads the [B, cs, S, D] output as it is.
                results[step] = attention_fn(qv, kv, vv, head_offset=offsets[step],
                                             attn_mask=attention_mask).type_as(query)
            elif getattr(attention_fn, "writes_into", False):
                # The kernel epilogue stores straight into the return-A2A send
                # layout (W_S, S, B, cs, D): no reshape/pad copies.
                send = torch.empty((W_S, Sq, B, cs, D), device=query.device, dtype=query.dtype)
                if pad > 0:
                    send[-1, Sq - pad:].zero_()
                view = send.flatten(0, 1).permute(1, 2, 0, 3)
                attention_fn(qv, kv, vv, head_offset=offsets[step], attn_mask=attention_mask,
                             out=view.narrow(2, 0, W_S * Sq - pad))
                results[step] = send.flatten(-2, -1)
            else:
                out = attention_fn(qv, kv, vv, head_offset=offsets[step], attn_mask=attention_mask)
                out = out.type_as(query)
                if pad > 0:
                    shape = list(out.shape)
                    shape[2] = pad
                    out = torch.cat([out, out.new_zeros(shape)], dim=2)
                results[step] = out.unflatten(2, (W_S, -1)).permute(2, 3, 0, 1, 4).flatten(-2, -1)
        attended[step].record()
        with acc.stream(comm_stream):
            if not gather_priority and pos + 1 < phaa_split_num:
                gather_chunk(order[pos + 1])
            ctx = acc.stream(scatter_stream) if scatter_stream is not None else nullcontext()
            with ctx:
                output_stream.wait_event(attended[step])
                if async_exchange:
                    pending_returns.append(submit_fp8_exchange(
                        None if direct_return else (returned[step],), (results[step],), D,
                        output_group, row_tiling=async_options.row_tiling,
                        return_shard_seq=Sq if fused_return_pack else 0))
                elif (fp8_transport and peer_wire.enabled() and
                      peer_wire.eligible((results[step].unflatten(-1, (-1, D)),), D, output_group)):
                    # B200: encode the output straight into the peers' receive buffers,
                    # then decode it into the layer's output in place
                    wire, peers, _, ticket = peer_wire.exchange_wire(
                        (results[step].unflatten(-1, (-1, D)),), D, output_group)
                    trace.mark("returned", comm_stream)
                    fp8.decode_view(wire, [fp8.WireView.of(final_chunk(step))], D)
                    trace.mark("decoded", comm_stream)
                    decoded_in_place.add(step)
                    peer_wire.release(ticket)
                else:
                    exchange_one(returned[step], results[step], output_group)
                if device_join:
                    results[step].record_stream(comm_stream)
                    for t in chunks[step]:
                        t.record_stream(comm_stream)

    if async_exchange:
        for step, pending in zip(order, pending_returns):
            if direct_return:
                layout = (Sq, B, W_S, hpd, sizes[step], offsets[step])
                finish_fp8_exchange(pending, output=final, return_layout=layout)
            else:
                finish_fp8_exchange(pending)
    elif device_join:
        acc.current_stream().wait_stream(comm_stream)
    else:
        comm_stream.synchronize()
    if scatter_stream is not None:
        scatter_stream.synchronize()
    trace.mark("end")
    if direct_return:
        return final
    for i, b in enumerate(returned):
        if i not in decoded_in_place:
            final_chunk(i).copy_(b.unflatten(-1, (sizes[i], D)))
    return final


def _int8_wire(query, key, value, *, comm_stream, sp_group, sp_size, heads, phaa_split_num,
               head_dim, rotary_emb, attention_mask, pad_key, attention_fn, fp8_transport,
               device_join):
    """PHAA with the INT8 wire: one chunk of all local heads (see module doc)."""
    from .sage_wire import SageWire, sage_wire_attention, sage_wire_exchange

    if phaa_split_num != 1:
        raise ValueError("INT8 wire transport exchanges all local heads at once (phaa_split_num=1)")
    if getattr(attention_fn, "precision", None) != "sage" or attention_mask is not None:
        raise ValueError("INT8 wire transport needs the B200 Sage backend and no attention mask")
    if query.device.type != "cuda" or head_dim != 128:
        raise ValueError("INT8 wire transport needs CUDA and head_dim 128")
    W = sp_size
    B, Sq, H = query.shape
    hpd = heads // W
    pad = get_pad_manager().get_or_default(pad_key, 0)
    seq_real = W * Sq - pad
    rank = dist.get_rank(sp_group) if W > 1 else 0
    cur = torch.cuda.current_stream(query.device)
    # Buffers belong to the compute stream, which waits for the exchange
    # before reading them, so their reuse stays ordered after it.
    bufs = SageWire(W, Sq, B, hpd, query.device)
    comm_stream.wait_stream(cur)
    with torch.cuda.stream(comm_stream):
        sage_wire_exchange(query, key, value, heads=heads, group=sp_group, peers=W,
                           rotary_emb=rotary_emb, seq_real=seq_real, bufs=bufs)
    cur.wait_stream(comm_stream)
    send = torch.empty((W, Sq, B, hpd, head_dim), device=query.device, dtype=query.dtype)
    if pad > 0:
        send[-1, Sq - pad:].zero_()
    view = send.flatten(0, 1).permute(1, 2, 0, 3).narrow(2, 0, W * Sq - pad)
    sage_wire_attention(bufs, view, seq_real, rank)
    attention_fn.calls += 1
    attention_fn.kernel_calls += 1
    returned = torch.empty((W, Sq, B, hpd * head_dim), device=query.device, dtype=query.dtype)
    comm_stream.wait_stream(cur)
    with torch.cuda.stream(comm_stream):
        if fp8_transport:
            fp8.fp8_all_to_all(returned, send.flatten(-2, -1), head_dim, sp_group)
        else:
            dist.all_to_all_single(returned, send.flatten(-2, -1), group=sp_group)
        for t in (query, key, value, send):
            t.record_stream(comm_stream)
    if device_join:
        cur.wait_stream(comm_stream)
    else:
        comm_stream.synchronize()
    return returned.permute(2, 1, 0, 3).flatten(-2, -1)
