"""Local packed input/output of the H3 transformer under Ulysses SP.

Same contract as x_diffusers/x_diffusers/framework/transformer/h3_local_io.py
:41-92. Each SP rank owns the contiguous span `LocalSpan.for_rank(S, sp,
rank)` of the packed sequence (text, video and audio rows at their packed
positions). Only the rows it owns are projected into its hidden state, and
the tail of the last span is zero padding. The final predictions are
gathered over the SP group and split back into video and audio rows.

`model` supplies what the reference's MiniMaxH3Model does:
- `parallel_manager` (None or a ParallelManager);
- `proj_in`, `audio_proj_in`, `proj_out`, `audio_proj_out`;
- `norm_out(hidden, temb, indices)` and `rope(positions)`;
- text projection: `project_text(text)` if present, otherwise
  `token_refiner(context_embedder(text))`.

An optional `_h3_shared_sequence_exchange` (the TP-shared layout) is
honoured as the reference does.
"""
from __future__ import annotations

import torch

from ..sp.comm import gather_sequence
from ..sp.padding import set_pad
from .adaln import LocalSpan

PAD_KEY = "mmh3_seq"


def _sp(model):
    manager = getattr(model, "parallel_manager", None)
    peers = manager.sp_size if manager is not None else 1
    rank = manager.sp_rank if peers > 1 else 0
    return manager, peers, rank


def _project_text(model, text):
    project = getattr(model, "project_text", None)
    if project is not None:
        return project(text)
    embeds = model.context_embedder(text.to(model.context_embedder.weight.dtype))
    return model.token_refiner(embeds)


def prepare_local(model, video, audio, text, positions, text_indices, video_indices, audio_indices):
    """(hidden [B, span.length, H], rotary, span) of this rank: the text
    projection over the full text context, then this span's rows of every
    modality scattered to their packed positions."""
    manager, peers, rank = _sp(model)
    span = LocalSpan.for_rank(len(positions), peers, rank)
    for inputs, indices in ((video, video_indices), (audio, audio_indices), (text, text_indices)):
        if indices.ndim != 1 or len(indices) != inputs.shape[1]:
            raise ValueError("H3 packed modality indices must match the input rows")
        # an index outside the sequence would be dropped silently by the span filter
        torch._assert_async(((indices >= 0) & (indices < len(positions))).all(),
                            "H3 packed modality index is outside the sequence")
    if peers > 1:
        set_pad(PAD_KEY, len(positions), manager.sp_group)
    embeds = _project_text(model, text)  # the text refiner needs the full text context
    hidden = embeds.new_zeros((embeds.shape[0], span.length, embeds.shape[-1]))
    source, target = span.indices(text_indices)
    hidden.index_copy_(1, target, embeds.index_select(1, source))
    del embeds
    for inputs, indices, projection in ((video, video_indices, model.proj_in),
                                        (audio, audio_indices, model.audio_proj_in)):
        source, target = span.indices(indices)
        local = inputs.index_select(1, source).to(projection.weight.dtype)
        hidden.index_copy_(1, target, projection(local).to(hidden.dtype))
    shared = getattr(model, "_h3_shared_sequence_exchange", None)
    if shared is not None:
        shared.set_tokens(len(positions))
        rotary = model.rope(positions)
    else:
        rotary = model.rope(span.slice_padded(positions))
    return hidden, rotary, span


def gather_local_output(model, hidden, temb, span, timestep_indices, video_indices, audio_indices):
    """Output AdaLN and prediction heads on this rank's span, then the
    sequence gather (pad dropped) and the split into (video, audio) rows."""
    local_indices = span.slice_padded(timestep_indices)
    hidden = model.norm_out(hidden, temb, local_indices).to(model.proj_out.weight.dtype)
    video = model.proj_out(hidden)
    audio = model.audio_proj_out(hidden.to(model.audio_proj_out.weight.dtype))
    if (getattr(model, "_h3_cuda_precision", "none") in ("fp8-bf16", "fp8-sage")
            and (video.dtype != torch.float32 or audio.dtype != torch.float32)):
        raise ValueError("H3 TP/CP final prediction heads must remain FP32")
    width = video.shape[-1]
    prediction = torch.cat((video, audio), dim=-1)
    manager, peers, _ = _sp(model)
    if peers > 1:
        pad = span.length * peers - len(timestep_indices)
        prediction = gather_sequence(prediction, manager.sp_group, dim=1, pad=pad)
    return (prediction[..., :width].index_select(1, video_indices),
            prediction[..., width:].index_select(1, audio_indices))
