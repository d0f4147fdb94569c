"""Rank-local packed input and output of the H3 transformer under Ulysses SP.

The contract is that of x_diffusers/x_diffusers/framework/transformer/
h3_local_io.py:14-92: SP rank r owns the contiguous block of
ceil(S / sp) packed positions starting at r * ceil(S / sp), the last block
padded with zero rows. A rank projects only the video and audio rows whose
packed position falls in its block, places the (full-context) text
projection's rows of its block, builds RoPE for its block, and at the end
the prediction heads run on the block before one sequence gather returns
the full (video, audio) predictions.

Here a rank's block is a `LocalSpan`; `prepare_local` builds a placement
(which input rows land on which local rows) per modality from the packed
indices and fills one zero-initialised buffer with each modality's projected
rows. `model` supplies what the reference's MiniMaxH3Model does:
`parallel_manager` (None, or with sp_size / sp_rank / sp_group),
`proj_in`, `audio_proj_in`, `proj_out`, `audio_proj_out`,
`norm_out(hidden, temb, indices)`, `rope(positions)`, and the text path
`project_text(text)` or else `token_refiner(context_embedder(text))`.
A model with `_h3_shared_sequence_exchange` (the TP-shared layout) gets
RoPE over the whole sequence and announces the token count to it.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ..sp.comm import gather_sequence
from ..sp.padding import set_pad

PAD_KEY = "mmh3_seq"


@dataclass(frozen=True)
class LocalSpan:
    """One rank's block of the packed sequence: packed positions
    [start, start + valid) are real, local rows [valid, length) are padding."""

    start: int
    length: int
    valid: int

    @classmethod
    def for_rank(cls, total: int, peers: int, rank: int) -> "LocalSpan":
        if total < 1 or peers < 1 or rank < 0 or rank >= peers:
            raise ValueError(f"Invalid H3 local sequence layout: {total} tokens, rank {rank} of {peers}")
        block = -(-total // peers)
        first = rank * block
        return cls(start=first, length=block, valid=min(block, max(total - first, 0)))

    @property
    def stop(self) -> int:
        return self.start + self.valid

    def slice_padded(self, tensor: torch.Tensor, dim: int = 0, value=0) -> torch.Tensor:
        """This block of `tensor` along `dim`, `length` long, with `value`
        in the padding rows."""
        shape = list(tensor.shape)
        shape[dim] = self.length
        out = tensor.new_full(shape, value)
        if self.valid:
            out.narrow(dim, 0, self.valid).copy_(tensor.narrow(dim, self.start, self.valid))
        return out

    def indices(self, packed_indices: torch.Tensor):
        """(input rows, local rows): the input rows whose packed position is
        in this block, and where they land in it."""
        offset = packed_indices - self.start
        rows = torch.nonzero((offset >= 0) & (offset < self.valid), as_tuple=True)[0]
        return rows, offset.index_select(0, rows)


def _sp(model):
    """(group, peers, rank) of the model's SP layout; one rank without SP."""
    manager = getattr(model, "parallel_manager", None)
    if manager is None or manager.sp_size <= 1:
        return None, 1, 0
    return manager.sp_group, manager.sp_size, manager.sp_rank


def _text_embeddings(model, text):
    project = getattr(model, "project_text", None)
    if project is not None:
        return project(text)
    return model.token_refiner(model.context_embedder(text.to(model.context_embedder.weight.dtype)))


def _check_placement(total, pairs):
    for rows, packed in pairs:
        if packed.ndim != 1 or packed.numel() != rows.shape[1]:
            raise ValueError("H3 packed modality indices must match the input rows")
        # Positions outside the sequence would simply fall outside every
        # block; refuse them without a host sync.
        torch._assert_async(((packed >= 0) & (packed < total)).all(),
                            "H3 packed modality index is outside the sequence")


def prepare_local(model, video, audio, text, positions, text_indices, video_indices, audio_indices):
    """(hidden [B, span.length, H], rotary, span) of this rank."""
    group, peers, rank = _sp(model)
    total = len(positions)
    span = LocalSpan.for_rank(total, peers, rank)
    _check_placement(total, ((video, video_indices), (audio, audio_indices), (text, text_indices)))
    if peers > 1:
        set_pad(PAD_KEY, total, group)
    # The text refiner attends over the whole text context, so every rank
    # projects all text rows and keeps those in its block.
    text_rows = _text_embeddings(model, text)
    hidden = text_rows.new_zeros((text_rows.shape[0], span.length, text_rows.shape[-1]))
    placements = (
        (text_indices, lambda rows: text_rows.index_select(1, rows)),
        (video_indices, lambda rows: model.proj_in(video.index_select(1, rows).to(model.proj_in.weight.dtype))),
        (audio_indices, lambda rows: model.audio_proj_in(
            audio.index_select(1, rows).to(model.audio_proj_in.weight.dtype))),
    )
    for packed, project in placements:
        rows, local = span.indices(packed)
        hidden.index_copy_(1, local, project(rows).to(hidden.dtype))
    del text_rows
    exchange = getattr(model, "_h3_shared_sequence_exchange", None)
    if exchange is None:
        rotary = model.rope(span.slice_padded(positions))
    else:
        exchange.set_tokens(total)
        rotary = model.rope(positions)
    return hidden, rotary, span


def gather_local_output(model, hidden, temb, span, timestep_indices, video_indices, audio_indices):
    """Output AdaLN and both prediction heads on this rank's block, one
    gather over the SP group, then the video and audio rows."""
    hidden = model.norm_out(hidden, temb, span.slice_padded(timestep_indices)).to(model.proj_out.weight.dtype)
    heads = (model.proj_out(hidden), model.audio_proj_out(hidden.to(model.audio_proj_out.weight.dtype)))
    if getattr(model, "_h3_cuda_precision", None) in ("fp8-bf16", "fp8-sage") and any(
            h.dtype != torch.float32 for h in heads):
        raise ValueError("H3 TP/CP final prediction heads must remain FP32")
    split = heads[0].shape[-1]
    joined = torch.cat(heads, dim=-1)  # one gather for both heads
    group, peers, _ = _sp(model)
    if peers > 1:
        joined = gather_sequence(joined, group, dim=1, pad=span.length * peers - len(timestep_indices))
    return (joined.narrow(-1, 0, split).index_select(1, video_indices),
            joined.narrow(-1, split, joined.shape[-1] - split).index_select(1, audio_indices))
