"""Opt-in CUDA-event timeline of the SP attention layer's stages.

While a timeline is open (`start()` ... `stop()`), the SP path records a
timing event at each stage boundary on the stream that runs the stage:

  start      the layer begins (compute stream)
  gathered   the Q/K/V wire has arrived from every peer (comm stream)
  prepared   the Sage operands are written (compute stream)
  attended   the attention output is written (compute stream)
  returned   the output wire has arrived from every peer (comm stream)
  decoded    the output is decoded into the layer's result (comm stream)
  end        the compute stream has joined the exchange (compute stream)

Stages are ordered by their dependencies, so the time between consecutive
marks is the time each stage added to the layer. With no timeline open,
`mark` does nothing.
"""
from __future__ import annotations

import torch

_events: list | None = None


def start() -> None:
    """Open a timeline; marks recorded from now on are kept."""
    global _events
    _events = []


def mark(name: str, stream: torch.cuda.Stream | None = None) -> None:
    """Record `name` on `stream` (default: the current stream) if a timeline is open."""
    if _events is None:
        return
    ev = torch.cuda.Event(enable_timing=True)
    ev.record(stream if stream is not None else torch.cuda.current_stream())
    _events.append((name, ev))


def stop() -> list:
    """Close the timeline; returns [(name, event), ...] in recording order."""
    global _events
    events, _events = _events or [], None
    return events


def stage_ms(events: list) -> dict:
    """Milliseconds between each mark and the previous one (call after the
    events have completed), summed per stage name."""
    out: dict = {}
    for (_, prev), (name, ev) in zip(events, events[1:]):
        out[name] = out.get(name, 0.0) + prev.elapsed_time(ev)
    return out
