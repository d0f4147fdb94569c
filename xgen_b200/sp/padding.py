"""Sequence-parallel padding registry.

Same contract as x_base/x_base/sequence_parallelism/padding.py:18-92: a
named pad per sequence key, pad = (sp - S % sp) % sp, `get` raising when a
key was never set. The H3 processor uses key "mmh3_seq"
(x_diffusers/x_diffusers/framework/transformer/minimax_h3.py:377).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, Optional

from .errors import SequenceParallelError


class PadNotSetError(SequenceParallelError, KeyError):
    """Raised when a padding key is read before it was set
    (x_base/x_base/sequence_parallelism/errors.py:17)."""

    def __init__(self, name: str):
        super().__init__(f"padding for '{name}' has not been set")
        self.name = name


@dataclass
class PadManager:
    _pads: Dict[str, int] = field(default_factory=dict)

    def set(self, name: str, dim_size: int, sp_size: int) -> int:
        pad = (sp_size - (dim_size % sp_size)) % sp_size
        self._pads[name] = pad
        return pad

    def set_from_group(self, name: str, dim_size: int, group) -> int:
        import torch.distributed as dist

        return self.set(name, dim_size, dist.get_world_size(group))

    def get(self, name: str) -> int:
        if name not in self._pads:
            raise PadNotSetError(name)
        return self._pads[name]

    def get_or_default(self, name: str, default: int = 0) -> int:
        return self._pads.get(name, default)

    def is_set(self, name: str) -> bool:
        return name in self._pads

    def clear(self) -> None:
        self._pads.clear()


_pad_manager: Optional[PadManager] = None


def get_pad_manager() -> PadManager:
    global _pad_manager
    if _pad_manager is None:
        _pad_manager = PadManager()
    return _pad_manager


def set_pad(name: str, dim_size: int, parallel_group) -> int:
    import torch.distributed as dist

    return get_pad_manager().set(name, dim_size, dist.get_world_size(parallel_group))


def get_pad(name: str) -> int:
    return get_pad_manager().get(name)
