"""Sequence-parallel error types, named as in
x_base/x_base/sequence_parallelism/errors.py (SequenceParallelError :9,
ParallelConfigError :41, BackendNotAvailableError :75) so callers that catch
them by name keep working."""
from __future__ import annotations

from typing import Optional


class SequenceParallelError(Exception):
    """Base of every sequence-parallel error."""


class ParallelConfigError(SequenceParallelError):
    """A parallel configuration whose sizes do not fit the world or each other."""


class BackendNotAvailableError(SequenceParallelError):
    """A communication backend the configuration asks for is not installed."""

    def __init__(self, backend_name: str, install_hint: Optional[str] = None):
        message = f"Communication backend '{backend_name}' is not available."
        if install_hint:
            message += f" Install with: {install_hint}"
        super().__init__(message)
        self.backend_name = backend_name
