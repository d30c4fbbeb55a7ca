"""Argument normalisation shared by the functional and module APIs.

Mirrors the reference's ``_geometry.py`` contract (``DEFAULT_WORKSPACE_BYTES`` and the
``_tuple`` messages, ``src/torch_convnd/_geometry.py:5-41``) so that callers see the same
errors.
"""

from __future__ import annotations

from collections.abc import Sequence

# The reference's default patch budget (64 MiB). The B200 kernels never build patch
# matrices; the value is still validated so the operator contract is unchanged.
DEFAULT_WORKSPACE_BYTES = 64 * 1024 * 1024


def has_rank(ndim: int, rank: int) -> bool:
    """Whether ``ndim`` dimensions hold a batched or an unbatched rank-``rank`` input."""
    return ndim == rank + 2 or ndim == rank + 1


def _tuple(value: int | Sequence[int], rank: int, name: str) -> tuple[int, ...]:
    """Expand an int to ``rank`` copies or check a sequence of exactly ``rank`` ints."""
    if isinstance(value, int) and not isinstance(value, bool):
        return (value,) * rank
    if isinstance(value, (str, bytes)) or not isinstance(value, Sequence):
        raise TypeError(f"{name} must be an integer or a sequence of integers")
    result = tuple(value)
    if len(result) != rank or any(not isinstance(v, int) or isinstance(v, bool) for v in result):
        raise ValueError(f"{name} must contain exactly {rank} integers")
    return result
