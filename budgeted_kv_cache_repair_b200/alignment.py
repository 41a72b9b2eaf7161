"""Common token prefix/suffix across an edit.

Same results as ``token_alignment`` in the reference (alignment.py:6-30):
the longest common prefix, then the longest common suffix of what the prefix
leaves in the shorter sequence, and the derived offsets. The dict keys are
the reference's (callers read them), the computation is vectorised: both id
sequences become int64 arrays and the first mismatch of each direction is one
``flatnonzero`` over the compared window, so a 32k-token prompt costs a few
array passes instead of a Python loop per token.
"""

from __future__ import annotations

from typing import Sequence

import numpy as np


def _as_ids(ids: Sequence[int]) -> np.ndarray:
    return np.asarray(list(ids) if not isinstance(ids, np.ndarray) else ids, dtype=np.int64).reshape(-1)


def _equal_run(left: np.ndarray, right: np.ndarray) -> int:
    """Length of the leading stretch where two equally long windows agree."""
    mismatch = np.flatnonzero(left != right)
    return int(mismatch[0]) if mismatch.size else int(left.size)


def shared_prefix_len(left: Sequence[int], right: Sequence[int]) -> int:
    """Number of leading ids the two sequences have in common."""
    a, b = _as_ids(left), _as_ids(right)
    window = min(a.size, b.size)
    return _equal_run(a[:window], b[:window])


def shared_suffix_len(left: Sequence[int], right: Sequence[int], prefix_len: int) -> int:
    """Number of trailing ids in common, never reaching into the first
    ``prefix_len`` ids of either sequence."""
    a, b = _as_ids(left), _as_ids(right)
    window = max(0, min(a.size, b.size) - prefix_len)
    return _equal_run(a[::-1][:window], b[::-1][:window])


def token_alignment(old_ids: Sequence[int], new_ids: Sequence[int]) -> dict[str, int]:
    """Prefix/suffix alignment of the original and the edited prompt ids.

    ``position_shift`` is how far the retained suffix moves (negative for a
    deletion); ``mandatory_changed_tokens`` the edited ids between the common
    prefix and suffix, which have no counterpart in the old cache.
    """
    old, new = _as_ids(old_ids), _as_ids(new_ids)
    prefix = shared_prefix_len(old, new)
    suffix = shared_suffix_len(old, new, prefix)
    old_start, new_start = old.size - suffix, new.size - suffix
    return {
        "prefix": prefix,
        "suffix": suffix,
        "old_suffix_start": int(old_start),
        "new_suffix_start": int(new_start),
        "mandatory_changed_tokens": int(new.size - prefix - suffix),
        "position_shift": int(new_start - old_start),
    }
