"""Host and device plans for the selected rows of one request.

Mirrors ``IndexedPlan`` / ``DeviceIndexedPlan`` of the reference
(kernels/indexed_attention.py:42-158): the same constructor, fields, tile
metadata (BLOCK_M=16 query rows, BLOCK_N=64 keys: ``full_prefix_tiles`` key
tiles visible to every row of a query tile, ``total_tiles`` tiles reaching its
last row), validation messages and sealing against mutation. The sm_100a
attention kernel tiles differently (128 packed (row, head) entries per CTA) and
derives its own bounds on the device from ``positions``; the tile fields stay
for callers that read them.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from numbers import Integral
from typing import Sequence

import torch

BLOCK_M = 16
BLOCK_N = 64


_INT64_MAX = (1 << 63) - 1


def _host_length(value) -> int:
    if isinstance(value, bool) or not isinstance(value, Integral):
        raise ValueError("logical_length must be a host integer")
    if not 0 <= int(value) <= _INT64_MAX:
        raise ValueError("logical_length must fit nonnegative signed int64")
    return int(value)


def scan_positions(positions, length: int) -> tuple[tuple[int, ...], tuple[int, ...], tuple[int, ...]]:
    """Validate host positions and derive the per-tile key bounds in one pass.

    Each element is classified as it streams by (not an integer, outside
    ``[0, length)``, not above its predecessor); the pass remembers which
    kinds of fault it saw and, at the end, reports the most basic one, so the
    message for a given input is the reference's (kernels/indexed_attention.py:
    54-76 checks the three kinds in that order over the whole sequence). Tile
    bounds ride along: a 16-row tile opens at its first row
    (``full = (p + 1) // 64`` key tiles every row sees) and closes at its last
    (``total = (p + 64) // 64`` tiles reaching it).
    """
    if isinstance(positions, torch.Tensor):
        raise ValueError("positions must be host integers, not a tensor")
    try:
        items = iter(positions)
    except TypeError as error:
        raise ValueError("positions must be a sequence of host integers") from error
    values: list[int] = []
    full: list[int] = []
    total: list[int] = []
    not_int = out_of_range = unordered = False
    previous = None
    for index, item in enumerate(items):
        if isinstance(item, bool) or not isinstance(item, Integral):
            not_int = True
            continue
        p = int(item)
        out_of_range |= not 0 <= p < length
        unordered |= previous is not None and p <= previous
        previous = p
        values.append(p)
        if index % BLOCK_M == 0:
            full.append((p + 1) // BLOCK_N)
    if not_int:
        raise ValueError("positions must contain host integers")
    if out_of_range:
        raise ValueError("positions must lie within logical_length")
    if unordered:
        raise ValueError("positions must be strictly increasing and unique")
    for last in range(BLOCK_M - 1, len(values) + BLOCK_M - 1, BLOCK_M):
        total.append((values[min(last, len(values) - 1)] + BLOCK_N) // BLOCK_N)
    return tuple(values), tuple(full), tuple(total)


@dataclass(frozen=True)
class IndexedPlan:
    """Sorted absolute positions, validated entirely on the CPU.

    The constructor, public fields and error texts are the reference's
    (kernels/indexed_attention.py:42-110). Tensor positions are rejected:
    building a plan never hides a device-to-host synchronisation.
    """

    positions: Sequence[int]
    logical_length: int
    full_prefix_tiles: tuple[int, ...] = field(init=False)
    total_tiles: tuple[int, ...] = field(init=False)

    def __post_init__(self):
        length = _host_length(self.logical_length)
        positions, full, total = scan_positions(self.positions, length)
        for name, value in (("positions", positions), ("logical_length", length),
                            ("full_prefix_tiles", full), ("total_tiles", total)):
            object.__setattr__(self, name, value)

    @property
    def selected_count(self) -> int:
        return len(self.positions)

    @property
    def max_position(self) -> int:
        return self.positions[-1] if self.positions else -1

    def to(self, device) -> "DeviceIndexedPlan":
        """Upload O(B) metadata on the caller's current stream for this device."""
        if isinstance(device, int):
            device = torch.device("cuda", device)
        else:
            device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("device plan requires a CUDA device")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        from .staging import upload_int64

        with torch.cuda.device(device), torch.inference_mode(False):
            # One stream-ordered copy through the pinned staging ring (no sync).
            packed = upload_int64([*self.positions, *self.full_prefix_tiles, *self.total_tiles], device)
            count, tiles = len(self.positions), len(self.full_prefix_tiles)
            positions = packed[:count]
            full = packed[count:count + tiles]
            total = packed[count + tiles:]
        tensors = (positions, full, total)
        seal = (id(self), tuple(id(t) for t in tensors), tuple(t._version for t in tensors))
        return DeviceIndexedPlan(self, positions, full, total, seal)


@dataclass(frozen=True)
class DeviceIndexedPlan:
    """Device metadata from IndexedPlan.to; tensors are immutable by contract
    (kernels/indexed_attention.py:113-139)."""

    host_plan: IndexedPlan
    positions: torch.Tensor
    full_prefix_tiles: torch.Tensor
    total_tiles: torch.Tensor
    _seal: tuple | None = field(default=None, repr=False, compare=False)

    @property
    def logical_length(self) -> int:
        return self.host_plan.logical_length

    @property
    def selected_count(self) -> int:
        return self.host_plan.selected_count

    @property
    def device(self) -> torch.device:
        return self.positions.device


def validate_device_plan(plan, device: torch.device) -> None:
    """Reject plans that were replaced, mutated or not factory-made
    (kernels/indexed_attention.py:142-158)."""
    if not isinstance(plan, DeviceIndexedPlan) or not isinstance(plan.host_plan, IndexedPlan):
        raise ValueError("device_plan must be produced by IndexedPlan.to")
    tiles = (plan.selected_count + BLOCK_M - 1) // BLOCK_M
    for tensor, count in ((plan.positions, plan.selected_count),
                          (plan.full_prefix_tiles, tiles), (plan.total_tiles, tiles)):
        if (not isinstance(tensor, torch.Tensor) or tensor.device != device
                or not tensor.is_cuda or tensor.dtype != torch.int64
                or tensor.shape != (count,) or not tensor.is_contiguous()):
            raise ValueError("device plan has incompatible metadata shape, dtype, or device")
    tensors = (plan.positions, plan.full_prefix_tiles, plan.total_tiles)
    try:
        seal = (id(plan.host_plan), tuple(id(t) for t in tensors), tuple(t._version for t in tensors))
    except RuntimeError as error:
        raise ValueError("device plan must be produced by IndexedPlan.to") from error
    if plan._seal != seal:
        raise ValueError("device plan metadata was replaced, mutated, or not factory-created")
