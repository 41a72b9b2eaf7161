"""Host-to-device upload of small per-request metadata without stalls.

Pinning host memory per request (``tensor.pin_memory()``) goes through the
pinned-memory allocator, which can wait for the GPU to drain earlier work; a
pageable ``torch.tensor(..., device=...)`` copy synchronises the stream. Both
serialise the host behind the GPU. This module keeps one pinned ring of
staging slots per process: a request's positions or ids are written into the
next slot and copied with ``cudaMemcpyAsync`` on the caller's stream; a slot
is reused only after the event of its previous copy has completed (a copy
issued many requests ago, so the wait is normally free).
"""

from __future__ import annotations

import threading

import torch

SLOTS = 16
SLOT_BYTES = 1 << 19  # 512 KiB: 65536 int64 values


class _Ring:
    def __init__(self):
        self.lock = threading.Lock()
        self.buffer = None
        self.events = [None] * SLOTS
        self.next = 0

    def upload(self, values, device: torch.device) -> torch.Tensor:
        """int64 device tensor with ``values`` (a host sequence or CPU tensor)."""
        host_values = values if isinstance(values, torch.Tensor) else torch.tensor(values, dtype=torch.int64)
        host_values = host_values.reshape(-1).to(torch.int64)
        count = host_values.numel()
        out = torch.empty(count, dtype=torch.int64, device=device)
        if count == 0:
            return out
        if count * 8 > SLOT_BYTES:  # rare: very long prompts; one-off pinned buffer
            out.copy_(host_values.pin_memory(), non_blocking=True)
            return out
        with self.lock:
            if self.buffer is None:
                self.buffer = torch.empty(SLOTS * SLOT_BYTES, dtype=torch.uint8).pin_memory()
            slot = self.next
            self.next = (slot + 1) % SLOTS
            event = self.events[slot]
            if event is not None:
                event.synchronize()
            host = self.buffer[slot * SLOT_BYTES: slot * SLOT_BYTES + count * 8].view(torch.int64)
            host.copy_(host_values)
            with torch.cuda.device(device):
                out.copy_(host, non_blocking=True)
                done = torch.cuda.Event()
                done.record()
            self.events[slot] = done
        return out


_ring = _Ring()


def upload_int64(values, device) -> torch.Tensor:
    return _ring.upload(values, torch.device(device))
