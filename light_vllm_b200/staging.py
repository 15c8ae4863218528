"""One pinned host-to-device copy for all of a step's small integer arrays.

Same contract as the reference's ``SingleStepCudaStagingBuffer``
(runtime/execution/cuda_staging.py:11-70): the returned device views stay valid
until the next ``copy_groups`` call, and only an earlier copy (not later
compute) is waited for before a pinned buffer is reused.
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np
import torch
from torch import Tensor


class SingleStepStaging:
    """Pinned int32 staging area with one H2D copy per step.

    The pinned side is a ring of ``RING`` host buffers: a step fills the slot
    whose copy was issued ``RING`` steps earlier, so the host waits only if it
    has run that many steps ahead of the GPU, and then by polling the slot's
    event (a blocking-sync event sleeps the thread and costs tens to hundreds
    of microseconds of wake-up latency per step).  One device buffer receives
    every copy in stream order.
    """

    RING = 4

    def __init__(self, device: torch.device) -> None:
        if device.type != "cuda":
            raise ValueError("CUDA staging requires a CUDA device")
        self._device = device
        self._hosts: list[Tensor | None] = [None] * self.RING
        self._events: list[torch.cuda.Event | None] = [None] * self.RING
        self._slot = 0
        self._dev: Tensor | None = None

    def _acquire(self, required: int) -> tuple[int, Tensor]:
        """The next ring slot's pinned buffer, free to overwrite and holding at
        least ``required`` values; the device buffer grows to match."""

        slot = self._slot
        self._slot = (slot + 1) % self.RING
        event = self._events[slot]
        if event is not None and not event.query():
            event.synchronize()
        capacity = 1 << max(0, (required - 1).bit_length())
        host = self._hosts[slot]
        if host is None or host.numel() < required:
            host = torch.empty(capacity, dtype=torch.int32, pin_memory=True)
            self._hosts[slot] = host
        if self._dev is None or self._dev.numel() < required:
            self._dev = torch.empty(capacity, dtype=torch.int32, device=self._device)
        return slot, host

    def _issue(self, slot: int, host: Tensor, total: int) -> Tensor:
        dev = self._dev
        assert dev is not None
        dev[:total].copy_(host[:total], non_blocking=True)
        event = self._events[slot]
        if event is None:
            event = self._events[slot] = torch.cuda.Event()
        event.record(torch.cuda.current_stream(self._device))
        return dev

    def copy_groups(self, *groups: Sequence[int] | np.ndarray) -> tuple[Tensor, ...]:
        lengths = [len(group) for group in groups]
        total = sum(lengths)
        if total == 0:
            raise ValueError("CUDA staging requires at least one value")
        slot, host_t = self._acquire(total)
        host = host_t.numpy()
        offset = 0
        for group, length in zip(groups, lengths):
            host[offset : offset + length] = np.asarray(group, dtype=np.int32)
            offset += length
        dev = self._issue(slot, host_t, total)
        views = []
        offset = 0
        for length in lengths:
            views.append(dev[offset : offset + length])
            offset += length
        return tuple(views)

    def copy_packed(self, capacity: int, fill) -> Tensor:
        """Let ``fill(host_int32_view)`` write up to ``capacity`` values into a
        pinned buffer and return how many it wrote; one H2D copy follows.  The
        returned device view stays valid until the next copy."""

        slot, host = self._acquire(capacity)
        total = int(fill(host))
        return self._issue(slot, host, total)[:total]
