"""One pinned host-to-device copy for all of a step's small integer arrays.

Same contract as the reference's ``SingleStepCudaStagingBuffer``
(runtime/execution/cuda_staging.py:11-70): the returned device views stay valid
until the next ``copy_groups`` call, and only an earlier copy (not later
compute) is waited for before a pinned buffer is reused.
"""

from __future__ import annotations

import ctypes
import weakref
from collections.abc import Callable, Sequence

import numpy as np
import torch
from torch import Tensor

from light_vllm_b200 import _native


def _destroy_events(lib, events: list) -> None:
    for event in events:
        if event is not None:
            lib.lvb_event_destroy(event)  # best effort: the context may already be gone


class SingleStepStaging:
    """Pinned int32 staging area with one H2D copy per step.

    The pinned side is a ring of ``RING`` host buffers: a step fills the slot
    whose copy was issued ``RING`` steps earlier, so the host waits only if it
    has run that many steps ahead of the GPU, and then by polling the slot's
    event (a blocking-sync event sleeps the thread and costs tens to hundreds
    of microseconds of wake-up latency per step).  Slot events are native
    (``lvb_event_*``); ``stage`` lets one native call wait for the slot, fill
    it, issue the copy and record the event (``lvb_stage_step_metadata``).
    One device buffer receives every copy in stream order.
    """

    RING = 4

    def __init__(self, device: torch.device) -> None:
        if device.type != "cuda":
            raise ValueError("CUDA staging requires a CUDA device")
        self._device = device
        self._lib = _native.library()
        self._hosts: list[Tensor | None] = [None] * self.RING
        self._events: list[int | None] = [None] * self.RING
        self._slot = 0
        self._dev: Tensor | None = None
        weakref.finalize(self, _destroy_events, self._lib, self._events)

    def _event(self, slot: int) -> int:
        event = self._events[slot]
        if event is None:
            handle = ctypes.c_void_p()
            with torch.cuda.device(self._device):
                _native.check(self._lib.lvb_event_create(ctypes.byref(handle)), "lvb_event_create")
            event = self._events[slot] = handle.value
        return event

    def _next_slot(self, required: int) -> tuple[int, Tensor, Tensor]:
        """The next ring slot's pinned buffer (at least ``required`` values) and
        the device buffer, grown to match.  The caller waits on the slot's
        event before writing the pinned buffer."""

        slot = self._slot
        self._slot = (slot + 1) % self.RING
        capacity = 1 << max(0, (required - 1).bit_length())
        host = self._hosts[slot]
        if host is None or host.numel() < required:
            if self._events[slot] is not None:
                # A native copy may still read the old buffer; the pinned
                # allocator does not know about it, so wait before letting go.
                _native.check(self._lib.lvb_event_wait_host(self._events[slot]), "lvb_event_wait_host")
            host = torch.empty(capacity, dtype=torch.int32, pin_memory=True)
            self._hosts[slot] = host
        if self._dev is None or self._dev.numel() < required:
            self._dev = torch.empty(capacity, dtype=torch.int32, device=self._device)
        return slot, host, self._dev

    def _stream(self) -> int:
        return _native.stream_handle(self._device)

    def copy_groups(self, *groups: Sequence[int] | np.ndarray) -> tuple[Tensor, ...]:
        lengths = [len(group) for group in groups]
        total = sum(lengths)
        if total == 0:
            raise ValueError("CUDA staging requires at least one value")
        dev = self.copy_packed(total, lambda host: self._fill_groups(host, groups, lengths))
        views = []
        offset = 0
        for length in lengths:
            views.append(dev[offset : offset + length])
            offset += length
        return tuple(views)

    @staticmethod
    def _fill_groups(host_t: Tensor, groups, lengths) -> int:
        host = host_t.numpy()
        offset = 0
        for group, length in zip(groups, lengths):
            host[offset : offset + length] = np.asarray(group, dtype=np.int32)
            offset += length
        return offset

    def copy_packed(self, capacity: int, fill: Callable[[Tensor], int]) -> Tensor:
        """Let ``fill(host_int32_view)`` write up to ``capacity`` values into a
        pinned buffer and return how many it wrote; one H2D copy follows.  The
        returned device view stays valid until the next copy."""

        slot, host, dev = self._next_slot(capacity)
        event = self._event(slot)
        _native.check(self._lib.lvb_event_wait_host(event), "lvb_event_wait_host")
        total = int(fill(host))
        dev[:total].copy_(host[:total], non_blocking=True)
        _native.check(self._lib.lvb_event_record(event, self._stream()), "lvb_event_record")
        return dev[:total]

    def stage(self, capacity: int, run: Callable[[int, int, int, int, int, int], int]) -> Tensor:
        """``run(pinned_ptr, pinned_capacity, device_ptr, device_capacity,
        slot_event, stream)`` waits for the slot, fills it, copies and records
        the event natively, returning how many values it staged."""

        slot, host, dev = self._next_slot(capacity)
        total = int(run(host.data_ptr(), host.numel(), dev.data_ptr(), dev.numel(), self._event(slot),
                        self._stream()))
        return dev[:total]

    def slot(self, capacity: int) -> tuple[Tensor, int, int, int, int, int, int]:
        """The next ring slot for a native stager: (device buffer, pinned
        address, pinned capacity, device address, device capacity, slot
        event, stream).  The device buffer is returned whole (the payload
        starts at its first value); keep it alive while launches read it."""

        slot, host, dev = self._next_slot(capacity)
        return dev, host.data_ptr(), host.numel(), dev.data_ptr(), dev.numel(), self._event(slot), self._stream()
