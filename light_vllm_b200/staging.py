"""One pinned host-to-device copy for all of a step's small integer arrays.

Same contract as the reference's ``SingleStepCudaStagingBuffer``
(runtime/execution/cuda_staging.py:11-70): the returned device views stay valid
until the next ``copy_groups`` call, and only the previous copy (not later
compute) is waited for before the pinned buffer is reused.
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np
import torch
from torch import Tensor


class SingleStepStaging:
    """Pinned int32 staging area with one H2D copy per step."""

    def __init__(self, device: torch.device) -> None:
        if device.type != "cuda":
            raise ValueError("CUDA staging requires a CUDA device")
        self._device = device
        self._host: Tensor | None = None
        self._dev: Tensor | None = None
        self._copied: torch.cuda.Event | None = None

    def copy_groups(self, *groups: Sequence[int] | np.ndarray) -> tuple[Tensor, ...]:
        lengths = [len(group) for group in groups]
        total = sum(lengths)
        if total == 0:
            raise ValueError("CUDA staging requires at least one value")
        if self._copied is not None:
            self._copied.synchronize()
        self._reserve(total)
        assert self._host is not None and self._dev is not None
        host = self._host.numpy()
        offset = 0
        for group, length in zip(groups, lengths):
            host[offset : offset + length] = np.asarray(group, dtype=np.int32)
            offset += length
        self._dev[:total].copy_(self._host[:total], non_blocking=True)
        if self._copied is None:
            self._copied = torch.cuda.Event(blocking=True)
        self._copied.record(torch.cuda.current_stream(self._device))
        views = []
        offset = 0
        for length in lengths:
            views.append(self._dev[offset : offset + length])
            offset += length
        return tuple(views)

    def copy_packed(self, capacity: int, fill) -> Tensor:
        """Let ``fill(host_int32_view)`` write up to ``capacity`` values into the
        pinned buffer and return how many it wrote; one H2D copy follows.  The
        returned device view stays valid until the next copy."""

        if self._copied is not None:
            self._copied.synchronize()
        self._reserve(capacity)
        assert self._host is not None and self._dev is not None
        total = int(fill(self._host))
        self._dev[:total].copy_(self._host[:total], non_blocking=True)
        if self._copied is None:
            self._copied = torch.cuda.Event(blocking=True)
        self._copied.record(torch.cuda.current_stream(self._device))
        return self._dev[:total]

    def _reserve(self, required: int) -> None:
        if self._dev is not None and self._dev.numel() >= required:
            return
        capacity = 1 << max(0, (required - 1).bit_length())
        # Device views are 16-byte aligned at every group start the caller
        # relies on only through element offsets; int32 is all we need.
        self._host = torch.empty(capacity, dtype=torch.int32, pin_memory=True)
        self._dev = torch.empty(capacity, dtype=torch.int32, device=self._device)
