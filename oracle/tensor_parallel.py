"""CPU restatement of the tensor-parallel row-parallel epilogue (test oracle).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

The reference combines the ranks' partial sums with ``all_reduce_sum``
(modeling/tensor_parallel.py:18-27; an fp16 NCCL sum on GPUs) and then calls
``fused_add_rms_norm`` (modeling/models/_qwen2_kernels.py:145-180), whose CPU
path is ``residual = hidden + residual`` followed by ``F.rms_norm`` and whose
Triton path (lines 20-43) computes in fp32 and stores both results in the
tensor dtype.
"""

from __future__ import annotations

import torch
from torch.nn import functional as F


def all_reduce_add_rms_norm(partials, residual: torch.Tensor, weight: torch.Tensor,
                            eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """``(normed, new_residual)`` for fp16 ``partials`` (one per rank).

    The sum over ranks is taken in fp32 and rounded to fp16 (the all-reduced
    tensor), then the residual add and the norm follow the Triton kernel in
    fp32 (``_qwen2_kernels.py:33-43``).
    """

    total = torch.stack([p.float() for p in partials]).sum(0).half()
    values = total.float() + residual.float()
    normed = F.rms_norm(values, (values.shape[-1],), weight.float(), eps)
    return normed.half(), values.half()
