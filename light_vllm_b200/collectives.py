"""Tensor-parallel collectives and AWQ shard arithmetic.

Under torchrun tensor parallelism the AWQ column shards (QKV, gate_up) and the
KV heads stay rank-local; the row-parallel outputs (o_proj, down_proj) are
partial sums that one all-reduce per block combines, and the vocab-parallel
logits are gathered along the last dimension.

* ``TensorParallelCollectives`` implements light-vllm's ``TensorCollectives``
  protocol (modeling/tensor_parallel.py:18-27) over a ``torch.distributed``
  process group: NCCL over NVLink/NVSwitch on GPUs, gloo on the CPU.  Both
  calls are stream-ordered with the caller's current stream and keep the
  reference's semantics (runtime/execution/distributed.py:190-224): the sum is
  in place; the gather pads every rank's slice to the widest partition and
  concatenates the unpadded slices in rank order.
* ``partition_dimension`` is the reference's contiguous split
  (tensor_parallel.py:62-83): leading ranks take one extra element.
* ``awq_column_shard`` / ``awq_row_shard`` slice a full AutoAWQ checkpoint
  tensor set the way ``AWQColumnParallelLinear.checkpoint_shards`` and
  ``AWQRowParallelLinear.checkpoint_shards`` declare it
  (modeling/quantization/awq.py:165-198, 272-297), including their alignment
  rules (output partitions aligned to 8 packed values, row partitions aligned
  to the group size).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist
from torch import Tensor

_PACK = 8


@dataclass(frozen=True, slots=True)
class TensorPartition:
    total_size: int
    rank: int
    world_size: int
    start: int
    end: int
    sizes: tuple[int, ...]

    @property
    def local_size(self) -> int:
        return self.end - self.start


def partition_dimension(total_size: int, rank: int, world_size: int) -> TensorPartition:
    """Contiguous split of one dimension; leading ranks take the remainder."""

    if type(total_size) is not int or total_size <= 0:
        raise ValueError("partitioned dimension must be a positive integer")
    if type(world_size) is not int or world_size <= 0:
        raise ValueError("tensor parallel world size must be a positive integer")
    if type(rank) is not int or not 0 <= rank < world_size:
        raise ValueError("tensor parallel rank must be within the world size")
    base, extra = divmod(total_size, world_size)
    sizes = tuple(base + (i < extra) for i in range(world_size))
    if any(size == 0 for size in sizes):
        raise ValueError("tensor parallel world size exceeds the partitioned dimension")
    start = sum(sizes[:rank])
    return TensorPartition(total_size, rank, world_size, start, start + sizes[rank], sizes)


def awq_column_shard(qweight: Tensor, qzeros: Tensor, scales: Tensor, bias: Tensor | None,
                     partition: TensorPartition):
    """This rank's output-column slice of a full AWQ linear."""

    if partition.start % _PACK or partition.local_size % _PACK:
        raise ValueError("AWQ tensor-parallel output partitions must align to 8 packed values")
    p0, p1 = partition.start // _PACK, partition.end // _PACK
    return (qweight[:, p0:p1].contiguous(), qzeros[:, p0:p1].contiguous(),
            scales[:, partition.start:partition.end].contiguous(),
            None if bias is None else bias[partition.start:partition.end].contiguous())


def awq_row_shard(qweight: Tensor, qzeros: Tensor, scales: Tensor, group_size: int,
                  partition: TensorPartition):
    """This rank's input-row slice of a full AWQ linear (bias is added once,
    after the all-reduce, by the caller)."""

    if group_size != partition.total_size and (partition.start % group_size
                                               or partition.local_size % group_size):
        raise ValueError("AWQ row-parallel input partitions must align to group_size")
    rows = qweight[partition.start:partition.end].contiguous()
    if group_size == partition.total_size:
        return rows, qzeros.contiguous(), scales.contiguous()
    g0, g1 = partition.start // group_size, partition.end // group_size
    return rows, qzeros[g0:g1].contiguous(), scales[g0:g1].contiguous()


class TensorParallelCollectives:
    """``TensorCollectives`` over a torch.distributed group (NCCL or gloo)."""

    def __init__(self, group: dist.ProcessGroup | None = None) -> None:
        if not dist.is_initialized():
            raise RuntimeError("torch.distributed must be initialised before building collectives")
        self._group = group
        self.world_size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def all_reduce_sum(self, tensor: Tensor) -> Tensor:
        if not tensor.is_contiguous():
            raise ValueError("tensor-parallel all-reduce requires a contiguous tensor")
        if self.world_size > 1:
            dist.all_reduce(tensor, op=dist.ReduceOp.SUM, group=self._group)
        return tensor

    def all_gather_last_dim(self, tensor: Tensor, partition_sizes: tuple[int, ...]) -> Tensor:
        if len(partition_sizes) != self.world_size:
            raise ValueError("gather partitions must contain one size per rank")
        if tensor.shape[-1] != partition_sizes[self.rank]:
            raise ValueError("local tensor width does not match its gather partition")
        if self.world_size == 1:
            return tensor
        widest = max(partition_sizes)
        if tensor.shape[-1] < widest:
            pad = tensor.new_zeros(*tensor.shape[:-1], widest - tensor.shape[-1])
            tensor = torch.cat((tensor, pad), dim=-1)
        tensor = tensor.contiguous()
        flat = tensor.new_empty((self.world_size * tensor.numel(),))
        dist.all_gather_into_tensor(flat, tensor.view(-1), group=self._group)
        gathered = flat.view(self.world_size, *tensor.shape)
        return torch.cat([gathered[r][..., :size] for r, size in enumerate(partition_sizes)], dim=-1)
