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
* ``PeerWorkspace`` + ``all_reduce_add_rms_norm``: the row-parallel epilogue
  of a Qwen2 block (all-reduce, residual add, RMSNorm) as one launch that
  reads the ranks' partial sums over NVLink peer memory; the workspaces are
  shared through CUDA IPC handles exchanged over the process group.
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


class PeerWorkspace:
    """One peer-writable workspace per rank, mapped by every rank of the group.

    Each rank allocates its workspace with ``lvb_ipc_alloc`` and the ranks
    exchange the CUDA IPC handles over the process group; afterwards
    ``pointers`` holds every rank's workspace as mapped in this process, the
    argument of ``lvb_allreduce_add_rmsnorm``.  All ranks must build and close
    it together (it is a collective).  Without a process group it serves a
    single rank.  The call counter lives in the workspace itself, so the
    launches that use it can be captured in CUDA graphs.
    """

    def __init__(self, max_tokens: int, hidden: int, device: torch.device,
                 group: dist.ProcessGroup | None = None, *, distributed: bool = True) -> None:
        import ctypes

        from light_vllm_b200 import _native

        self._lib = _native.library()
        self._native = _native
        self.max_tokens = int(max_tokens)
        self.hidden = int(hidden)
        self.device = torch.device(device)
        self._group = group
        self.group = group
        use_dist = distributed and dist.is_initialized()
        self.world_size = dist.get_world_size(group) if use_dist else 1
        self.rank = dist.get_rank(group) if use_dist else 0
        nbytes = int(self._lib.lvb_allreduce_workspace_bytes(self.world_size, self.max_tokens, self.hidden))
        if nbytes == 0:
            raise ValueError("invalid all-reduce workspace shape")
        self.nbytes = nbytes
        own = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        with torch.cuda.device(self.device):
            _native.check(self._lib.lvb_ipc_alloc(nbytes, ctypes.byref(own), handle), "lvb_ipc_alloc")
            _native.check(self._lib.lvb_allreduce_workspace_init(own.value, self.world_size, self.max_tokens,
                                                                 self.hidden), "lvb_allreduce_workspace_init")
        self._own = own.value
        handles = [handle.raw]
        if self.world_size > 1:
            handles = [None] * self.world_size
            dist.all_gather_object(handles, handle.raw, group=group)
        pointers = []
        self._opened = []
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    pointers.append(self._own)
                    continue
                ptr = ctypes.c_void_p()
                _native.check(self._lib.lvb_ipc_open(h, ctypes.byref(ptr)), "lvb_ipc_open")
                pointers.append(ptr.value)
                self._opened.append(ptr.value)
        self.pointers = (ctypes.c_void_p * self.world_size)(*pointers)

    def close(self) -> None:
        """Unmap the peers' workspaces and free this rank's (collective)."""

        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world_size > 1:
            dist.barrier(group=self._group)  # no rank still pushes into a workspace
        with torch.cuda.device(self.device):
            for ptr in self._opened:
                self._native.check(self._lib.lvb_ipc_close(ptr), "lvb_ipc_close")
        self._opened = []
        if self.world_size > 1:
            dist.barrier(group=self._group)  # every peer has unmapped this rank's workspace
        with torch.cuda.device(self.device):
            self._native.check(self._lib.lvb_ipc_free(self._own), "lvb_ipc_free")
        self._own = None


ALL_REDUCE_AUTO, ALL_REDUCE_ONE_SHOT, ALL_REDUCE_TWO_SHOT, ALL_REDUCE_SENTINEL, ALL_REDUCE_SENTINEL_TWO_SHOT = 0, 1, 2, 3, 4


def _check_rows(workspace: PeerWorkspace, tensor: Tensor, what: str) -> None:
    if tensor.dim() != 2 or tensor.dtype != torch.float16 or not tensor.is_contiguous():
        raise ValueError(f"{what} must be a contiguous fp16 [tokens, hidden] tensor")
    if tensor.device != workspace.device:
        raise ValueError(f"{what} is on {tensor.device}, the workspace on {workspace.device}")
    if tensor.shape[1] != workspace.hidden:
        raise ValueError("hidden size does not match the all-reduce workspace")
    if tensor.shape[0] > workspace.max_tokens:
        raise ValueError("more tokens than the all-reduce workspace holds")


def _peer_path(workspace: PeerWorkspace, tensor: Tensor, mode: int) -> bool:
    """Whether the peer-memory kernel does the exchange (else NCCL does)."""

    if mode != ALL_REDUCE_AUTO or workspace.world_size == 1:
        return True
    from light_vllm_b200 import _native

    limit = int(_native.library().lvb_allreduce_peer_max_bytes(workspace.world_size))
    return tensor.numel() * tensor.element_size() <= limit


def _launch(workspace: PeerWorkspace, partial: Tensor, residual: Tensor | None, weight: Tensor | None,
            out: Tensor, eps: float, mode: int, *, local: bool = False) -> None:
    """``local``: the ranks' sum is already in ``partial`` (world 1 launch)."""

    from light_vllm_b200 import _native

    rank, world = (0, 1) if local else (workspace.rank, workspace.world_size)
    _native.check(
        _native.library().lvb_allreduce_add_rmsnorm(
            workspace.pointers, rank, world, partial.data_ptr(),
            0 if residual is None else residual.data_ptr(), 0 if weight is None else weight.data_ptr(),
            out.data_ptr(), partial.shape[0], partial.shape[1], workspace.max_tokens, float(eps), int(mode),
            _native.stream_handle(partial.device)),
        "lvb_allreduce_add_rmsnorm",
    )


def all_reduce_add_rms_norm(workspace: PeerWorkspace, partial: Tensor, residual: Tensor,
                            weight: Tensor, eps: float, *, mode: int = ALL_REDUCE_AUTO) -> tuple[Tensor, Tensor]:
    """Sum ``partial`` over the ranks, add ``residual`` and RMSNorm the result,
    in one sm_100a launch over peer memory (``lvb_allreduce_add_rmsnorm``).

    Returns ``(normed, residual)``; ``residual`` is updated in place, like
    ``fused_add_rms_norm`` after ``all_reduce_sum`` in the reference
    (modeling/models/qwen2.py:497-514, _qwen2_kernels.py:145-180).  Every rank
    calls it with the same shapes in the same order.
    """

    _check_rows(workspace, partial, "partial")
    _check_rows(workspace, residual, "residual")
    if partial.shape != residual.shape:
        raise ValueError("partial and residual must have one shape")
    if residual.data_ptr() == partial.data_ptr():
        raise ValueError("residual must not alias partial")
    if weight.dtype != torch.float16 or weight.shape != (workspace.hidden,) or not weight.is_contiguous():
        raise ValueError("weight must be a contiguous fp16 [hidden] tensor")
    out = torch.empty_like(partial)
    if _peer_path(workspace, partial, mode):
        _launch(workspace, partial, residual, weight, out, eps, mode)
    else:
        # Large messages: NCCL's ring all-reduce in place (the reference's
        # all_reduce_sum), then the add + RMSNorm without an exchange.
        dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=workspace.group)
        _launch(workspace, partial, residual, weight, out, eps, mode, local=True)
    return out, residual


def all_reduce_sum_peer(workspace: PeerWorkspace, tensor: Tensor, *, mode: int = ALL_REDUCE_AUTO) -> Tensor:
    """In-place fp16 sum over the ranks through peer memory (the contract of
    ``TensorCollectives.all_reduce_sum``, modeling/tensor_parallel.py:18-27)."""

    _check_rows(workspace, tensor, "tensor")
    if _peer_path(workspace, tensor, mode):
        _launch(workspace, tensor, None, None, tensor, 0.0, mode)
    else:
        dist.all_reduce(tensor, op=dist.ReduceOp.SUM, group=workspace.group)
    return tensor


class PeerCollectives(TensorParallelCollectives):
    """``TensorParallelCollectives`` whose fp16 row sums run through the
    peer-memory kernel, plus the fused ``all_reduce_add_rms_norm`` a Qwen2
    layer uses after its row-parallel projections.  Tensors the workspace
    does not cover (other dtypes, wider rows, more tokens) take the NCCL
    path of the base class."""

    def __init__(self, workspace: PeerWorkspace, group: dist.ProcessGroup | None = None) -> None:
        super().__init__(group)
        self.workspace = workspace

    def _covers(self, tensor: Tensor) -> bool:
        ws = self.workspace
        return (tensor.dtype == torch.float16 and tensor.is_contiguous() and tensor.dim() >= 1
                and tensor.shape[-1] == ws.hidden and tensor.numel() // ws.hidden <= ws.max_tokens
                and tensor.device == ws.device)

    def all_reduce_sum(self, tensor: Tensor) -> Tensor:
        if not self._covers(tensor):
            return super().all_reduce_sum(tensor)
        all_reduce_sum_peer(self.workspace, tensor.view(-1, self.workspace.hidden))
        return tensor

    def all_reduce_add_rms_norm(self, partial: Tensor, residual: Tensor, weight: Tensor,
                                eps: float) -> tuple[Tensor, Tensor]:
        shape = partial.shape
        out, res = all_reduce_add_rms_norm(self.workspace, partial.view(-1, shape[-1]),
                                           residual.view(-1, shape[-1]), weight, eps)
        return out.view(shape), residual
