"""B200 paged-attention backend (drop-in ``PagedAttentionBackend``).

``B200PagedAttentionBackend().create(cache, metadata)`` returns a context whose
``forward(layer_id, query, key, value, *, scale)`` writes this step's K/V into
the paged cache and attends, exactly the contract of
``PagedAttentionBackend`` / ``AttentionContext.forward``
(runtime/execution/paged_attention.py:209-223, modeling/attention/interfaces.py:48-62).
It replaces ``TritonPagedAttentionBackend``
(runtime/execution/triton_paged_attention.py:399-581) with the sm_100a kernels
of ``lvb_paged_kv_write`` and ``lvb_paged_attention``:

* per step, the block tables, computed counts, query starts, request
  indices and the decode launch order (longest context first) go to the GPU
  in one pinned copy and are shared by every layer;
* decode steps (one linear query per request) take the split-context kernel;
  prefill chunks, mixed batches and tree layouts the tensor-core tile kernel,
  with a mixed batch's one-token requests on the split-context kernel (head
  sizes 32 / 80 / 256 run a scalar kernel);
* errors follow the reference: ``KVCacheError`` for a repeated layer, a shape,
  dtype or device mismatch, and any block-table violation.

No attention arithmetic runs on the CPU; the host side only gathers,
validates and stages the step metadata, in native code.
"""

from __future__ import annotations

import ctypes
import weakref
from typing import NamedTuple

import numpy as np
import torch
from torch import Tensor

from light_vllm_b200 import _native
from light_vllm_b200.kv_cache import KVCacheError
from light_vllm_b200.staging import SingleStepStaging

_SUPPORTED_DTYPES = (torch.float16, torch.bfloat16)


def _heads_contiguous(t: Tensor, *, align: int) -> Tensor:
    """A [tokens, heads, dim] view usable by the kernels without a copy when
    heads and dims are dense and rows keep ``align``-element alignment."""

    if t.is_contiguous():
        # Dense rows: row stride heads x dim; only alignment to check.
        if t.data_ptr() % (2 * align) == 0 and (t.shape[1] * t.shape[2]) % align == 0:
            return t
    elif (t.stride(2) == 1 and t.stride(1) == t.shape[2] and t.stride(0) % align == 0
            and t.data_ptr() % (2 * align) == 0):
        return t
    return t.contiguous()


class StepShape(NamedTuple):
    num_seqs: int
    total_blocks: int
    max_blocks: int
    num_tokens: int
    max_query_len: int
    max_seq_len: int
    linear: bool
    num_single: int  # requests with one query token (listed first in the launch order)

    @property
    def packed_size(self) -> int:
        """int32 values of the packed payload: padded tables, computed counts,
        query starts, request indices, launch order (longest context first)
        with the listed requests' computed counts."""
        return self.num_seqs * self.max_blocks + 4 * self.num_seqs + 1 + self.num_tokens


class StepMetadataPacker:
    """Host half of a step's metadata, with buffers reused across steps.

    ``gather`` reads a ``PagedAttentionMetadata`` (its tuples of Python ints)
    into flat C arrays through the ``_hostpack`` module; ``pack`` runs
    ``lvb_pack_step_metadata`` on them: the reference's block-table checks
    (runtime/execution/paged_attention.py:138-172, same order and messages),
    then the padded tables, computed counts, query starts, request indices
    and decode launch order written into the caller's int32 buffer; ``stage``
    does the same into a pinned staging slot and issues the device copy
    (``lvb_stage_step_metadata``).  All of it is native; the Python here only
    sizes buffers.
    """

    def __init__(self) -> None:
        self._hostpack = _native.hostpack()
        self._lib = _native.library()
        self._ids = np.empty(0, dtype=np.int32)
        self._offsets = np.empty(0, dtype=np.int64)
        self._rows = np.empty(0, dtype=np.int32)
        self._ids_ptr = self._offsets_ptr = self._rows_ptr = 0
        self._stride = ctypes.c_int64(0)
        self._ntok = ctypes.c_int64(0)
        self._stride_ref = ctypes.byref(self._stride)
        self._ntok_ref = ctypes.byref(self._ntok)
        self._step: StepShape | None = None

    def _reserve(self, num_seqs: int, total_blocks: int) -> None:
        if self._ids.size < max(total_blocks, 1):
            self._ids = np.empty(1 << max(total_blocks - 1, 1).bit_length(), dtype=np.int32)
            self._ids_ptr = self._ids.ctypes.data
        if self._offsets.size < num_seqs + 1:
            self._offsets = np.empty(1 << num_seqs.bit_length(), dtype=np.int64)
            self._rows = np.empty(4 * self._offsets.size, dtype=np.int32)
            self._offsets_ptr = self._offsets.ctypes.data
            self._rows_ptr = self._rows.ctypes.data

    def gather(self, metadata) -> StepShape:
        tables = metadata.block_tables
        n = len(tables)
        if self._offsets.size < n + 1:
            self._reserve(n, sum(map(len, tables)))
        try:
            total, max_blocks, ntok, max_q, max_seq, linear, single = self._hostpack.gather_step(
                tables, metadata.num_computed_tokens, metadata.query_layouts,
                metadata.num_reserved_query_tokens, metadata.num_readonly_prefix_blocks,
                self._ids_ptr, self._ids.size, self._offsets_ptr, self._rows_ptr)
        except ValueError:
            # The block-id buffer is too small for this step: grow it, retry.
            needed = sum(map(len, tables))
            if needed <= self._ids.size:
                raise
            self._reserve(n, needed)
            total, max_blocks, ntok, max_q, max_seq, linear, single = self._hostpack.gather_step(
                tables, metadata.num_computed_tokens, metadata.query_layouts,
                metadata.num_reserved_query_tokens, metadata.num_readonly_prefix_blocks,
                self._ids_ptr, self._ids.size, self._offsets_ptr, self._rows_ptr)
        self._step = StepShape(n, total, max_blocks, ntok, max_q, max_seq, linear, single)
        return self._step

    def pack(self, num_blocks: int, block_size: int, out_ptr: int, out_capacity: int) -> None:
        """Validate the gathered step and write its payload (``packed_size``
        int32 values) at ``out_ptr``; raises ``KVCacheError`` with the
        reference's message for a block-table violation."""

        step = self._step
        if step is None:
            raise RuntimeError("StepMetadataPacker.pack before gather")
        n = step.num_seqs
        rows = self._rows_ptr
        _native.check(
            self._lib.lvb_pack_step_metadata(
                self._ids_ptr, self._offsets_ptr, rows, rows + 4 * n, rows + 8 * n,
                rows + 12 * n, n, num_blocks, block_size, out_ptr, out_capacity,
                self._stride_ref, self._ntok_ref),
            "lvb_pack_step_metadata")

    def stage(self, staging: SingleStepStaging, num_blocks: int, block_size: int) -> Tensor:
        """Validate, pack and copy the gathered step to the device in one
        native call (``lvb_stage_step_metadata``) through a staging slot;
        returns the device buffer whose first ``packed_size`` int32 values
        are the payload."""

        step = self._step
        if step is None:
            raise RuntimeError("StepMetadataPacker.stage before gather")
        dev, host_ptr, host_cap, dev_ptr, dev_cap, event, stream = staging.slot(step.packed_size)
        status, _, _ = self._hostpack.stage_step(self._ids_ptr, self._offsets_ptr, self._rows_ptr, step.num_seqs,
                                                 num_blocks, block_size, host_ptr, host_cap, dev_ptr, dev_cap,
                                                 event, stream)
        if status:
            _native.check(status, "lvb_stage_step_metadata")
        return dev


class _LayerInfo(NamedTuple):
    """Per (cache, layer) constants of the attention launches."""

    spec: object
    q_tail: tuple[int, int]
    kv_tail: tuple[int, int]
    args: tuple  # (key_cache, value_cache, hq, hkv, head_size, block_size, num_blocks, dtype)
    keys: Tensor
    values: Tensor


class B200PagedAttention:
    """Per-step attention context; one ``forward`` per layer."""

    def __init__(self, cache, metadata, staging: SingleStepStaging, backend: "B200PagedAttentionBackend"):
        config = cache.config
        device = backend._device_of(config)
        if config.dtype not in _SUPPORTED_DTYPES:
            raise KVCacheError("B200 paged attention supports fp16 and bf16 KV caches")
        self._cache = cache
        self._metadata = metadata
        self._backend = backend
        self._layer_ids: set[str] = set()
        self._device = device
        self._device_index = device.index
        self._dtype = config.dtype
        # Gathering from the metadata objects, validation (the reference's
        # block-table rules, same order and messages), packing and the one
        # pinned host-to-device copy of the per-step int32 payload all run in
        # native code (_hostpack.gather_step, lvb_stage_step_metadata).
        packer = backend._packer
        step = packer.gather(metadata)
        packed = packer.stage(staging, config.num_blocks, config.block_size)
        n, max_blocks = step.num_seqs, step.max_blocks
        self._packed = packed  # keeps the device payload alive; the launches take raw addresses
        base = packed.data_ptr()
        self._tables_ptr = base
        self._computed_ptr = base + 4 * n * max_blocks
        self._query_start_ptr = self._computed_ptr + 4 * n
        self._request_indices_ptr = self._query_start_ptr + 4 * (n + 1)
        self._request_order_ptr = self._request_indices_ptr + 4 * step.num_tokens
        self._table_stride = max_blocks
        self._num_seqs = n
        self._num_decode = step.num_single
        self._num_tokens = step.num_tokens
        self._max_query_len = step.max_query_len
        self._max_seq_len = step.max_seq_len
        self._linear = step.linear
        self._visibility: Tensor | None = None
        self._visibility_start: Tensor | None = None
        self._step_args = (self._tables_ptr, max_blocks, self._computed_ptr, self._query_start_ptr,
                           self._request_indices_ptr, self._request_order_ptr, 0, 0, n, step.num_single,
                           step.num_tokens, step.max_query_len, step.max_seq_len)
        self._workspace: tuple | None = None

    @property
    def layer_ids(self) -> frozenset[str]:
        return frozenset(self._layer_ids)

    # Tensors of the step's payload, for callers that want views (tests, the
    # fused RoPE + K/V write).
    def _view(self, offset_ptr: int, count: int) -> Tensor:
        start = (offset_ptr - self._tables_ptr) // 4
        return self._packed[start : start + count]

    @property
    def _tables(self) -> Tensor:
        return self._view(self._tables_ptr, self._num_seqs * self._table_stride)

    @property
    def _computed(self) -> Tensor:
        return self._view(self._computed_ptr, self._num_seqs)

    @property
    def _query_start(self) -> Tensor:
        return self._view(self._query_start_ptr, self._num_seqs + 1)

    @property
    def _request_indices(self) -> Tensor:
        return self._view(self._request_indices_ptr, self._num_tokens)

    @property
    def _request_order(self) -> Tensor:
        return self._view(self._request_order_ptr, 2 * self._num_seqs)

    def forward(self, layer_id: str, query: Tensor, key: Tensor, value: Tensor, *, scale: float,
                write_kv: bool = True) -> Tensor:
        """Write this step's K/V for ``layer_id`` and return the attention output.

        ``write_kv=False``: the step's K/V are already in the cache
        (``rope_write_kv``)."""

        if layer_id in self._layer_ids:
            raise KVCacheError(f"paged attention layer {layer_id!r} ran more than once")
        self._layer_ids.add(layer_id)
        info = self._backend._layer_info(self._cache, layer_id)
        # Shape rules shared with the reference backends (paged_attention.py:226-247).
        qs, ks = query.shape, key.shape
        if len(qs) != 3:
            raise KVCacheError("paged attention query must have three dimensions")
        if qs[0] != ks[0] or value.shape != ks:
            raise KVCacheError("paged attention Q/K/V token dimensions must match")
        if qs[0] != self._num_tokens:
            raise KVCacheError("paged attention metadata token count does not match query")
        if qs[1:] != info.q_tail:
            raise KVCacheError("paged attention query shape does not match the layer spec")
        if ks[1:] != info.kv_tail:
            raise KVCacheError("paged attention K/V shape does not match the layer spec")
        dt, index = self._dtype, self._device_index
        if (query.dtype != dt or key.dtype != dt or value.dtype != dt or query.get_device() != index
                or key.get_device() != index or value.get_device() != index):
            raise KVCacheError("B200 query/key/value dtype and device must match the KV cache")
        if info.kv_tail[1] % 8 or info.kv_tail[1] > 256:
            raise KVCacheError("B200 paged attention supports head sizes that are multiples of 8 up to 256")
        out = torch.empty_like(query, memory_format=torch.contiguous_format)
        return self._launch(info, query, key, value, float(scale), out, write_kv)

    def rope_write_kv(self, layer_id: str, qkv: Tensor, q_heads: int, kv_heads: int, positions: Tensor,
                      cos: Tensor, sin: Tensor) -> None:
        """RoPE on the query and key heads of merged QKV rows, fused with this
        step's K/V write for ``layer_id`` (``lvb_rope_kv_write``); follow with
        ``forward(..., write_kv=False)``."""

        _rope_write_kv(self._cache, layer_id, qkv, q_heads, kv_heads, positions, cos, sin, self._tables_ptr,
                       self._table_stride, self._computed_ptr, self._query_start_ptr, self._request_indices_ptr,
                       self._device)

    def kv_write_args(self, layer_id: str) -> tuple | None:
        """Device addresses a projection epilogue needs to write this step's
        K/V of ``layer_id`` (``lvb_awq_qkv_rope_packed``); None when the
        fused write does not cover the cache (fp16 caches only)."""

        if self._dtype != torch.float16:
            return None
        info = self._backend._layer_info(self._cache, layer_id)
        return (info.args[0], info.args[1], self._tables_ptr, self._table_stride, self._computed_ptr,
                self._query_start_ptr, self._request_indices_ptr, info.args[5])

    def launch(self, layer_id: str, query: Tensor, key: Tensor, value: Tensor, *, scale: float,
               out: Tensor, write_kv: bool = True) -> Tensor:
        """Enqueue the K/V write and the attention into ``out`` without the
        once-per-layer bookkeeping of ``forward`` (no allocation, no host
        synchronisation), so repeated steps can be captured in a CUDA graph.
        Shapes must already satisfy ``forward``'s checks."""

        return self._launch(self._backend._layer_info(self._cache, layer_id), query, key, value, float(scale), out,
                            write_kv)

    def _launch(self, info: _LayerInfo, query: Tensor, key: Tensor, value: Tensor, scale: float, out: Tensor,
                write_kv: bool) -> Tensor:
        if not self._linear and self._visibility is None:
            vis, starts = self._metadata.visibility_tensor(device=self._device)
            self._visibility = vis.to(torch.uint8)
            self._visibility_start = starts
            self._step_args = self._step_args[:6] + (self._visibility.data_ptr(),
                                                     self._visibility_start.data_ptr()) + self._step_args[8:]
        if self._workspace is None or self._workspace[0] != info.args[2:5]:
            spec = info.spec
            ptr, nbytes = self._backend._workspace(self._device, self._num_seqs, spec.num_query_heads,
                                                   spec.num_kv_heads, spec.head_size, self._max_seq_len)
            self._workspace = (info.args[2:5], ptr, nbytes)
        if write_kv:
            key = _heads_contiguous(key, align=8)
            value = _heads_contiguous(value, align=8)
        query = _heads_contiguous(query, align=2)
        _, ws_ptr, ws_bytes = self._workspace
        status, which = self._backend._hostpack.attention_step(
            self._step_args, info.args, query.data_ptr(), query.stride(0), key.data_ptr(), key.stride(0),
            value.data_ptr(), value.stride(0), out.data_ptr(), out.stride(0), write_kv, scale, ws_ptr, ws_bytes,
            _native.stream_handle(self._device))
        if status:
            _native.check(status, "lvb_paged_attention" if which else "lvb_paged_kv_write")
        return out


def _rope_write_kv(cache, layer_id, qkv, q_heads, kv_heads, positions, cos, sin, tables, table_stride, computed,
                   query_start, request_indices, device) -> None:
    """``lvb_rope_kv_write`` for one layer; the step metadata (tables,
    computed counts, query starts, request indices) as device addresses."""

    spec = cache.layer_spec(layer_id)
    config = cache.config
    if config.dtype != torch.float16 or qkv.dtype != torch.float16:
        raise KVCacheError("the fused RoPE + K/V write covers fp16 caches")
    if (q_heads, kv_heads) != (spec.num_query_heads, spec.num_kv_heads) or positions.dtype != torch.int32:
        raise KVCacheError("QKV heads or positions do not match the layer")
    layer = cache.layer(layer_id)
    _native.check(_native.library().lvb_rope_kv_write(
        qkv.data_ptr(), qkv.stride(0), qkv.shape[0], q_heads, kv_heads, spec.head_size, positions.data_ptr(),
        cos.data_ptr(), sin.data_ptr(), cos.shape[0], layer.keys.data_ptr(), layer.values.data_ptr(),
        tables, table_stride, computed, query_start, request_indices,
        config.block_size, _native.stream_handle(device)), "lvb_rope_kv_write")


class B200PagedAttentionBackend:
    """Creates one ``B200PagedAttention`` per model step.

    Owns the pinned metadata staging buffer, the split-context workspace and
    per-(cache, layer) launch constants; all are reused by later steps.
    """

    name = "b200"

    def __init__(self) -> None:
        _native.library()  # fail loudly at construction when the library is missing
        self._hostpack = _native.hostpack()
        self._staging: SingleStepStaging | None = None
        self._packer = StepMetadataPacker()
        self._workspaces: dict[torch.device, Tensor] = {}
        self._layers: "weakref.WeakKeyDictionary[object, dict[str, _LayerInfo]]" = weakref.WeakKeyDictionary()
        self._devices: dict[object, torch.device] = {}

    def _device_of(self, config) -> torch.device:
        device = self._devices.get(config.device)
        if device is None:
            device = torch.device(config.device)
            if device.type != "cuda":
                raise KVCacheError("B200 paged attention requires a CUDA KV cache")
            if device.index is None:
                device = torch.device("cuda", torch.cuda.current_device())
            self._devices[config.device] = device
        return device

    def create(self, cache, metadata) -> B200PagedAttention:
        device = self._device_of(cache.config)
        if self._staging is None:
            self._staging = SingleStepStaging(device)
        return B200PagedAttention(cache, metadata, self._staging, self)

    def _layer_info(self, cache, layer_id: str) -> _LayerInfo:
        try:
            return self._layers[cache][layer_id]
        except KeyError:
            pass
        spec = cache.layer_spec(layer_id)  # the cache's own KVCacheError for an unknown layer
        layer = cache.layer(layer_id)
        config = cache.config
        dtype = _native.DTYPE_BF16 if config.dtype == torch.bfloat16 else _native.DTYPE_F16
        info = _LayerInfo(spec, (spec.num_query_heads, spec.head_size), (spec.num_kv_heads, spec.head_size),
                          (layer.keys.data_ptr(), layer.values.data_ptr(), spec.num_query_heads, spec.num_kv_heads,
                           spec.head_size, config.block_size, config.num_blocks, dtype),
                          layer.keys, layer.values)
        self._layers.setdefault(cache, {})[layer_id] = info
        return info

    def _workspace(self, device: torch.device, num_seqs: int, hq: int, hkv: int, d: int,
                   max_seq_len: int) -> tuple[int, int]:
        need = int(_native.library().lvb_paged_attention_workspace_bytes(num_seqs, hq, hkv, d, max_seq_len))
        buf = self._workspaces.get(device)
        if buf is None or buf.numel() < need:
            # Zero once: the split-merge semaphores start at zero and every call
            # leaves them zero.
            buf = torch.zeros(max(need, 1 << 20), dtype=torch.uint8, device=device)
            self._workspaces[device] = buf
        return buf.data_ptr(), buf.numel()
