"""KV-cache operations of the B200 backend over light-vllm's ``PagedKVCache``.

The backend takes the reference's own cache and metadata objects and touches
them only through the reference's surface: ``cache.config`` (``num_blocks``,
``block_size``, ``dtype``, ``device``), ``cache.model_spec.layers``,
``cache.layer_spec(layer_id)`` and ``cache.layer(layer_id).keys / .values``
([num_blocks, block_size, num_kv_heads, head_size] each,
runtime/execution/paged_cache.py:328-338).  Nothing here re-implements the
reference's types.

* ``KVCacheError`` -- raised for every cache-contract violation the backend
  detects; it derives from light-vllm's ``KVCacheError``
  (runtime/kv_cache.py:21-22) when light-vllm is importable, so the Worker's
  handlers catch it.
* ``compact_kv`` -- the tree-acceptance compaction of
  ``PagedKVCache.compact`` (runtime/execution/paged_cache.py:257-326) on the
  device: the argument rules are checked and the (source, target) slot pairs
  planned natively (``lvb_kv_compact_plan``), and each layer's rows move in
  one launch that reads every source row before writing any target
  (``lvb_kv_move_rows``).
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

try:  # interoperate with an installed light-vllm
    from light_vllm.runtime.kv_cache import KVCacheError as _BaseKVCacheError
except ImportError:  # standalone
    _BaseKVCacheError = RuntimeError


class KVCacheError(_BaseKVCacheError):
    """A KV cache contract was violated."""


def _ints(values) -> np.ndarray:
    """int64 array of Python ints; anything that is not an int becomes -1,
    which the native rules reject with the message of the field it is in."""

    return np.fromiter((v if type(v) is int else -1 for v in values), dtype=np.int64)


def compact_kv(cache, block_ids, *, num_computed_tokens: int, num_query_tokens: int,
               num_reserved_query_tokens: int, retained_query_indices, num_readonly_prefix_blocks: int = 0) -> int:
    """Move the retained query tokens' K/V of every layer of ``cache`` from
    their flattened query slots to the contiguous tail after the computed
    prefix; returns how many tokens changed slot.  Same arguments, result,
    exception types and messages as ``PagedKVCache.compact``."""

    from light_vllm_b200 import _native

    config = cache.config
    table = _ints(tuple(block_ids))
    retained = _ints(tuple(retained_query_indices))
    counts = _ints((num_computed_tokens, num_query_tokens, num_reserved_query_tokens, num_readonly_prefix_blocks))
    n = retained.size
    src = np.empty(max(n, 1), dtype=np.int32)
    dst = np.empty(max(n, 1), dtype=np.int32)
    moved = ctypes.c_int64(0)
    lib = _native.library()
    _native.check(lib.lvb_kv_compact_plan(
        table.ctypes.data, table.size, counts.ctypes.data, retained.ctypes.data, n, config.num_blocks,
        config.block_size, src.ctypes.data, dst.ctypes.data, ctypes.byref(moved)), "lvb_kv_compact_plan")
    if moved.value == 0:
        return 0
    device = torch.device(config.device)
    if device.type != "cuda":
        raise KVCacheError("the B200 KV compaction requires a CUDA KV cache")
    if config.dtype not in (torch.float16, torch.bfloat16):
        raise KVCacheError("the B200 KV compaction moves fp16 or bf16 caches")
    slots = torch.from_numpy(np.stack([src[:n], dst[:n]])).to(device)
    stream = _native.stream_handle(device)
    dtype_code = _native.DTYPE_BF16 if config.dtype == torch.bfloat16 else _native.DTYPE_F16
    for spec in cache.model_spec.layers:
        layer = cache.layer(spec.layer_id)
        _native.check(lib.lvb_kv_move_rows(
            layer.keys.data_ptr(), layer.values.data_ptr(), slots[0].data_ptr(), slots[1].data_ptr(), n,
            spec.num_kv_heads, spec.head_size, config.num_blocks * config.block_size, dtype_code, stream),
            "lvb_kv_move_rows")
    return int(moved.value)
