"""B200-native (sm_100a) hot path for light-vllm.

Two drop-in plugins behind light-vllm's own extension points:

* ``B200AWQScheme`` -- an ``AWQScheme`` whose ``LinearOperation`` runs the
  AutoAWQ W4A16 linear on tcgen05 tensor cores (``light_vllm_b200.awq``);
* ``B200PagedAttentionBackend`` -- a ``PagedAttentionBackend`` that writes
  paged K/V and attends with sm_100a kernels (``light_vllm_b200.paged_attention``);

plus ``TensorParallelCollectives`` for the row-parallel all-reduce on the
caller's stream (``light_vllm_b200.collectives``) and ``compact_kv``, the
tree-acceptance K/V compaction on the device (``light_vllm_b200.kv_cache``).
Both plugins take light-vllm's own ``PagedKVCache`` and
``PagedAttentionMetadata`` objects; this package defines no copies of them.  All GPU work goes through
the C-ABI library ``_lib/liblvb200.so`` (``include/lvb200.h``); there is no
CPU or Triton fallback.
"""

from light_vllm_b200.awq import B200AWQOperation, B200AWQScheme, b200_awq_dequantize, b200_awq_linear
from light_vllm_b200.kv_cache import KVCacheError, compact_kv
from light_vllm_b200.paged_attention import B200PagedAttention, B200PagedAttentionBackend

__all__ = [
    "B200AWQOperation",
    "B200AWQScheme",
    "B200PagedAttention",
    "B200PagedAttentionBackend",
    "KVCacheError",
    "b200_awq_dequantize",
    "b200_awq_linear",
    "compact_kv",
]
