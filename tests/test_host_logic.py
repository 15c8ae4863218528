"""CPU tests of the host side (no GPU work).

* The paged-KV stand-ins of ``oracle/paged_cache.py`` (used where light-vllm
  is not importable) and, when it is, light-vllm's own
  ``PagedAttentionMetadata``: both must reproduce every golden metadata case
  the reference produced (slot mapping, request indices, tree visibility,
  the exact block-table validation error) and the known answers of the
  reference's tests.
* The backend's host checks: a CPU cache is refused, ``KVCacheError``
  derives from the reference's class, and ``compact_kv``'s native argument
  rules raise what ``PagedKVCache.compact`` raises, in the same order.
"""

from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch

from oracle import paged_cache as stand_in
from oracle.paged_cache import reference_types

META = json.loads((Path(__file__).resolve().parent / "golden" / "paged_meta.json").read_text())
REF = reference_types()
TYPES = [pytest.param(stand_in, id="oracle-stand-ins")]
if REF.source == "light_vllm":
    TYPES.append(pytest.param(REF, id="light-vllm"))


def _metadata(kv, case):
    return kv.PagedAttentionMetadata(
        block_tables=tuple(tuple(t) for t in case["tables"]),
        num_computed_tokens=tuple(case["computed"]),
        query_layouts=tuple(kv.QueryLayout(tuple(p)) for p in case["layouts"]),
        num_reserved_query_tokens=tuple(case.get("reserved") or ()),
        num_readonly_prefix_blocks=tuple(case.get("readonly") or ()),
    )


@pytest.mark.parametrize("kv", TYPES)
@pytest.mark.parametrize("case", META, ids=[c["name"] for c in META])
def test_metadata_types_match_reference_golden(kv, case):
    md = _metadata(kv, case)
    assert list(md.query_start_loc) == case["query_start_loc"]
    assert list(md.request_indices) == case["request_indices"]
    assert md.has_only_linear_queries == case["has_only_linear_queries"]
    vis, starts = md.visibility_tensor(device=torch.device("cpu"))
    assert vis.tolist() == case["visibility"]
    assert starts.tolist() == case["visibility_start"]
    try:
        slots = md.slot_mapping(block_size=case["block_size"], device=torch.device("cpu")).tolist()
        error = None
    except kv.KVCacheError as exc:
        slots, error = None, str(exc)
    assert slots == case["slot_mapping"]
    assert error == case["slot_error"]
    try:
        md.validate_block_tables(num_blocks=case["num_blocks"], block_size=case["block_size"])
        error = None
    except kv.KVCacheError as exc:
        error = str(exc)
    assert error == case["validate_error"]


def test_stand_in_rules():
    kv = stand_in
    with pytest.raises(ValueError):
        kv.QueryLayout((-1, 1))
    with pytest.raises(ValueError):
        kv.QueryLayout(())
    with pytest.raises(ValueError):
        kv.PagedAttentionMetadata(block_tables=((0,),), num_computed_tokens=(0, 1),
                                  query_layouts=(kv.linear_query_layout(1),))
    with pytest.raises(ValueError, match="reserved query counts must cover"):
        kv.PagedAttentionMetadata(block_tables=((0,),), num_computed_tokens=(0,),
                                  query_layouts=(kv.linear_query_layout(2),),
                                  num_reserved_query_tokens=(1,))
    with pytest.raises(ValueError):
        kv.AttentionLayerSpec("a", 6, 4, 8)
    with pytest.raises(ValueError):
        kv.ModelKVCacheSpec((kv.AttentionLayerSpec("a", 4, 2, 8), kv.AttentionLayerSpec("a", 4, 2, 8)))


def test_kv_bytes_per_block_known_answer():
    # tests/test_paged_attention.py:51-71 in the reference: 128 bytes per block.
    spec = stand_in.ModelKVCacheSpec((stand_in.AttentionLayerSpec("attention", 2, 2, 4),))
    assert stand_in.kv_cache_bytes_per_block(spec, block_size=2, dtype=torch.float32) == 128


@pytest.mark.parametrize("kv", TYPES)
def test_backend_refuses_cpu_cache(kv):
    from light_vllm_b200 import KVCacheError
    from light_vllm_b200.paged_attention import B200PagedAttentionBackend

    spec = kv.ModelKVCacheSpec((kv.AttentionLayerSpec("attention", 2, 2, 8),))
    cache = kv.PagedKVCache(spec, kv.PagedKVCacheConfig(4, 2, dtype=torch.float16))
    md = kv.PagedAttentionMetadata(block_tables=((0,),), num_computed_tokens=(0,),
                                   query_layouts=(kv.linear_query_layout(1),))
    with pytest.raises(KVCacheError, match="requires a CUDA KV cache"):
        B200PagedAttentionBackend().create(cache, md)


@pytest.mark.skipif(REF.source != "light_vllm", reason="light-vllm is not importable here")
def test_backend_error_is_the_reference_error_type():
    from light_vllm_b200 import KVCacheError

    assert issubclass(KVCacheError, REF.KVCacheError)


@pytest.mark.parametrize("kv", TYPES)
def test_reference_known_answers_for_metadata(kv):
    """Known answers of the reference's tests/test_paged_attention.py:121-175:
    slot mapping across non-contiguous blocks, packed request indices and the
    tree visibility vector."""

    from oracle import paged_attention as opa

    md = kv.PagedAttentionMetadata(block_tables=((2, 0), (1, 3)), num_computed_tokens=(0, 1),
                                   query_layouts=(kv.linear_query_layout(3), kv.linear_query_layout(2)))
    assert md.slot_mapping(block_size=2, device=torch.device("cpu")).tolist() == [4, 5, 0, 3, 6]
    assert list(opa.slot_mapping(((2, 0), (1, 3)), (0, 1), (3, 2), (3, 2), 2)) == [4, 5, 0, 3, 6]

    tree = kv.PagedAttentionMetadata(block_tables=((0, 1), (2,)), num_computed_tokens=(0, 0),
                                     query_layouts=(kv.QueryLayout((-1, 0, 0)), kv.linear_query_layout(2)))
    vis, starts = tree.visibility_tensor(device=torch.device("cpu"))
    expected = [True, False, False, True, True, False, True, False, True, True, False, True, True]
    assert tuple(tree.query_start_loc) == (0, 3, 5)
    assert tree.request_indices_tensor(device=torch.device("cpu")).tolist() == [0, 0, 0, 1, 1]
    assert starts.tolist() == [0, 9, 13]
    assert vis.tolist() == expected
    ovis, ostarts = opa.visibility_tensor([(-1, 0, 0), (-1, 0)])
    assert list(ovis) == expected and list(ostarts) == [0, 9, 13]


def test_reference_known_answer_for_compaction_slots():
    """tests/test_paged_attention.py:178-228: retained queries (0, 2, 4) of a
    5-token tree over blocks (1, 3, 0, 2) move to slots (6, 7, 0)."""

    import ctypes

    import numpy as np

    from light_vllm_b200 import _native
    from oracle import paged_attention as opa

    source, target = opa.compact_slots((1, 3, 0, 2), num_computed_tokens=2, retained_query_indices=(0, 2, 4),
                                       block_size=2)
    assert target == (6, 7, 0)
    assert source == (6, 0, 4)
    # the native plan of compact_kv gives the same pairs
    table = np.array([1, 3, 0, 2], dtype=np.int64)
    counts = np.array([2, 5, 5, 0], dtype=np.int64)
    retained = np.array([0, 2, 4], dtype=np.int64)
    src = np.empty(3, dtype=np.int32)
    dst = np.empty(3, dtype=np.int32)
    moved = ctypes.c_int64(-1)
    _native.check(_native.library().lvb_kv_compact_plan(
        table.ctypes.data, 4, counts.ctypes.data, retained.ctypes.data, 3, 4, 2, src.ctypes.data, dst.ctypes.data,
        ctypes.byref(moved)), "plan")
    assert tuple(src) == source and tuple(dst) == target and moved.value == 2


COMPACT_CASES = [
    # (block_ids, computed, queries, reserved, retained, readonly, exception type, message)
    ((1, 3, 0), -1, 3, 3, (0,), 0, ValueError, "paged compact counts must be non-negative integers"),
    ((1, 3, 0), 2.0, 3, 3, (0,), 0, ValueError, "paged compact counts must be non-negative integers"),
    ((1, 3, 0), 2, 5, 4, (0,), 0, ValueError, "reserved query tokens must cover every actual query"),
    ((1, 3, 0), 2, 3, 3, (0, -1), 0, ValueError, "retained query indices must be non-negative integers"),
    ((1, 3, 0), 2, 3, 3, (0, 0), 0, ValueError, "retained query indices must be unique"),
    ((1, 3, 0), 2, 3, 3, (3,), 0, "kv", "retained query index exceeds the paged KV tail"),
    ((1, 3), 2, 3, 3, (0,), 0, "kv", "block table does not exactly cover the reserved query slots"),
    ((1, 3, 9), 2, 3, 3, (0,), 0, "kv", "block table contains an invalid physical block"),
    ((1, 3, "0"), 2, 3, 3, (0,), 0, "kv", "block table contains an invalid physical block"),
    ((1, 1, 0), 2, 3, 3, (0,), 0, "kv", "block table aliases a physical block within one request"),
    ((1, 3, 0), 2, 3, 3, (0,), 2, "kv", "readonly prefix blocks exceed the computed prefix"),
]


@pytest.mark.parametrize("case", COMPACT_CASES, ids=[c[-1][:24] + str(i) for i, c in enumerate(COMPACT_CASES)])
def test_compact_kv_rules_match_the_reference(case):
    """``compact_kv`` (native plan) raises the exception type and message of
    ``PagedKVCache.compact`` for each broken rule, before any device work."""

    from light_vllm_b200 import KVCacheError, compact_kv

    table, computed, queries, reserved, retained, readonly, etype, message = case
    kv = REF if REF.source == "light_vllm" else stand_in
    spec = kv.ModelKVCacheSpec((kv.AttentionLayerSpec("attention", 2, 2, 8),))
    cache = kv.PagedKVCache(spec, kv.PagedKVCacheConfig(4, 2, dtype=torch.float16))
    args = dict(num_computed_tokens=computed, num_query_tokens=queries, num_reserved_query_tokens=reserved,
                retained_query_indices=retained, num_readonly_prefix_blocks=readonly)
    ours = KVCacheError if etype == "kv" else etype
    with pytest.raises(ours) as got:
        compact_kv(cache, table, **args)
    assert message in str(got.value)
    theirs = kv.KVCacheError if etype == "kv" else etype
    with pytest.raises(theirs, match=message):
        cache.compact(table, **args)


def test_compact_kv_without_movement_needs_no_device():
    from light_vllm_b200 import compact_kv

    kv = REF if REF.source == "light_vllm" else stand_in
    spec = kv.ModelKVCacheSpec((kv.AttentionLayerSpec("attention", 2, 2, 8),))
    cache = kv.PagedKVCache(spec, kv.PagedKVCacheConfig(4, 2, dtype=torch.float16))
    # retained (0, 1) already sit at the tail: nothing moves, as in the reference
    assert compact_kv(cache, (1, 3, 0), num_computed_tokens=2, num_query_tokens=3, num_reserved_query_tokens=3,
                      retained_query_indices=(0, 1)) == 0
    assert cache.compact((1, 3, 0), num_computed_tokens=2, num_query_tokens=3, num_reserved_query_tokens=3,
                         retained_query_indices=(0, 1)) == 0
