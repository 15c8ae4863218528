"""CPU tests of the host-side interface mirror (no GPU work).

The product's ``PagedAttentionMetadata`` must agree with the reference on every
golden metadata case: slot mapping, request indices, tree visibility and the
exact block-table validation error.
"""

from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch

from light_vllm_b200 import kv_cache as kv

META = json.loads((Path(__file__).resolve().parent / "golden" / "paged_meta.json").read_text())


def _metadata(case) -> kv.PagedAttentionMetadata:
    return kv.PagedAttentionMetadata(
        block_tables=tuple(tuple(t) for t in case["tables"]),
        num_computed_tokens=tuple(case["computed"]),
        query_layouts=tuple(kv.QueryLayout(tuple(p)) for p in case["layouts"]),
        num_reserved_query_tokens=tuple(case.get("reserved") or ()),
        num_readonly_prefix_blocks=tuple(case.get("readonly") or ()),
    )


@pytest.mark.parametrize("case", META, ids=[c["name"] for c in META])
def test_metadata_mirror_matches_reference(case):
    md = _metadata(case)
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


def test_query_layout_rejects_forward_parents():
    with pytest.raises(ValueError):
        kv.QueryLayout((-1, 1))
    with pytest.raises(ValueError):
        kv.QueryLayout(())


def test_metadata_rejects_mismatched_fields():
    with pytest.raises(ValueError):
        kv.PagedAttentionMetadata(block_tables=((0,),), num_computed_tokens=(0, 1),
                                  query_layouts=(kv.linear_query_layout(1),))
    with pytest.raises(ValueError, match="reserved query counts must cover"):
        kv.PagedAttentionMetadata(block_tables=((0,),), num_computed_tokens=(0,),
                                  query_layouts=(kv.linear_query_layout(2),),
                                  num_reserved_query_tokens=(1,))


def test_layer_spec_rules():
    with pytest.raises(ValueError):
        kv.AttentionLayerSpec("a", 6, 4, 8)
    with pytest.raises(ValueError):
        kv.ModelKVCacheSpec((kv.AttentionLayerSpec("a", 4, 2, 8), kv.AttentionLayerSpec("a", 4, 2, 8)))


def test_kv_bytes_per_block_known_answer():
    # tests/test_paged_attention.py:51-71 in the reference: 128 bytes per block.
    spec = kv.ModelKVCacheSpec((kv.AttentionLayerSpec("attention", 2, 2, 4),))
    assert kv.kv_cache_bytes_per_block(spec, block_size=2, dtype=torch.float32) == 128


def test_cpu_cache_write_is_refused():
    spec = kv.ModelKVCacheSpec((kv.AttentionLayerSpec("attention", 2, 2, 8),))
    cache = kv.PagedKVCache(spec, kv.PagedKVCacheConfig(4, 2, dtype=torch.float16))
    with pytest.raises(kv.KVCacheError, match="requires a CUDA device"):
        cache.write("attention", torch.zeros(1, 2, 8, dtype=torch.float16),
                    torch.zeros(1, 2, 8, dtype=torch.float16), torch.tensor([0]))


def test_backend_refuses_cpu_cache():
    from light_vllm_b200.paged_attention import B200PagedAttentionBackend

    spec = kv.ModelKVCacheSpec((kv.AttentionLayerSpec("attention", 2, 2, 8),))
    cache = kv.PagedKVCache(spec, kv.PagedKVCacheConfig(4, 2, dtype=torch.float16))
    md = kv.PagedAttentionMetadata(block_tables=((0,),), num_computed_tokens=(0,),
                                   query_layouts=(kv.linear_query_layout(1),))
    with pytest.raises(kv.KVCacheError, match="requires a CUDA KV cache"):
        B200PagedAttentionBackend().create(cache, md)


def test_reference_known_answers_for_metadata():
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
    assert tree.query_start_loc == (0, 3, 5)
    assert tree.request_indices_tensor(device=torch.device("cpu")).tolist() == [0, 0, 0, 1, 1]
    assert starts.tolist() == [0, 9, 13]
    assert vis.tolist() == expected
    ovis, ostarts = opa.visibility_tensor([(-1, 0, 0), (-1, 0)])
    assert list(ovis) == expected and list(ostarts) == [0, 9, 13]


def test_reference_known_answer_for_compaction_slots():
    """tests/test_paged_attention.py:178-228: retained queries (0, 2, 4) of a
    5-token tree over blocks (1, 3, 0, 2) move to slots (6, 7, 0)."""

    from oracle import paged_attention as opa

    source, target = opa.compact_slots((1, 3, 0, 2), num_computed_tokens=2, retained_query_indices=(0, 2, 4),
                                       block_size=2)
    assert target == (6, 7, 0)
    assert source == (6, 0, 4)


def test_compaction_checks_match_the_reference_order():
    spec = kv.ModelKVCacheSpec((kv.AttentionLayerSpec("attention", 2, 2, 8),))
    cache = kv.PagedKVCache.__new__(kv.PagedKVCache)  # checks run before any device work
    cache._config = kv.PagedKVCacheConfig(4, 2, dtype=torch.float16)
    cache._layers = {}
    with pytest.raises(ValueError, match="reserved query tokens must cover"):
        cache.compact((1, 3, 0), num_computed_tokens=2, num_query_tokens=5, num_reserved_query_tokens=4,
                      retained_query_indices=(0,))
    with pytest.raises(ValueError, match="unique"):
        cache.compact((1, 3, 0), num_computed_tokens=2, num_query_tokens=3, num_reserved_query_tokens=3,
                      retained_query_indices=(0, 0))
    with pytest.raises(kv.KVCacheError, match="exceeds the paged KV tail"):
        cache.compact((1, 3, 0), num_computed_tokens=2, num_query_tokens=3, num_reserved_query_tokens=3,
                      retained_query_indices=(3,))
    with pytest.raises(kv.KVCacheError, match="exactly cover"):
        cache.compact((1, 3), num_computed_tokens=2, num_query_tokens=3, num_reserved_query_tokens=3,
                      retained_query_indices=(0,))
    with pytest.raises(kv.KVCacheError, match="aliases"):
        cache.compact((1, 1, 0), num_computed_tokens=2, num_query_tokens=3, num_reserved_query_tokens=3,
                      retained_query_indices=(0,))
    with pytest.raises(kv.KVCacheError, match="readonly prefix"):
        cache.compact((1, 3, 0), num_computed_tokens=2, num_query_tokens=3, num_reserved_query_tokens=3,
                      retained_query_indices=(0,), num_readonly_prefix_blocks=2)
