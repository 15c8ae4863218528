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
