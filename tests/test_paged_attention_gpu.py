"""GPU parity of the B200 paged-attention backend.

* The reference's Triton test matrix (tests/test_triton_paged_attention.py):
  packed GQA prefill for head sizes 32/80/128/256 in fp16/bf16, the Qwen
  28q/4kv group, history across chunks, tree visibility, decode after
  prefill, a shared read-only prefix and unused lookahead slots -- against the
  CPU oracle with the reference's tolerances (fp16 3e-3, bf16 2e-2) and
  bit-exact cache slots.
* The golden fixtures produced by the reference's own TorchPagedAttention.
* Decode batches on the split-context kernel up to the BASELINE config-2 shape
  (64 sequences, contexts 512..4096, 28q/4kv, D=128, bf16) against a float64
  evaluation of the same visible positions: max-abs <= 2e-2 and rel-L2 <= 1e-3
  after rounding to the cache dtype.
"""

from __future__ import annotations

import json
from math import sqrt
from pathlib import Path

import numpy as np
import pytest
import torch

from light_vllm_b200 import KVCacheError, _native, compact_kv
from light_vllm_b200.paged_attention import B200PagedAttentionBackend
from oracle.paged_cache import reference_types

# light-vllm's own cache and metadata classes when importable, else the
# oracle's stand-ins (same surface): the backend is driven through them.
_T = reference_types()
AttentionLayerSpec, ModelKVCacheSpec = _T.AttentionLayerSpec, _T.ModelKVCacheSpec
PagedAttentionMetadata, QueryLayout, linear_query_layout = _T.PagedAttentionMetadata, _T.QueryLayout, _T.linear_query_layout
PagedKVCache, PagedKVCacheConfig = _T.PagedKVCache, _T.PagedKVCacheConfig
from oracle import awq as oawq
from oracle import paged_attention as opa

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
GOLDEN = Path(__file__).resolve().parent / "golden"


def _layouts(*lengths):
    return tuple(linear_query_layout(n) for n in lengths)


def _cache(head_size, dtype, *, block_size=2, hq=4, hkv=2, num_blocks=16):
    spec = ModelKVCacheSpec((AttentionLayerSpec("attention", hq, hkv, head_size),))
    return PagedKVCache(spec, PagedKVCacheConfig(num_blocks, block_size, dtype=dtype, device=DEV))


def _run_and_compare(cache, md, q, k, v, *, tol=None):
    """Run the B200 backend and the CPU oracle on copies of the same cache."""

    layer = cache.layer("attention")
    k_before = layer.keys.cpu()
    v_before = layer.values.cpu()
    scale = 1.0 / sqrt(q.shape[-1])
    actual = B200PagedAttentionBackend().create(cache, md).forward("attention", q, k, v, scale=scale)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    kc, vc = k_before.clone(), v_before.clone()
    expected = opa.attend(q.cpu(), k.cpu(), v.cpu(), kc, vc,
                          md.block_tables, md.num_computed_tokens,
                          [layout.parent_indices for layout in md.query_layouts],
                          scale=scale, reserved=md.num_reserved_query_tokens)
    if tol is None:
        tol = 3e-3 if q.dtype == torch.float16 else 2e-2
    torch.testing.assert_close(actual.cpu(), expected, atol=tol, rtol=tol)
    # Bit-exact slot contents (every slot, not only the written ones); compared
    # as bit patterns because never-written slots may hold NaN encodings.
    assert torch.equal(_bits(layer.keys.cpu()), _bits(kc))
    assert torch.equal(_bits(layer.values.cpu()), _bits(vc))
    return actual


def _bits(t):
    return t.view(torch.int16)


def _randomise(cache):
    layer = cache.layer("attention")
    layer.keys.copy_(torch.randn(layer.keys.shape, device=DEV).to(layer.keys.dtype))
    layer.values.copy_(torch.randn(layer.values.shape, device=DEV).to(layer.values.dtype))


@pytest.mark.parametrize("head_size", (32, 80, 128, 256))
@pytest.mark.parametrize("dtype", (torch.float16, torch.bfloat16))
def test_packed_gqa_prefill(head_size, dtype):
    torch.manual_seed(20260817)
    cache = _cache(head_size, dtype, block_size=4)
    _randomise(cache)
    md = PagedAttentionMetadata(block_tables=((7, 1), (4,)), num_computed_tokens=(0, 0),
                                query_layouts=_layouts(6, 3))
    q = torch.randn(9, 4, head_size, device=DEV, dtype=dtype)
    k = torch.randn(9, 2, head_size, device=DEV, dtype=dtype)
    v = torch.randn(9, 2, head_size, device=DEV, dtype=dtype)
    _run_and_compare(cache, md, q, k, v)


def test_qwen_gqa_group():
    torch.manual_seed(20260822)
    cache = _cache(128, torch.bfloat16, block_size=4, hq=28, hkv=4)
    _randomise(cache)
    md = PagedAttentionMetadata(block_tables=((7, 1), (4,)), num_computed_tokens=(0, 0),
                                query_layouts=_layouts(6, 3))
    q = torch.randn(9, 28, 128, device=DEV, dtype=torch.bfloat16)
    k = torch.randn(9, 4, 128, device=DEV, dtype=torch.bfloat16)
    v = torch.randn(9, 4, 128, device=DEV, dtype=torch.bfloat16)
    _run_and_compare(cache, md, q, k, v)


def test_qwen_gqa_across_history_chunks():
    torch.manual_seed(20260822)
    cache = _cache(128, torch.bfloat16, block_size=16, hq=28, hkv=4)
    prefix = 130
    pk = torch.randn(prefix, 4, 128, device=DEV, dtype=torch.bfloat16)
    pv = torch.randn(prefix, 4, 128, device=DEV, dtype=torch.bfloat16)
    cache.write("attention", pk, pv, torch.arange(prefix, device=DEV))
    md = PagedAttentionMetadata(block_tables=(tuple(range(9)),), num_computed_tokens=(prefix,),
                                query_layouts=_layouts(1))
    q = torch.randn(1, 28, 128, device=DEV, dtype=torch.bfloat16)
    k = torch.randn(1, 4, 128, device=DEV, dtype=torch.bfloat16)
    v = torch.randn(1, 4, 128, device=DEV, dtype=torch.bfloat16)
    _run_and_compare(cache, md, q, k, v)


@pytest.mark.parametrize("dtype", (torch.float16, torch.bfloat16))
@pytest.mark.parametrize("prefix", (130, 15, 511))
def test_decode_ignores_unwritten_slots(dtype, prefix):
    """Slots past the context end (never written, here NaN) do not leak into
    the output: the split-context kernel must not weight them even by zero."""

    torch.manual_seed(prefix)
    cache = _cache(128, dtype, block_size=16, hq=28, hkv=4, num_blocks=40)
    layer = cache.layer("attention")
    layer.keys.fill_(float("nan"))
    layer.values.fill_(float("nan"))
    pk = torch.randn(prefix, 4, 128, device=DEV, dtype=dtype)
    pv = torch.randn(prefix, 4, 128, device=DEV, dtype=dtype)
    cache.write("attention", pk, pv, torch.arange(prefix, device=DEV))
    pages = -(-(prefix + 1) // 16)
    md = PagedAttentionMetadata(block_tables=(tuple(range(pages)),), num_computed_tokens=(prefix,),
                                query_layouts=_layouts(1))
    q = torch.randn(1, 28, 128, device=DEV, dtype=dtype)
    k = torch.randn(1, 4, 128, device=DEV, dtype=dtype)
    v = torch.randn(1, 4, 128, device=DEV, dtype=dtype)
    _run_and_compare(cache, md, q, k, v)


def test_packed_tree_visibility():
    torch.manual_seed(20260819)
    cache = _cache(64, torch.float16)
    _randomise(cache)
    md = PagedAttentionMetadata(block_tables=((7, 1), (4, 6)), num_computed_tokens=(0, 0),
                                query_layouts=(QueryLayout((-1, 0, 0, 2)), QueryLayout((-1, 0, 0))))
    q = torch.randn(7, 4, 64, device=DEV, dtype=torch.float16)
    k = torch.randn(7, 2, 64, device=DEV, dtype=torch.float16)
    v = torch.randn(7, 2, 64, device=DEV, dtype=torch.float16)
    _run_and_compare(cache, md, q, k, v)


def test_decode_after_prefill():
    torch.manual_seed(20260817)
    cache = _cache(64, torch.float16)
    _randomise(cache)
    pre = PagedAttentionMetadata(block_tables=((3, 0, 5), (2, 6)), num_computed_tokens=(0, 0),
                                 query_layouts=_layouts(5, 3))
    _run_and_compare(cache, pre, *(torch.randn(8, h, 64, device=DEV, dtype=torch.float16)
                                   for h in (4, 2, 2)))
    dec = PagedAttentionMetadata(block_tables=((3, 0, 5), (2, 6)), num_computed_tokens=(5, 3),
                                 query_layouts=_layouts(1, 1))
    _run_and_compare(cache, dec, *(torch.randn(2, h, 64, device=DEV, dtype=torch.float16)
                                   for h in (4, 2, 2)))


def test_shared_readonly_prefix():
    torch.manual_seed(20260817)
    cache = _cache(64, torch.float16)
    _randomise(cache)
    cache.write("attention", torch.randn(2, 2, 64, device=DEV, dtype=torch.float16),
                torch.randn(2, 2, 64, device=DEV, dtype=torch.float16), torch.tensor([0, 1], device=DEV))
    md = PagedAttentionMetadata(block_tables=((0, 5), (0, 7)), num_computed_tokens=(2, 2),
                                query_layouts=_layouts(1, 1), num_readonly_prefix_blocks=(1, 1))
    _run_and_compare(cache, md, *(torch.randn(2, h, 64, device=DEV, dtype=torch.float16)
                                  for h in (4, 2, 2)))


def test_unused_lookahead_slots():
    torch.manual_seed(20260817)
    cache = _cache(64, torch.float16)
    _randomise(cache)
    md = PagedAttentionMetadata(block_tables=((8, 3, 12), (10, 14)), num_computed_tokens=(0, 0),
                                query_layouts=_layouts(3, 1), num_reserved_query_tokens=(5, 4))
    _run_and_compare(cache, md, *(torch.randn(4, h, 64, device=DEV, dtype=torch.float16)
                                  for h in (4, 2, 2)))


ATTN = np.load(GOLDEN / "paged_attn.npz")
ATTN_INDEX = json.loads(bytes(ATTN["index_json"]).decode())


def _golden(name, key, dtype):
    arr = ATTN[f"{name}_{key}"]
    if dtype == "bfloat16":
        return torch.from_numpy(arr.view(np.int16)).view(torch.bfloat16)
    return torch.from_numpy(arr)


@pytest.mark.parametrize("case", [c for c in ATTN_INDEX if c["dtype"] != "float32"],
                         ids=[c["name"] for c in ATTN_INDEX if c["dtype"] != "float32"])
def test_reference_golden_outputs(case):
    dtype = getattr(torch, case["dtype"])
    cache = _cache(case["d"], dtype, block_size=case["bs"], hq=case["hq"], hkv=case["hkv"],
                   num_blocks=case["nb"])
    layer = cache.layer("attention")
    layer.keys.copy_(_golden(case["name"], "k_before", case["dtype"]).to(DEV))
    layer.values.copy_(_golden(case["name"], "v_before", case["dtype"]).to(DEV))
    md = PagedAttentionMetadata(
        block_tables=tuple(tuple(t) for t in case["tables"]),
        num_computed_tokens=tuple(case["computed"]),
        query_layouts=tuple(QueryLayout(tuple(p)) for p in case["layouts"]),
        num_reserved_query_tokens=tuple(case.get("reserved") or ()),
        num_readonly_prefix_blocks=tuple(case.get("readonly") or ()),
    )
    q, k, v = (_golden(case["name"], key, case["dtype"]).to(DEV) for key in ("q", "k", "v"))
    out = B200PagedAttentionBackend().create(cache, md).forward("attention", q, k, v, scale=case["scale"])
    tol = 3e-3 if dtype == torch.float16 else 2e-2
    torch.testing.assert_close(out.cpu(), _golden(case["name"], "o", case["dtype"]), atol=tol, rtol=tol)
    assert torch.equal(_bits(layer.keys.cpu()), _bits(_golden(case["name"], "k_after", case["dtype"])))
    assert torch.equal(_bits(layer.values.cpu()), _bits(_golden(case["name"], "v_after", case["dtype"])))


def decode_batch(num_seqs, ctx_lo, ctx_hi, hq, hkv, d, dtype, *, num_blocks, seed, block_size=16):
    """Seeded decode workload: contexts ~ U[ctx_lo, ctx_hi], tables carved from
    a random permutation of the block pool, K/V pages ~ N(0, 1)."""

    gen = torch.Generator().manual_seed(seed)
    ctx = torch.randint(ctx_lo, ctx_hi + 1, (num_seqs,), generator=gen).tolist()
    perm = torch.randperm(num_blocks, generator=gen).tolist()
    tables, offset = [], 0
    for c in ctx:
        n = -(-c // block_size)
        tables.append(tuple(perm[offset:offset + n]))
        offset += n
    assert offset <= num_blocks
    md = PagedAttentionMetadata(block_tables=tuple(tables), num_computed_tokens=tuple(c - 1 for c in ctx),
                                query_layouts=_layouts(*([1] * num_seqs)))
    spec = ModelKVCacheSpec((AttentionLayerSpec("attention", hq, hkv, d),))
    cache = PagedKVCache(spec, PagedKVCacheConfig(num_blocks, block_size, dtype=dtype, device=DEV))
    layer = cache.layer("attention")
    torch.manual_seed(seed)
    layer.keys.normal_()
    layer.values.normal_()
    q = torch.randn(num_seqs, hq, d, device=DEV, dtype=dtype)
    k = torch.randn(num_seqs, hkv, d, device=DEV, dtype=dtype)
    v = torch.randn(num_seqs, hkv, d, device=DEV, dtype=dtype)
    return cache, md, q, k, v


def _check_decode(cache, md, q, k, v):
    scale = 1.0 / sqrt(q.shape[-1])
    out = B200PagedAttentionBackend().create(cache, md).forward("attention", q, k, v, scale=scale)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    layer = cache.layer("attention")
    slots = md.slot_mapping(block_size=cache.config.block_size, device=DEV)
    flat_k = layer.keys.view(-1, *k.shape[1:])
    assert torch.equal(_bits(flat_k.index_select(0, slots)), _bits(k.contiguous()))
    expected = opa.attend_dense_fp64(
        q.cpu(), layer.keys.cpu(), layer.values.cpu(), md.block_tables, md.num_computed_tokens,
        [layout.parent_indices for layout in md.query_layouts], scale=scale)
    rounded = expected.to(q.dtype).double()
    max_abs, rel = oawq.error_metrics(out.double().cpu().numpy(), rounded.numpy())
    assert max_abs <= 2e-2 and rel <= 1e-3, (max_abs, rel)
    return out


@pytest.mark.parametrize("dtype", (torch.bfloat16, torch.float16))
@pytest.mark.parametrize("hq,hkv,d", [(28, 4, 128), (8, 8, 128), (32, 2, 64), (16, 1, 128)])
def test_decode_split_context(dtype, hq, hkv, d):
    cache, md, q, k, v = decode_batch(6, 1, 700, hq, hkv, d, dtype, num_blocks=512, seed=hq * 31 + d)
    _check_decode(cache, md, q, k, v)


def test_decode_baseline_config2():
    cache, md, q, k, v = decode_batch(64, 512, 4096, 28, 4, 128, torch.bfloat16, num_blocks=40000,
                                      seed=20261201)
    _check_decode(cache, md, q, k, v)


def decode_batch_ctx(ctx, hq, hkv, d, dtype, *, seed, block_size=16):
    """Decode workload with the given context lengths (tables carved from a
    random permutation of a pool that just holds them)."""

    gen = torch.Generator().manual_seed(seed)
    pages = sum(-(-c // block_size) for c in ctx)
    perm = torch.randperm(pages + 7, generator=gen).tolist()
    tables, offset = [], 0
    for c in ctx:
        n = -(-c // block_size)
        tables.append(tuple(perm[offset:offset + n]))
        offset += n
    md = PagedAttentionMetadata(block_tables=tuple(tables), num_computed_tokens=tuple(c - 1 for c in ctx),
                                query_layouts=_layouts(*([1] * len(ctx))))
    spec = ModelKVCacheSpec((AttentionLayerSpec("attention", hq, hkv, d),))
    cache = PagedKVCache(spec, PagedKVCacheConfig(pages + 7, block_size, dtype=dtype, device=DEV))
    layer = cache.layer("attention")
    torch.manual_seed(seed)
    layer.keys.normal_()
    layer.values.normal_()
    n = len(ctx)
    q = torch.randn(n, hq, d, device=DEV, dtype=dtype)
    k = torch.randn(n, hkv, d, device=DEV, dtype=dtype)
    v = torch.randn(n, hkv, d, device=DEV, dtype=dtype)
    return cache, md, q, k, v


_BALANCED_CASES = {
    # 32+ requests with 2 or 4 KV heads per CTA run the balanced decode: one
    # wave of CTAs over the requests' pages laid end to end.
    "short_contexts_many_per_cta": (dict(n=32, lo=1, hi=40), (28, 4, 128)),
    "300_requests": (dict(n=300, lo=1, hi=100), (28, 4, 128)),
    "two_head_groups_long": (dict(n=48, lo=1, hi=12000), (16, 8, 64)),
    "extreme_mix": (dict(n=40, choices=(1, 16, 17, 1000, 9000)), (32, 2, 64)),
}


@pytest.mark.parametrize("dtype", (torch.bfloat16, torch.float16))
@pytest.mark.parametrize("name", sorted(_BALANCED_CASES))
def test_decode_balanced_ranges(dtype, name):
    shape, (hq, hkv, d) = _BALANCED_CASES[name]
    rng = np.random.default_rng(len(name) * 7 + (dtype == torch.float16))
    if "choices" in shape:
        ctx = [int(x) for x in rng.choice(shape["choices"], size=shape["n"])]
    else:
        ctx = [int(x) for x in rng.integers(shape["lo"], shape["hi"] + 1, size=shape["n"])]
    cache, md, q, k, v = decode_batch_ctx(ctx, hq, hkv, d, dtype, seed=len(ctx))
    _check_decode(cache, md, q, k, v)


def test_decode_balanced_replays_are_identical():
    """Graph replays of the balanced decode (merge semaphores reset by the
    merging CTA) give bit-identical outputs, equal to the eager call."""

    cache, md, q, k, v = decode_batch(64, 512, 4096, 28, 4, 128, torch.bfloat16, num_blocks=40000,
                                      seed=20261201)
    scale = 1.0 / sqrt(q.shape[-1])
    eager = _check_decode(cache, md, q, k, v)
    ctx = B200PagedAttentionBackend().create(cache, md)
    out = torch.empty_like(q)
    ctx.launch("attention", q, k, v, scale=scale, out=out, write_kv=False)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ctx.launch("attention", q, k, v, scale=scale, out=out, write_kv=False)
    for _ in range(3):
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(_bits(out), _bits(eager))
    assert _native.device_error() == 0


def test_decode_single_token_context():
    cache, md, q, k, v = decode_batch(3, 1, 1, 28, 4, 128, torch.bfloat16, num_blocks=8, seed=3)
    _check_decode(cache, md, q, k, v)


def test_layer_runs_once_and_dtype_is_checked():
    cache, md, q, k, v = decode_batch(2, 5, 40, 28, 4, 128, torch.bfloat16, num_blocks=16, seed=4)
    ctx = B200PagedAttentionBackend().create(cache, md)
    ctx.forward("attention", q, k, v, scale=0.1)
    with pytest.raises(KVCacheError, match="ran more than once"):
        ctx.forward("attention", q, k, v, scale=0.1)
    ctx2 = B200PagedAttentionBackend().create(cache, md)
    with pytest.raises(KVCacheError, match="dtype and device"):
        ctx2.forward("attention", q.half(), k.half(), v.half(), scale=0.1)
    assert ctx.layer_ids == frozenset({"attention"})


def test_strided_qkv_views_are_accepted():
    """Q/K/V as views of one fused QKV row, as the model produces them."""

    cache, md, q, k, v = decode_batch(4, 20, 90, 28, 4, 128, torch.bfloat16, num_blocks=64, seed=8)
    fused = torch.cat([q.reshape(4, -1), k.reshape(4, -1), v.reshape(4, -1)], dim=1)
    qv, kv_, vv = fused.split([28 * 128, 4 * 128, 4 * 128], dim=1)
    out = _check_decode(cache, md, qv.view(4, 28, 128), kv_.view(4, 4, 128), vv.view(4, 4, 128))
    assert out.shape == (4, 28, 128)


def test_compaction_moves_retained_queries_like_the_reference():
    """The reference's compaction test (tests/test_paged_attention.py:178-228)
    through ``compact_kv`` (native plan + ``lvb_kv_move_rows``; head size 8
    instead of 4: the kernel moves 16-byte rows): retained queries (0, 2, 4)
    land in slots (6, 7, 0), the readonly prefix block is untouched, and the
    cache equals the one the cache's own ``compact`` produces."""

    spec = ModelKVCacheSpec((AttentionLayerSpec("attention", 2, 2, 8),))
    device = torch.device("cuda", 0)
    cache = PagedKVCache(spec, PagedKVCacheConfig(4, 2, dtype=torch.float16, device=device))
    layer = cache.layer("attention")
    layer.keys.zero_()
    layer.values.zero_()
    prefix_keys = torch.arange(32, dtype=torch.float32).reshape(2, 2, 8).half().to(device)
    prefix_values = prefix_keys + 100
    cache.write("attention", prefix_keys, prefix_values, torch.tensor([2, 3], device=device))
    md = PagedAttentionMetadata(block_tables=((1, 3, 0, 2),), num_computed_tokens=(2,),
                                query_layouts=(QueryLayout((-1, 0, 0, 2, 3)),), num_readonly_prefix_blocks=(1,))
    query_keys = (torch.arange(80, dtype=torch.float32).reshape(5, 2, 8) + 40).half().to(device)
    query_values = query_keys + 200
    cache.write("attention", query_keys, query_values, md.slot_mapping(block_size=2, device=device))
    twin = PagedKVCache(spec, PagedKVCacheConfig(4, 2, dtype=torch.float16, device=device))
    twin.layer("attention").keys.copy_(layer.keys)
    twin.layer("attention").values.copy_(layer.values)
    args = dict(num_computed_tokens=2, num_query_tokens=5, num_reserved_query_tokens=5,
                retained_query_indices=(0, 2, 4), num_readonly_prefix_blocks=1)
    moved = compact_kv(cache, md.block_tables[0], **args)
    assert twin.compact(md.block_tables[0], **args) == moved
    torch.cuda.synchronize()
    assert moved == 2
    assert torch.equal(layer.keys, twin.layer("attention").keys)
    assert torch.equal(layer.values, twin.layer("attention").values)
    assert torch.equal(layer.keys[1], prefix_keys)
    flat_k = layer.keys.view(8, 2, 8)
    flat_v = layer.values.view(8, 2, 8)
    assert torch.equal(flat_k[[6, 7, 0]], query_keys[[0, 2, 4]])
    assert torch.equal(flat_v[[6, 7, 0]], query_values[[0, 2, 4]])
    assert _native.device_error() == 0


def test_staging_ring_copies_groups_and_grows():
    """The pinned ring (native slot events): group copies land intact across
    ring wrap-around and buffer growth; each view is read before the next copy."""

    from light_vllm_b200.staging import SingleStepStaging

    staging = SingleStepStaging(DEV)
    for i in range(11):
        tail = np.arange(i * 97 + 1, dtype=np.int32)
        head, rest = staging.copy_groups([i, i + 1, i + 2], tail)
        assert head.tolist() == [i, i + 1, i + 2]
        assert torch.equal(rest.cpu(), torch.from_numpy(tail))
        packed = staging.copy_packed(5, lambda host: host[:5].copy_(torch.arange(5, dtype=torch.int32) + i).numel())
        assert packed.tolist() == [i, i + 1, i + 2, i + 3, i + 4]


def _mixed_batch(requests, hq, hkv, d, dtype, *, seed, block_size=16):
    """A packed batch of (computed tokens, query layout parents) requests over
    tables carved from a random permutation of the pool."""

    gen = torch.Generator().manual_seed(seed)
    need = [-(-(c + len(p)) // block_size) for c, p in requests]
    pages = sum(need)
    perm = torch.randperm(pages + 5, generator=gen).tolist()
    tables, offset = [], 0
    for n in need:
        tables.append(tuple(perm[offset:offset + n]))
        offset += n
    md = PagedAttentionMetadata(block_tables=tuple(tables), num_computed_tokens=tuple(c for c, _ in requests),
                                query_layouts=tuple(QueryLayout(tuple(p)) for _, p in requests))
    spec = ModelKVCacheSpec((AttentionLayerSpec("attention", hq, hkv, d),))
    cache = PagedKVCache(spec, PagedKVCacheConfig(pages + 5, block_size, dtype=dtype, device=DEV))
    layer = cache.layer("attention")
    torch.manual_seed(seed)
    layer.keys.normal_()
    layer.values.normal_()
    t = sum(len(p) for _, p in requests)
    q = torch.randn(t, hq, d, device=DEV, dtype=dtype)
    k = torch.randn(t, hkv, d, device=DEV, dtype=dtype)
    v = torch.randn(t, hkv, d, device=DEV, dtype=dtype)
    return cache, md, q, k, v


def _linear(n):
    return tuple(range(-1, n - 1))


_MIXED_CASES = {
    # a prefill chunk after a long prefix, a fresh short prompt, and decodes
    "chunk_prompt_decodes": [(500, _linear(300)), (0, _linear(7)), (37, _linear(1)), (2999, _linear(1)),
                             (16, _linear(1))],
    # prefill only: ragged prompts, one of them a single token
    "prefill_only": [(0, _linear(129)), (0, _linear(1)), (48, _linear(64)), (0, _linear(33))],
    # tree (speculative) layouts beside a linear chunk and decodes
    "tree": [(200, (-1, 0, 0, 1, 1, 2, 5, -1)), (63, _linear(1)), (10, _linear(20)), (0, (-1, 0, 1, 0))],
}


@pytest.mark.parametrize("dtype", (torch.bfloat16, torch.float16))
@pytest.mark.parametrize("hq,hkv,d", [(28, 4, 128), (10, 2, 128), (16, 2, 64), (8, 8, 128)])
@pytest.mark.parametrize("case", sorted(_MIXED_CASES))
def test_prefill_tiles_and_mixed_batches(case, dtype, hq, hkv, d):
    """Prefill chunks, mixed prefill + decode batches and tree layouts (16-token
    pages, head sizes 64 / 128) run the tensor-core tile kernel, a mixed
    batch's one-token requests the split decode kernel: against a float64
    evaluation of the same visible positions, rounded to the cache dtype,
    max-abs <= 2e-2 and rel-L2 <= 1e-3; this step's K/V rows bit-exact in
    their slots."""

    cache, md, q, k, v = _mixed_batch(_MIXED_CASES[case], hq, hkv, d, dtype, seed=hq * 7 + d + len(case))
    _check_decode(cache, md, q, k, v)


def test_config5_shaped_mixed_step():
    """BASELINE config 5 per TP = 4 rank (10 query / 2 KV heads, D = 128): one
    2048-token prefill chunk and 64 decodes with contexts in [256, 8192],
    fp16 cache."""

    gen = torch.Generator().manual_seed(5)
    ctx = torch.randint(256, 8193, (64,), generator=gen).tolist()
    requests = [(0, _linear(2048))] + [(c - 1, _linear(1)) for c in ctx]
    cache, md, q, k, v = _mixed_batch(requests, 10, 2, 128, torch.float16, seed=55)
    _check_decode(cache, md, q, k, v)
