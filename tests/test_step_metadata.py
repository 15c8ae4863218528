"""Native step-metadata validation and packing against the oracle (CPU only).

``lvb_pack_step_metadata`` is host code (no device calls).  Over the golden
metadata cases and a few thousand random ones (aliasing, shared read-only
prefixes, out-of-range ids, coverage errors), it must report exactly the first
violation the reference reports, with the same message, and otherwise pack the
same block tables, computed counts, query starts and request indices.
"""

from __future__ import annotations

import ctypes
import json
import random
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest

from light_vllm_b200 import KVCacheError, _native
from light_vllm_b200.paged_attention import StepMetadataPacker
from oracle import paged_attention as opa
from oracle.paged_cache import reference_types

# The packer reads light-vllm's own PagedAttentionMetadata / QueryLayout
# objects when light-vllm is importable, else the oracle's stand-ins.
_T = reference_types()
PagedAttentionMetadata, QueryLayout, linear_query_layout = _T.PagedAttentionMetadata, _T.QueryLayout, _T.linear_query_layout

META = json.loads((Path(__file__).resolve().parent / "golden" / "paged_meta.json").read_text())


def native_pack(tables, computed, qlens, reserved, readonly, num_blocks, block_size):
    lib = _native.library()
    offsets = np.zeros(len(tables) + 1, dtype=np.int64)
    np.cumsum([len(t) for t in tables], out=offsets[1:])
    flat = np.array([b for t in tables for b in t] or [0], dtype=np.int32)
    arrs = [np.asarray(v, dtype=np.int32) for v in (computed, qlens, reserved, readonly)]
    n = len(tables)
    cap = n * max(len(t) for t in tables) + 4 * n + 1 + sum(qlens)
    out = np.zeros(max(cap, 1), dtype=np.int32)
    stride, ntok = ctypes.c_int64(0), ctypes.c_int64(0)
    status = lib.lvb_pack_step_metadata(flat.ctypes.data, offsets.ctypes.data,
                                        *(a.ctypes.data for a in arrs), n, num_blocks, block_size,
                                        out.ctypes.data, out.size, ctypes.byref(stride), ctypes.byref(ntok))
    if status == _native.LVB_ERR_METADATA:
        return lib.lvb_last_error().decode(), None
    assert status == _native.LVB_OK, lib.lvb_last_error()
    return None, (out, int(stride.value), int(ntok.value))


def packer_pack(packer, tables, computed, qlens, reserved, readonly, num_blocks, block_size):
    """The product path: Python objects -> ``_hostpack.gather_step`` ->
    ``lvb_pack_step_metadata`` through ``StepMetadataPacker``."""

    md = SimpleNamespace(block_tables=tuple(tuple(t) for t in tables), num_computed_tokens=tuple(computed),
                         query_layouts=tuple(linear_query_layout(q) for q in qlens),
                         num_reserved_query_tokens=tuple(reserved), num_readonly_prefix_blocks=tuple(readonly))
    step = packer.gather(md)
    out = np.zeros(step.packed_size, dtype=np.int32)
    try:
        packer.pack(num_blocks, block_size, out.ctypes.data, out.size)
    except KVCacheError as exc:
        return str(exc), None, step
    return None, (out, step.max_blocks, step.num_tokens), step


def oracle_error(tables, computed, reserved, readonly, num_blocks, block_size):
    try:
        opa.validate_block_tables(tables, computed, reserved, readonly,
                                  num_blocks=num_blocks, block_size=block_size)
    except opa.KVCacheError as exc:
        return str(exc)
    return None


def check_payload(payload, tables, computed, qlens):
    out, stride, ntok = payload
    n = len(tables)
    assert stride == max(len(t) for t in tables)
    for r, t in enumerate(tables):
        assert list(out[r * stride : r * stride + len(t)]) == list(t)
    base = n * stride
    assert list(out[base : base + n]) == list(computed)
    assert list(out[base + n : base + 2 * n + 1]) == list(opa.query_start_loc(qlens))
    assert list(out[base + 2 * n + 1 : base + 2 * n + 1 + ntok]) == list(opa.request_indices(qlens))
    # Launch order: one-token requests first, then the rest; each part by
    # descending context length (computed + query tokens), ties by index.
    order = list(out[base + 2 * n + 1 + ntok : base + 3 * n + 1 + ntok])
    assert order == sorted(range(n), key=lambda r: (qlens[r] != 1, -(computed[r] + qlens[r])))
    assert list(out[base + 3 * n + 1 + ntok : base + 4 * n + 1 + ntok]) == [computed[r] for r in order]


@pytest.mark.parametrize("case", META, ids=[c["name"] for c in META])
def test_golden_cases(case):
    qlens = [len(p) for p in case["layouts"]]
    reserved = case.get("reserved") or qlens
    readonly = case.get("readonly") or [0] * len(qlens)
    error, payload = native_pack(case["tables"], case["computed"], qlens, reserved, readonly,
                                 case["num_blocks"], case["block_size"])
    assert error == case["validate_error"]
    if error is None:
        check_payload(payload, case["tables"], case["computed"], qlens)


@pytest.mark.parametrize("case", META, ids=[c["name"] for c in META])
def test_golden_cases_through_the_metadata_objects(case):
    """The product path over the metadata objects themselves (light-vllm's own
    ``PagedAttentionMetadata`` when importable): gather + validate + pack give
    the reference's validation message, or the packed payload."""

    md = PagedAttentionMetadata(
        block_tables=tuple(tuple(t) for t in case["tables"]),
        num_computed_tokens=tuple(case["computed"]),
        query_layouts=tuple(QueryLayout(tuple(p)) for p in case["layouts"]),
        num_reserved_query_tokens=tuple(case.get("reserved") or ()),
        num_readonly_prefix_blocks=tuple(case.get("readonly") or ()),
    )
    packer = StepMetadataPacker()
    step = packer.gather(md)
    out = np.zeros(step.packed_size, dtype=np.int32)
    try:
        packer.pack(case["num_blocks"], case["block_size"], out.ctypes.data, out.size)
        error = None
    except KVCacheError as exc:
        if _T.source == "light_vllm":
            assert isinstance(exc, _T.KVCacheError)  # the Worker's handlers catch it
        error = str(exc)
    assert error == case["validate_error"]
    if error is None:
        qlens = [len(p) for p in case["layouts"]]
        check_payload((out, step.max_blocks, step.num_tokens), case["tables"], case["computed"], qlens)


def _random_case(rng: random.Random):
    block_size = rng.choice((1, 2, 4, 16))
    num_blocks = rng.randint(4, 40)
    n = rng.randint(1, 5)
    tables, computed, qlens, reserved, readonly = [], [], [], [], []
    shared = [rng.randrange(num_blocks) for _ in range(3)]
    for _ in range(n):
        q = rng.randint(1, 4)
        res = q + rng.choice((0, 0, 1, 3))
        c = rng.randint(0, 3 * block_size)
        need = -(-(c + res) // block_size)
        length = max(0, need + rng.choice((0, 0, 0, 0, -1, 1)))
        ro = rng.choice((0, 0, 1, 2))
        table = []
        for i in range(length):
            if i < len(shared) and rng.random() < 0.4:
                table.append(shared[i])
            elif rng.random() < 0.05:
                table.append(num_blocks + rng.randint(0, 3))
            else:
                table.append(rng.randrange(num_blocks))
        if not table:
            table = [rng.randrange(num_blocks)]
        tables.append(tuple(table))
        computed.append(c)
        qlens.append(q)
        reserved.append(res)
        readonly.append(ro)
    return tables, computed, qlens, reserved, readonly, num_blocks, block_size


def test_random_cases_agree_with_the_oracle():
    rng = random.Random(20261201)
    packer = StepMetadataPacker()
    seen_errors = set()
    for _ in range(3000):
        tables, computed, qlens, reserved, readonly, nb, bs = _random_case(rng)
        expected = oracle_error(tables, computed, reserved, readonly, nb, bs)
        error, payload = native_pack(tables, computed, qlens, reserved, readonly, nb, bs)
        assert error == expected, (tables, computed, reserved, readonly, nb, bs)
        error2, payload2, step = packer_pack(packer, tables, computed, qlens, reserved, readonly, nb, bs)
        assert error2 == expected, (tables, computed, reserved, readonly, nb, bs)
        assert step.num_tokens == sum(qlens) and step.max_query_len == max(qlens) and step.linear
        assert step.max_seq_len == max(c + q for c, q in zip(computed, qlens))
        seen_errors.add(expected)
        if error is None:
            check_payload(payload, tables, computed, qlens)
            check_payload(payload2, tables, computed, qlens)
    # The fuzzing reached every rule.
    assert len(seen_errors) >= 6, seen_errors


def test_small_buffer_is_rejected():
    lib = _native.library()
    flat = np.array([0, 1], dtype=np.int32)
    offsets = np.array([0, 2], dtype=np.int64)
    one = np.array([1], dtype=np.int32)
    zero = np.array([0], dtype=np.int32)
    out = np.zeros(2, dtype=np.int32)
    stride, ntok = ctypes.c_int64(0), ctypes.c_int64(0)
    status = lib.lvb_pack_step_metadata(flat.ctypes.data, offsets.ctypes.data, one.ctypes.data,
                                        one.ctypes.data, one.ctypes.data, zero.ctypes.data, 1, 4, 1,
                                        out.ctypes.data, out.size, ctypes.byref(stride), ctypes.byref(ntok))
    assert status == _native.LVB_ERR_WORKSPACE


def test_packer_reads_the_metadata_objects():
    """Gathering from the metadata objects: tuples and lists, tree layouts
    (not linear), ids beyond int32 (reported as out of range, as the
    reference reports any id >= num_blocks), counts beyond int32 refused."""

    packer = StepMetadataPacker()
    md = PagedAttentionMetadata(block_tables=((3, 1), (0,)), num_computed_tokens=(16, 3),
                                query_layouts=(linear_query_layout(2), QueryLayout((-1, 0, 0))))
    step = packer.gather(md)
    assert step == (2, 3, 2, 5, 3, 18, False, 0)
    out = np.zeros(step.packed_size, dtype=np.int32)
    packer.pack(4, 16, out.ctypes.data, out.size)
    assert out.tolist() == [3, 1, 0, 0, 16, 3, 0, 2, 5, 0, 0, 1, 1, 1, 0, 1, 16, 3]

    lists = SimpleNamespace(block_tables=[[3, 1], [0]], num_computed_tokens=[16, 3],
                            query_layouts=[linear_query_layout(2), linear_query_layout(1)],
                            num_reserved_query_tokens=[2, 1], num_readonly_prefix_blocks=[0, 0])
    assert packer.gather(lists).linear

    huge = SimpleNamespace(block_tables=((1 << 40,),), num_computed_tokens=(0,),
                           query_layouts=(linear_query_layout(1),), num_reserved_query_tokens=(1,),
                           num_readonly_prefix_blocks=(0,))
    step = packer.gather(huge)
    out = np.zeros(step.packed_size, dtype=np.int32)
    with pytest.raises(KVCacheError, match="out-of-range physical block"):
        packer.pack(4, 16, out.ctypes.data, out.size)

    bad = SimpleNamespace(block_tables=((0,),), num_computed_tokens=(1 << 40,),
                          query_layouts=(linear_query_layout(1),), num_reserved_query_tokens=(1,),
                          num_readonly_prefix_blocks=(0,))
    with pytest.raises(OverflowError):
        packer.gather(bad)
    short = SimpleNamespace(block_tables=((0,), (1,)), num_computed_tokens=(0,),
                            query_layouts=(linear_query_layout(1),) * 2, num_reserved_query_tokens=(1, 1),
                            num_readonly_prefix_blocks=(0, 0))
    with pytest.raises(ValueError, match="one entry per request"):
        packer.gather(short)


def test_packer_grows_its_buffers_and_reuses_them():
    packer = StepMetadataPacker()
    rng = random.Random(7)
    for n in (1, 64, 3, 200, 5):
        tables = tuple(tuple(range(i * 50, i * 50 + rng.randint(1, 40))) for i in range(n))
        computed = tuple(16 * len(t) - 1 for t in tables)
        md = PagedAttentionMetadata(block_tables=tables, num_computed_tokens=computed,
                                    query_layouts=tuple(linear_query_layout(1) for _ in tables))
        step = packer.gather(md)
        out = np.zeros(step.packed_size, dtype=np.int32)
        packer.pack(n * 50, 16, out.ctypes.data, out.size)
        check_payload((out, step.max_blocks, step.num_tokens), tables, computed, [1] * n)


def test_stage_rejects_violations_before_any_copy():
    """lvb_stage_step_metadata validates (host code) before its device copy:
    a block-table violation returns the reference's message and a missing
    device buffer is refused, with no CUDA call made."""

    lib = _native.library()
    flat = np.array([0, 0], dtype=np.int32)  # one request aliasing block 0 twice
    offsets = np.array([0, 2], dtype=np.int64)
    computed = np.array([17], dtype=np.int32)
    one = np.array([1], dtype=np.int32)
    zero = np.array([0], dtype=np.int32)
    host = np.zeros(16, dtype=np.int32)
    stride, ntok = ctypes.c_int64(0), ctypes.c_int64(0)
    args = (flat.ctypes.data, offsets.ctypes.data, computed.ctypes.data, one.ctypes.data, one.ctypes.data,
            zero.ctypes.data, 1, 4, 16, host.ctypes.data, host.size)
    status = lib.lvb_stage_step_metadata(*args, 8, 16, None, None, ctypes.byref(stride), ctypes.byref(ntok))
    assert status == _native.LVB_ERR_METADATA
    assert lib.lvb_last_error() == b"block table aliases a physical block within one request"
    status = lib.lvb_stage_step_metadata(*args, None, 16, None, None, ctypes.byref(stride), ctypes.byref(ntok))
    assert status == _native.LVB_ERR_INVALID
    assert lib.lvb_event_wait_host(None) == _native.LVB_OK
    assert lib.lvb_event_destroy(None) == _native.LVB_OK


def test_packer_input_types():
    """The gatherer takes any integer-like ids (numpy scalars included),
    refuses non-integers and layouts without ``parent_indices``, and hands
    negative ids to the validator, which reports them as out of range."""

    packer = StepMetadataPacker()

    def md(tables, layouts=None):
        return SimpleNamespace(block_tables=tables, num_computed_tokens=(15,) * len(tables),
                               query_layouts=layouts or (linear_query_layout(1),) * len(tables),
                               num_reserved_query_tokens=(1,) * len(tables),
                               num_readonly_prefix_blocks=(0,) * len(tables))

    step = packer.gather(md(((np.int64(2),), (np.int32(3),))))
    out = np.zeros(step.packed_size, dtype=np.int32)
    packer.pack(4, 16, out.ctypes.data, out.size)
    assert out[:2].tolist() == [2, 3]
    with pytest.raises(TypeError):
        packer.gather(md(((2.0,),)))
    with pytest.raises(AttributeError):
        packer.gather(md(((2,),), layouts=((-1,),)))  # has a length, no parent_indices
    step = packer.gather(md(((-5,),)))
    out = np.zeros(step.packed_size, dtype=np.int32)
    with pytest.raises(KVCacheError, match="out-of-range physical block"):
        packer.pack(4, 16, out.ctypes.data, out.size)


def test_ownership_stamps_reset_between_calls():
    """Ownership is per call: a block listed in one call may be listed again
    by any request of the next call; within a call only a read-only prefix
    block at the same logical index may be shared."""

    shared_ok = ([[7, 1], [7, 2]], [16, 16], [1, 1], [1, 1], [1, 1])
    wrong_index = ([[7, 1], [2, 7]], [16, 16], [1, 1], [1, 1], [1, 1])
    not_readonly = ([[7, 1], [7, 2]], [16, 16], [1, 1], [1, 1], [1, 0])
    for _ in range(3):
        for tables, computed, qlens, reserved, readonly in (shared_ok, ([[7, 1]], [16], [1], [1], [0])):
            error, payload = native_pack(tables, computed, qlens, reserved, readonly, 8, 16)
            assert error is None
        error, _ = native_pack(*wrong_index, 8, 16)
        assert error == "block tables alias a physical block across requests"
        error, _ = native_pack(*not_readonly, 8, 16)
        assert error == "block tables alias a physical block across requests"
        assert oracle_error(wrong_index[0], wrong_index[1], wrong_index[3], wrong_index[4], 8, 16) == error
