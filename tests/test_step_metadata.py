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

import numpy as np
import pytest

from light_vllm_b200 import _native
from oracle import paged_attention as opa

META = json.loads((Path(__file__).resolve().parent / "golden" / "paged_meta.json").read_text())


def native_pack(tables, computed, qlens, reserved, readonly, num_blocks, block_size):
    lib = _native.library()
    offsets = np.zeros(len(tables) + 1, dtype=np.int64)
    np.cumsum([len(t) for t in tables], out=offsets[1:])
    flat = np.array([b for t in tables for b in t] or [0], dtype=np.int32)
    arrs = [np.asarray(v, dtype=np.int32) for v in (computed, qlens, reserved, readonly)]
    n = len(tables)
    cap = n * max(len(t) for t in tables) + 2 * n + 1 + sum(qlens)
    out = np.zeros(max(cap, 1), dtype=np.int32)
    stride, ntok = ctypes.c_int64(0), ctypes.c_int64(0)
    status = lib.lvb_pack_step_metadata(flat.ctypes.data, offsets.ctypes.data,
                                        *(a.ctypes.data for a in arrs), n, num_blocks, block_size,
                                        out.ctypes.data, out.size, ctypes.byref(stride), ctypes.byref(ntok))
    if status == _native.LVB_ERR_METADATA:
        return lib.lvb_last_error().decode(), None
    assert status == _native.LVB_OK, lib.lvb_last_error()
    return None, (out, int(stride.value), int(ntok.value))


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
    seen_errors = set()
    for _ in range(3000):
        tables, computed, qlens, reserved, readonly, nb, bs = _random_case(rng)
        expected = oracle_error(tables, computed, reserved, readonly, nb, bs)
        error, payload = native_pack(tables, computed, qlens, reserved, readonly, nb, bs)
        assert error == expected, (tables, computed, reserved, readonly, nb, bs)
        seen_errors.add(expected)
        if error is None:
            check_payload(payload, tables, computed, qlens)
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
