"""GPU parity of the warp-MMA decode kernel (csrc/awq_mma.cuh) against the
CPU oracle.

lvb_awq_linear_packed runs it for 2..16 token rows over the packed layout:
one token tile (m <= 8) or two (m <= 16), one split or many, groups of 32 /
64 / 128 / 256 and per-column groups, stages cut short at the end of a range
(runs per range not a multiple of eight), with and without bias.  The kernel
multiplies the reference's fp16-rounded weight (modeling/quantization/
awq.py:433-450) by the fp16 x with fp32 accumulation, so the tolerance is
the north-star max-abs 2e-2 and rel-L2 1e-3 against the fp64-accumulated
oracle of that arithmetic (awq.py:453-465) and, per element, max-abs plus
one fp16 ulp of the output (the output's own rounding once it exceeds 32).
"""

from __future__ import annotations

import functools

import numpy as np
import pytest
import torch

from light_vllm_b200 import _native
from light_vllm_b200.awq import B200AWQScheme
from oracle import awq as oawq

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
MAX_ABS = 2e-2
REL_L2 = 1e-3


@functools.lru_cache(maxsize=None)
def _case(k, n, g, seed):
    """Weights, 16 rows of x, bias and the oracle's outputs for all 16 rows
    (each output row depends on its own x row only, so an m-row call is
    checked against the first m rows)."""

    qweight, qzeros, scales = oawq.random_checkpoint(k, n, g, seed=seed)
    rng = np.random.default_rng(seed + 1)
    x = rng.standard_normal((16, k)).astype(np.float16)
    bias = rng.standard_normal(n).astype(np.float16)
    expected = oawq.linear_fp32(x, qweight, qzeros, scales, g, bias)
    return qweight, qzeros, scales, x, bias, expected


def _assert_close(got, expected, what, check_max_abs=True):
    max_abs, rel = oawq.error_metrics(got, expected)
    assert rel <= REL_L2, (what, max_abs, rel)
    if check_max_abs:
        assert max_abs <= MAX_ABS, (what, max_abs, rel)
    excess = np.abs(got - expected) - (MAX_ABS + np.abs(expected) * 2.0**-10)
    assert float(excess.max()) <= 0.0, (what, "per element", float(excess.max()))


def _prepare(qweight, qzeros, scales, g, bias):
    qw, qz, sc = (torch.from_numpy(np.ascontiguousarray(a)).to(DEV) for a in (qweight, qzeros, scales))
    bg = torch.from_numpy(bias).to(DEV) if bias is not None else None
    return B200AWQScheme().prepare(qw, qz, sc, g, bg)


def _check(m, k, n, g, seed):
    qweight, qzeros, scales, x, bias, expected = _case(k, n, g, seed)
    op = _prepare(qweight, qzeros, scales, g, bias)
    xg = torch.from_numpy(x[:m].copy()).to(DEV)
    y = op(xg)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    _assert_close(y.float().cpu().numpy().astype(np.float64), expected[:m], (m, k, n, g))
    return op, xg, y


SHAPES = [
    (3584, 4608, 128),   # 7B merged QKV: many splits
    (3584, 37888, 128),  # 7B merged gate_up: one split per tile
    (18944, 3584, 128),  # 7B down: 28 tiles, long k
    (896, 4864, 128),
    (512, 1024, 64),
    (1024, 256, 256),
    (896, 256, 896),     # per-column groups
    (192, 384, 32),      # six runs per range: one stage cut short
]


@pytest.mark.parametrize("m", [2, 3, 5, 8, 9, 12, 16])
@pytest.mark.parametrize("k,n,g", SHAPES)
def test_mma_decode_batches(m, k, n, g):
    _check(m, k, n, g, seed=k + n + g)


def test_mma_split_reduction_is_deterministic_and_reusable():
    op, xg, y = _check(16, 3584, 4608, 128, seed=41)
    for _ in range(3):
        assert torch.equal(op(xg), y)
    torch.cuda.synchronize()
    assert _native.device_error() == 0


@pytest.mark.parametrize("m", [2, 16])
def test_mma_keeps_precision_beside_massive_outliers(m):
    """One channel per (token, group) at +-U[1e3, 3e4] against N(0, 0.2), and
    half of the columns with a zero weight (q == z) at every outlier channel,
    so their outputs stay O(1): there, max-abs <= 2e-2 and rel-L2 <= 1e-3
    against the fp32 oracle with no widened bound (the fp16 activations enter
    the MMA unchanged, so the small ones keep their precision); everywhere,
    rel-L2 and max-abs plus one fp16 ulp of the output."""

    k, n, g = 3584, 4736, 128
    qweight, qzeros, scales = oawq.random_checkpoint(k, n, g, seed=950 + m)
    rng = np.random.default_rng(900 + m)
    groups = k // g
    x = rng.standard_normal((m, k)) * 0.2
    channels = rng.integers(0, g, size=groups) + np.arange(groups) * g
    x[:, channels] = rng.uniform(1e3, 3e4, size=(m, groups)) * rng.choice((-1.0, 1.0), size=(m, groups))
    x = x.astype(np.float16)
    codes, zeros = oawq.unpack(qweight), oawq.unpack(qzeros)
    zero_cols = np.flatnonzero(rng.random(n) < 0.5)
    for gi, c in enumerate(channels):
        codes[c, zero_cols] = zeros[gi, zero_cols]
    qweight = oawq.pack(codes)
    op = _prepare(qweight, qzeros, scales, g, None)
    y = op(torch.from_numpy(x).to(DEV))
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    got = y.float().cpu().numpy().astype(np.float64)
    expected = oawq.linear_fp32(x, qweight, qzeros, scales, g, None)
    _assert_close(got[:, zero_cols], expected[:, zero_cols], m)
    _assert_close(got, expected, m, check_max_abs=False)


def test_mma_row_slices_of_a_larger_batch():
    """Rows 0..m-1 of the same x give the same outputs at every m (token rows
    past m are never read; each row's result does not depend on the others)."""

    k, n, g = 3584, 4608, 128
    qweight, qzeros, scales = oawq.random_checkpoint(k, n, g, seed=5)
    x = np.random.default_rng(6).standard_normal((16, k)).astype(np.float16)
    dev = [torch.from_numpy(np.ascontiguousarray(a)).to(DEV) for a in (qweight, qzeros, scales, x)]
    op = B200AWQScheme().prepare(dev[0], dev[1], dev[2], g, None)
    full = op(dev[3])
    for m in (2, 7, 8, 9, 15):
        part = op(dev[3][:m].contiguous())
        assert torch.equal(part, full[:m]), m
    torch.cuda.synchronize()
    assert _native.device_error() == 0
