"""GPU parity of the B200 AWQ scheme against the CPU oracle.

Matrix:
  * the reference's own CUDA test matrix (tests/test_cuda_awq.py:19-57):
    M in {1, 7, 64, 256}, K in {128, 384}, G=32, N=128 with bias, against
    F.linear(x, dequantized, bias), atol 3e-2 / rtol 2e-2; and the TP shard
    narrower than a group (K=896, G=128, N=64, M=7);
  * the BASELINE config-1 shape (M=16, K=896, N=4864, G=128, scales in
    [0.002, 0.02]) and tile-boundary shapes, against the fp64-accumulated
    oracle with the north-star tolerance: max-abs <= 2e-2 and rel-L2 <= 1e-3;
  * bit-exact dequantisation, determinism of the split-K reduction.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from torch.nn import functional as F

from light_vllm_b200 import _native
from light_vllm_b200.awq import B200AWQScheme, b200_awq_dequantize, b200_awq_linear
from oracle import awq as oawq

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
MAX_ABS = 2e-2
REL_L2 = 1e-3


def _gpu(*arrays):
    return [torch.from_numpy(np.ascontiguousarray(a)).to(DEV) for a in arrays]


def _quantized(out_features: int, in_features: int, group: int, seed: int):
    torch.manual_seed(seed)
    weight = torch.randn(out_features, in_features, dtype=torch.float16)
    qweight, qzeros, scales, deq = oawq.quantize_weight(weight, group)
    return qweight, qzeros, scales, deq


@pytest.mark.parametrize("num_tokens", [1, 7, 64, 256])
@pytest.mark.parametrize("inner", [128, 384])
def test_matches_dequantized_linear(num_tokens, inner):
    qweight, qzeros, scales, deq = _quantized(128, inner, 32, 3)
    torch.manual_seed(3)
    x = torch.randn(num_tokens, inner, dtype=torch.float16, device=DEV)
    bias = torch.randn(128, dtype=torch.float16, device=DEV)
    qw, qz, sc, w = _gpu(qweight, qzeros, scales, deq)
    expected = F.linear(x, w, bias)
    actual = b200_awq_linear(x, qw, qz, sc, 32, bias)
    torch.cuda.synchronize()
    torch.testing.assert_close(actual, expected, atol=3e-2, rtol=2e-2)


def test_tp_shard_narrower_than_group():
    qweight, qzeros, scales, deq = _quantized(64, 896, 128, 7)
    torch.manual_seed(7)
    x = torch.randn(7, 896, dtype=torch.float16, device=DEV)
    qw, qz, sc, w = _gpu(qweight, qzeros, scales, deq)
    actual = b200_awq_linear(x, qw, qz, sc, 128, None)
    torch.testing.assert_close(actual, F.linear(x, w), atol=3e-2, rtol=2e-2)


def _check_against_oracle(m, k, n, g, seed, with_bias=True):
    qweight, qzeros, scales = oawq.random_checkpoint(k, n, g, seed=seed)
    rng = np.random.default_rng(seed + 1)
    x = rng.standard_normal((m, k)).astype(np.float16)
    bias = rng.standard_normal(n).astype(np.float16) if with_bias else None
    expected = oawq.linear_fp32(x, qweight, qzeros, scales, g, bias)
    qw, qz, sc, xg = _gpu(qweight, qzeros, scales, x)
    bg = _gpu(bias)[0] if bias is not None else None
    op = B200AWQScheme().prepare(qw, qz, sc, g, bg)
    y = op(xg)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    max_abs, rel = oawq.error_metrics(y.float().cpu().numpy(), expected)
    assert max_abs <= MAX_ABS and rel <= REL_L2, (m, k, n, g, max_abs, rel)
    return op, xg, y


def test_baseline_config1_shape():
    _check_against_oracle(16, 896, 4864, 128, seed=20261201)


@pytest.mark.parametrize(
    "m,k,n,g",
    [
        (1, 896, 4864, 128),
        (2, 1024, 2112, 128),     # partial last n tile
        (15, 96, 256, 32),        # k not a multiple of the 64-wide k tile
        (17, 896, 4864, 128),     # BN=32 split-K
        (33, 512, 1024, 64),      # BN=64
        (65, 640, 512, 128),      # BN=128, no split
        (129, 384, 768, 128),     # BN=256
        (300, 256, 384, 32),      # two m tiles
        (513, 1024, 1280, 128),   # three m tiles, 72B TP=8 QKV width
        (16, 3584, 4608, 128),    # 7B merged QKV
    ],
)
def test_shapes_against_oracle(m, k, n, g):
    _check_against_oracle(m, k, n, g, seed=m * 7919 + k)


def test_split_k_reduction_is_deterministic_and_reusable():
    op, x, y = _check_against_oracle(16, 896, 4864, 128, seed=11)
    for _ in range(3):
        again = op(x)
        assert torch.equal(again, y)
    torch.cuda.synchronize()
    assert _native.device_error() == 0


def test_dequantize_is_bit_exact():
    k, n, g = 256, 512, 64
    qweight, qzeros, scales = oawq.random_checkpoint(k, n, g, seed=5)
    expected = oawq.dequantize(qweight, qzeros, scales, g)
    qw, qz, sc = _gpu(qweight, qzeros, scales)
    w = b200_awq_dequantize(qw, qz, sc, g)
    np.testing.assert_array_equal(w.cpu().numpy().view(np.uint16), expected.view(np.uint16))


def test_multi_dim_inputs_keep_leading_shape():
    qweight, qzeros, scales = oawq.random_checkpoint(256, 512, 128, seed=9)
    qw, qz, sc = _gpu(qweight, qzeros, scales)
    x = torch.randn(2, 3, 256, dtype=torch.float16, device=DEV)
    y = B200AWQScheme().prepare(qw, qz, sc, 128, None)(x)
    assert y.shape == (2, 3, 512)
    flat = B200AWQScheme().prepare(qw, qz, sc, 128, None)(x.reshape(6, 256))
    assert torch.equal(y.reshape(6, 512), flat)


def test_prepare_rejects_bad_layouts():
    qweight, qzeros, scales = oawq.random_checkpoint(256, 512, 128, seed=9)
    qw, qz, sc = _gpu(qweight, qzeros, scales)
    with pytest.raises(ValueError, match="group_size"):
        B200AWQScheme().prepare(qw, qz, sc, 48, None)
    with pytest.raises(ValueError, match="float16"):
        B200AWQScheme().prepare(qw, qz, sc.float(), 128, None)
    with pytest.raises(ValueError, match="bias"):
        B200AWQScheme().prepare(qw, qz, sc, 128, torch.zeros(7, dtype=torch.float16, device=DEV))
    with pytest.raises(ValueError, match="activations must be float16"):
        B200AWQScheme().prepare(qw, qz, sc, 128, None)(torch.zeros(1, 256, device=DEV))


@pytest.mark.parametrize("m,k,n,g", [(1, 896, 4864, 128), (16, 512, 1024, 64), (40, 96, 256, 32)])
def test_checkpoint_layout_entry_for_small_batches(m, k, n, g):
    """lvb_awq_linear (AutoAWQ layout, no packing) also serves decode sizes."""

    qweight, qzeros, scales = oawq.random_checkpoint(k, n, g, seed=m + k + n)
    rng = np.random.default_rng(m)
    x = rng.standard_normal((m, k)).astype(np.float16)
    expected = oawq.linear_fp32(x, qweight, qzeros, scales, g, None)
    qw, qz, sc, xg = _gpu(qweight, qzeros, scales, x)
    lib = _native.library()
    ws = torch.zeros(max(int(lib.lvb_awq_workspace_bytes(m, k, n, g)), 256), dtype=torch.uint8, device=DEV)
    y = torch.empty(m, n, dtype=torch.float16, device=DEV)
    _native.check(lib.lvb_awq_linear(xg.data_ptr(), qw.data_ptr(), qz.data_ptr(), sc.data_ptr(), None,
                                     y.data_ptr(), m, k, n, g, ws.data_ptr(), ws.numel(),
                                     torch.cuda.current_stream().cuda_stream), "lvb_awq_linear")
    torch.cuda.synchronize()
    max_abs, rel = oawq.error_metrics(y.float().cpu().numpy(), expected)
    assert max_abs <= MAX_ABS and rel <= REL_L2, (max_abs, rel)


@pytest.mark.parametrize("m,k,n,g", [(3, 896, 256, 896), (64, 3584, 512, 128), (8, 7168, 384, 128)])
def test_packed_decode_shapes(m, k, n, g):
    """Per-column groups (group = k), the largest packed batch, long k."""

    _check_against_oracle(m, k, n, g, seed=m * 31 + n)


@pytest.mark.parametrize("m,k,n", [(100, 512, 1024), (300, 640, 768), (2048, 1024, 1280)])
def test_packed_entry_prefill_sizes(m, k, n):
    """lvb_awq_linear_packed on 128- and 256-row tiles (several m tiles)."""

    from light_vllm_b200.awq import pack_awq_decode_layout

    g = 128
    qweight, qzeros, scales = oawq.random_checkpoint(k, n, g, seed=m + n)
    rng = np.random.default_rng(m)
    x = rng.standard_normal((m, k)).astype(np.float16)
    bias = rng.standard_normal(n).astype(np.float16)
    expected = oawq.linear_fp32(x, qweight, qzeros, scales, g, bias)
    qw, qz, sc, xg, bg = _gpu(qweight, qzeros, scales, x, bias)
    codes, groups = pack_awq_decode_layout(qw, qz, sc, g)
    lib = _native.library()
    ws = torch.zeros(max(int(lib.lvb_awq_workspace_bytes(m, k, n, g)), 256), dtype=torch.uint8, device=DEV)
    y = torch.empty(m, n, dtype=torch.float16, device=DEV)
    _native.check(lib.lvb_awq_linear_packed(xg.data_ptr(), codes.data_ptr(), groups.data_ptr(), bg.data_ptr(),
                                            y.data_ptr(), m, k, n, g, ws.data_ptr(), ws.numel(),
                                            torch.cuda.current_stream().cuda_stream), "lvb_awq_linear_packed")
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    max_abs, rel = oawq.error_metrics(y.float().cpu().numpy(), expected)
    assert max_abs <= MAX_ABS and rel <= REL_L2, (max_abs, rel)


def test_prepare_repacks_in_place_once():
    """prepare() replaces qweight's contents with the packed codes (no second
    resident copy); preparing the same storage again reuses that packing."""

    k, n, g = 512, 1024, 128
    qweight, qzeros, scales = oawq.random_checkpoint(k, n, g, seed=4)
    expected_codes, _ = oawq.pack_decode_layout(qweight, qzeros, scales, g)
    qw, qz, sc = _gpu(qweight, qzeros, scales)
    x = torch.randn(5, k, dtype=torch.float16, device=DEV)
    op1 = B200AWQScheme().prepare(qw, qz, sc, g, None)
    y1 = op1(x)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(qw.cpu().numpy().view(np.uint8).reshape(-1), expected_codes.reshape(-1))
    assert op1.codes.data_ptr() == qw.data_ptr()
    op2 = B200AWQScheme().prepare(qw, qz, sc, g, None)
    assert torch.equal(op2(x), y1)
    np.testing.assert_array_equal(qw.cpu().numpy().view(np.uint8).reshape(-1), expected_codes.reshape(-1))


def test_ragged_shapes_keep_the_checkpoint_layout():
    qweight, qzeros, scales = oawq.random_checkpoint(96, 256, 32, seed=2)
    qw, qz, sc = _gpu(qweight, qzeros, scales)
    op = B200AWQScheme().prepare(qw, qz, sc, 32, None)
    assert op.codes is None
    np.testing.assert_array_equal(qw.cpu().numpy(), qweight)


def _integer_path(m: int, k: int, n: int, g: int) -> bool:
    """Whether the packed scheme applies the zero point and scale exactly for
    this shape (the dispatch rules of lvb_awq_linear_packed): the one-row GEMV
    at m = 1.  The warp-MMA kernel (m = 2..16) and the fp16 packed kernel
    multiply the reference's fp16-rounded weight."""

    return n % 128 == 0 and k % 64 == 0 and m == 1 and g % 32 == 0


def _assert_fp16_output_close(actual: np.ndarray, expected: np.ndarray, what, x=None, weights=None) -> None:
    """North-star tolerance for fp16 outputs: relative L2 <= 1e-3 against the
    fp32 oracle and, per element, |error| <= 2e-2 + 2^-10 |expected| -- the
    absolute bound plus one fp16 ulp of the output, which rounding the output
    itself costs once outputs exceed 32.

    With ``x`` and ``weights`` = (qweight, qzeros, scales, group) and a shape
    that runs an integer-limb path, the kernel applies the zero point and the
    scale exactly: the per-element bound then holds against the
    unrounded-weight product, and against the reference's fp16-weight product
    up to the reference's own weight rounding, 2^-11 sum_k |x_k W_k| (half an
    fp16 ulp per weight)."""

    max_abs, rel = oawq.error_metrics(actual, expected)
    assert rel <= REL_L2, (what, "rel-L2", rel)
    got = actual.astype(np.float64)
    slack = 0.0
    if x is not None:
        qweight, qzeros, scales, g = weights
        k, n = qweight.shape[0], qweight.shape[1] * 8
        if _integer_path(int(np.asarray(x).reshape(-1, k).shape[0]), k, n, g):
            exact, abs_sum = oawq.linear_exact_weight(x, qweight, qzeros, scales, g, None)
            excess = np.abs(got - exact) - (MAX_ABS + np.abs(exact) * 2.0**-10)
            assert float(excess.max()) <= 0.0, (what, "vs exact weights", float(excess.max()))
            slack = abs_sum * 2.0**-11
    excess = np.abs(got - expected) - (MAX_ABS + np.abs(expected) * 2.0**-10 + slack)
    assert float(excess.max()) <= 0.0, (what, "vs reference", max_abs, float(np.max(excess)))


@pytest.mark.parametrize("m", [5, 16, 32])
def test_decode_batches_with_activation_outliers(m):
    """Decode batches with outliers 300x the typical value in the rows: m = 5
    and 16 run the warp-MMA kernel, m = 32 the fp16 packed kernel; the
    north-star tolerance holds."""

    k, n, g = 3584, 4736, 128  # 8.5 MB of packed weights: the int8 path
    qweight, qzeros, scales = oawq.random_checkpoint(k, n, g, seed=m + 77)
    rng = np.random.default_rng(m + 5)
    x = rng.standard_normal((m, k))
    outliers = rng.random((m, k)) < 0.01
    x[outliers] *= 300.0
    x = x.astype(np.float16)
    expected = oawq.linear_fp32(x, qweight, qzeros, scales, g, None)
    qw, qz, sc, xg = _gpu(qweight, qzeros, scales, x)
    op = B200AWQScheme().prepare(qw, qz, sc, g, None)
    y = op(xg)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    _assert_fp16_output_close(y.float().cpu().numpy(), expected, m, x, (qweight, qzeros, scales, g))


def _massive_outlier_case(m: int, k: int, n: int, g: int, seed: int):
    """Activations N(0, 0.2) with one channel per (token, group) at +-U[1e3,
    3e4] (the massive activations of real Qwen2 checkpoints), and codes where
    half of the output columns have q == z at every outlier channel (a zero
    weight there), so those columns' outputs stay O(1) and the absolute
    tolerance measures the precision kept for the small activations."""

    qweight, qzeros, scales = oawq.random_checkpoint(k, n, g, seed=seed)
    rng = np.random.default_rng(seed + 1)
    groups = k // g
    x = rng.standard_normal((m, k)) * 0.2
    channels = rng.integers(0, g, size=groups) + np.arange(groups) * g  # one channel per group, shared by tokens
    x[:, channels] = rng.uniform(1e3, 3e4, size=(m, groups)) * rng.choice((-1.0, 1.0), size=(m, groups))
    x = x.astype(np.float16)
    codes = oawq.unpack(qweight)
    zeros = oawq.unpack(qzeros)
    zero_cols = np.flatnonzero(rng.random(n) < 0.5)
    for gi, c in enumerate(channels):
        codes[c, zero_cols] = zeros[gi, zero_cols]
    return x, oawq.pack(codes), qzeros, scales, zero_cols


@pytest.mark.parametrize("m", [1, 4, 16])
def test_decode_paths_keep_precision_beside_massive_outliers(m):
    """m = 1 runs the dp4a GEMV, m = 4 and 16 the warp-MMA kernel (fp16 x
    unchanged, the reference's fp16 weight).  Columns whose outlier weights are zero: max-abs <= 2e-2
    and rel-L2 <= 1e-3 against the fp32 oracle, with no widened bound; all
    columns: the fp16-output tolerance."""

    k, n, g = 3584, 4736, 128
    x, qweight, qzeros, scales, zero_cols = _massive_outlier_case(m, k, n, g, seed=500 + m)
    expected = oawq.linear_fp32(x, qweight, qzeros, scales, g, None)
    qw, qz, sc, xg = _gpu(qweight, qzeros, scales, x)
    y = B200AWQScheme().prepare(qw, qz, sc, g, None)(xg)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    got = y.float().cpu().numpy()
    max_abs, rel = oawq.error_metrics(got[:, zero_cols], expected[:, zero_cols])
    assert max_abs <= MAX_ABS and rel <= REL_L2, (m, max_abs, rel)
    _assert_fp16_output_close(got, expected, m, x, (qweight, qzeros, scales, g))


@pytest.mark.parametrize("m", [1, 16])
def test_fused_silu_linear_keeps_precision_beside_massive_outliers(m):
    """The SiLU-mul fused into the down projection (GEMV at m = 1, int8 path
    at m = 16): gate/up rows whose product has one massive channel per group."""

    k, n, g = 4096, 4096, 128  # 8 MiB of packed weights
    act_target, qweight, qzeros, scales, zero_cols = _massive_outlier_case(m, k, n, g, seed=700 + m)
    # gate large and positive where the target is large (silu(g) ~ g), up = target / gate.
    big = np.abs(act_target.astype(np.float64)) > 100
    gate = np.where(big, 200.0, 1.0)
    up = np.where(big, act_target.astype(np.float64) / 200.0, act_target.astype(np.float64))
    gate_up = np.concatenate([gate, up], axis=1).astype(np.float16)
    gu = torch.from_numpy(gate_up).float()
    act = (torch.nn.functional.silu(gu[:, :k]) * gu[:, k:]).half().numpy()
    expected = oawq.linear_fp32(act, qweight, qzeros, scales, g, None)
    qw, qz, sc, gu_dev = _gpu(qweight, qzeros, scales, gate_up)
    y = B200AWQScheme().prepare(qw, qz, sc, g, None).silu_mul_linear(gu_dev)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    got = y.float().cpu().numpy()
    max_abs, rel = oawq.error_metrics(got[:, zero_cols], expected[:, zero_cols])
    assert max_abs <= MAX_ABS and rel <= REL_L2, (m, max_abs, rel)
    _assert_fp16_output_close(got, expected, m, act, (qweight, qzeros, scales, g))


@pytest.mark.parametrize("m", [1, 2, 3, 4])
@pytest.mark.parametrize("k,n,g", [(896, 4864, 128), (3584, 4608, 128), (18944, 384, 128), (512, 1024, 64),
                                   (1024, 256, 256), (896, 256, 896)])
def test_gemv_decode_batches(m, k, n, g):
    """m <= 4 runs the CUDA-core dp4a GEMV over the packed layout (one split
    or many, group sizes 64 / 128 / 256 / per column); with and without
    bias."""

    _check_against_oracle(m, k, n, g, seed=1000 * m + k + n, with_bias=(m % 2 == 1))


@pytest.mark.parametrize("m", [1, 4])
def test_gemv_with_activation_outliers(m):
    k, n, g = 3584, 512, 128
    qweight, qzeros, scales = oawq.random_checkpoint(k, n, g, seed=m + 91)
    rng = np.random.default_rng(m + 9)
    x = rng.standard_normal((m, k))
    x[rng.random((m, k)) < 0.01] *= 300.0
    x = x.astype(np.float16)
    expected = oawq.linear_fp32(x, qweight, qzeros, scales, g, None)
    qw, qz, sc, xg = _gpu(qweight, qzeros, scales, x)
    y = B200AWQScheme().prepare(qw, qz, sc, g, None)(xg)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    _assert_fp16_output_close(y.float().cpu().numpy(), expected, m, x, (qweight, qzeros, scales, g))


@pytest.mark.parametrize("m", [1, 3, 16, 32, 48])
def test_silu_mul_linear_matches_oracle(m):
    """down(silu(gate) * up): decode sizes fuse the SiLU-mul into the
    activation prologue (lvb_awq_silu_linear_packed), larger batches run
    lvb_silu_mul and the projection; both against the fp32 oracle on the
    fp16-rounded activation."""

    k, n, g = 4096, 4096, 128  # 8 MiB of packed weights: GEMV (m = 1), int8 path (m <= 16), fp16 packed above
    qweight, qzeros, scales = oawq.random_checkpoint(k, n, g, seed=m + 301)
    rng = np.random.default_rng(m + 17)
    gate_up = rng.standard_normal((m, 2 * k)).astype(np.float16)
    gu = torch.from_numpy(gate_up).float()
    act = (torch.nn.functional.silu(gu[:, :k]) * gu[:, k:]).half().numpy()
    expected = oawq.linear_fp32(act, qweight, qzeros, scales, g, None)
    qw, qz, sc, gu_dev = _gpu(qweight, qzeros, scales, gate_up)
    op = B200AWQScheme().prepare(qw, qz, sc, g, None)
    y = op.silu_mul_linear(gu_dev)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    _assert_fp16_output_close(y.float().cpu().numpy(), expected, m, act, (qweight, qzeros, scales, g))


@pytest.mark.parametrize("m", [9, 16])
def test_silu_mul_linear_on_a_wide_layer(m):
    """A down projection of 76 column tiles with 9..16 rows (10 MB of codes,
    groups of 128): lvb_silu_mul into the workspace, then the warp-MMA
    projection; against the fp32 oracle on the fp16-rounded activation."""

    k, n, g = 2048, 9728, 128
    qweight, qzeros, scales = oawq.random_checkpoint(k, n, g, seed=m + 401)
    rng = np.random.default_rng(m + 19)
    gate_up = rng.standard_normal((m, 2 * k)).astype(np.float16)
    gu = torch.from_numpy(gate_up).float()
    act = (torch.nn.functional.silu(gu[:, :k]) * gu[:, k:]).half().numpy()
    expected = oawq.linear_fp32(act, qweight, qzeros, scales, g, None)
    qw, qz, sc, gu_dev = _gpu(qweight, qzeros, scales, gate_up)
    y = B200AWQScheme().prepare(qw, qz, sc, g, None).silu_mul_linear(gu_dev)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    _assert_fp16_output_close(y.float().cpu().numpy(), expected, m, act, (qweight, qzeros, scales, g))


@pytest.mark.parametrize("m,k,n", [(40, 512, 18944), (64, 768, 18944), (100, 512, 18944), (128, 1024, 19200)])
def test_packed_two_ctas_per_sm_configs(m, k, n):
    """64- and 128-row token tiles with at least one output tile per SM run
    two CTAs per SM (half the tensor and shared memory each, the 128-row
    tile without the second accumulator)."""

    _check_against_oracle(m, k, n, 128, seed=m + k, with_bias=(m % 2 == 0))
