"""Pin the CPU oracle to golden vectors produced by the reference itself.

The fixtures in tests/golden/ were written by tests/golden/make_golden.py,
which ran light-vllm's own Torch AWQ scheme, PagedAttentionMetadata and
TorchPagedAttention on seeded inputs.  Known-answer constants come from the
reference's tests (tests/test_awq.py:149-163, tests/test_paged_attention.py:121-175).
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import awq as oawq
from oracle import paged_attention as opa

GOLDEN = Path(__file__).resolve().parent / "golden"
AWQ = np.load(GOLDEN / "awq_golden.npz")
META = json.loads((GOLDEN / "paged_meta.json").read_text())
ATTN = np.load(GOLDEN / "paged_attn.npz")
ATTN_INDEX = json.loads(bytes(ATTN["index_json"]).decode())
AWQ_CASES = [("q16x24g8", 8), ("q64x256g32", 32), ("q128x384g128", 128)]


def test_pack_known_answer():
    packed = oawq.pack(AWQ["pack_small_values"])
    assert packed[0, 0] == 0x75316420
    np.testing.assert_array_equal(packed, AWQ["pack_small_packed"])
    np.testing.assert_array_equal(oawq.unpack(packed), AWQ["pack_small_values"])


def test_pack_unpack_random_match_reference():
    np.testing.assert_array_equal(oawq.pack(AWQ["pack_rand_values"]), AWQ["pack_rand_packed"])
    np.testing.assert_array_equal(oawq.unpack(AWQ["pack_rand_packed"]), AWQ["pack_rand_values"])


def test_pack_rejects_out_of_range():
    with pytest.raises(ValueError):
        oawq.pack(np.full((1, 8), 16))
    with pytest.raises(ValueError):
        oawq.pack(np.zeros((1, 7), dtype=np.int32))


@pytest.mark.parametrize("name,group", AWQ_CASES)
def test_quantize_matches_reference(name, group):
    weight = torch.from_numpy(AWQ[f"{name}_weight"])
    qweight, qzeros, scales, deq = oawq.quantize_weight(weight, group)
    np.testing.assert_array_equal(qweight, AWQ[f"{name}_qweight"])
    np.testing.assert_array_equal(qzeros, AWQ[f"{name}_qzeros"])
    np.testing.assert_array_equal(scales.view(np.uint16), AWQ[f"{name}_scales"].view(np.uint16))
    np.testing.assert_array_equal(deq.view(np.uint16), AWQ[f"{name}_dequant"].view(np.uint16))


@pytest.mark.parametrize("name,group", AWQ_CASES)
def test_dequantize_is_bit_exact(name, group):
    w = oawq.dequantize(AWQ[f"{name}_qweight"], AWQ[f"{name}_qzeros"], AWQ[f"{name}_scales"], group)
    np.testing.assert_array_equal(w.T.view(np.uint16), AWQ[f"{name}_dequant"].view(np.uint16))


@pytest.mark.parametrize("name,group", AWQ_CASES)
def test_torch_linear_matches_reference_scheme(name, group):
    args = [torch.from_numpy(AWQ[f"{name}_{k}"]) for k in ("qweight", "qzeros", "scales")]
    x = torch.from_numpy(AWQ[f"{name}_x"])
    bias = torch.from_numpy(AWQ[f"{name}_bias"])
    y = oawq.torch_linear(x, *args, group, bias)
    np.testing.assert_array_equal(y.numpy().view(np.uint16), AWQ[f"{name}_y"].view(np.uint16))
    yf = oawq.torch_linear(x.float(), *args, group, None)
    np.testing.assert_allclose(yf.numpy(), AWQ[f"{name}_y_fp32"], rtol=0, atol=0)


@pytest.mark.parametrize("name,group", AWQ_CASES)
def test_fp64_linear_is_close_to_reference(name, group):
    y = oawq.linear_fp32(AWQ[f"{name}_x"], AWQ[f"{name}_qweight"], AWQ[f"{name}_qzeros"],
                         AWQ[f"{name}_scales"], group, AWQ[f"{name}_bias"])
    max_abs, rel = oawq.error_metrics(AWQ[f"{name}_y"], y)
    # The reference rounds x @ W to fp16 and then adds the bias in fp16: at most
    # ~1.5 fp16 ulps of the largest output away from the exact value.
    assert max_abs <= 1.5 * np.abs(y).max() * 2.0**-10 and rel < 1e-3


@pytest.mark.parametrize("case", META, ids=[c["name"] for c in META])
def test_metadata_matches_reference(case):
    lengths = [len(p) for p in case["layouts"]]
    reserved = case.get("reserved") or lengths
    readonly = case.get("readonly") or [0] * len(lengths)
    assert list(opa.query_start_loc(lengths)) == case["query_start_loc"]
    assert list(opa.request_indices(lengths)) == case["request_indices"]
    vis, starts = opa.visibility_tensor(case["layouts"])
    assert list(vis) == case["visibility"]
    assert list(starts) == case["visibility_start"]
    try:
        slots = list(opa.slot_mapping(case["tables"], case["computed"], lengths, reserved,
                                      case["block_size"]))
        error = None
    except opa.KVCacheError as exc:
        slots, error = None, str(exc)
    assert slots == case["slot_mapping"]
    assert error == case["slot_error"]
    try:
        opa.validate_block_tables(case["tables"], case["computed"], reserved, readonly,
                                  num_blocks=case["num_blocks"], block_size=case["block_size"])
        error = None
    except opa.KVCacheError as exc:
        error = str(exc)
    assert error == case["validate_error"]


def _load(name: str, key: str, dtype: str) -> torch.Tensor:
    arr = ATTN[f"{name}_{key}"]
    if dtype == "bfloat16":
        return torch.from_numpy(arr.view(np.int16)).view(torch.bfloat16)
    return torch.from_numpy(arr)


@pytest.mark.parametrize("case", ATTN_INDEX, ids=[c["name"] for c in ATTN_INDEX])
def test_attention_matches_reference(case):
    dt = case["dtype"]
    kc = _load(case["name"], "k_before", dt).clone()
    vc = _load(case["name"], "v_before", dt).clone()
    q, k, v = (_load(case["name"], key, dt) for key in ("q", "k", "v"))
    out = opa.attend(q, k, v, kc, vc, case["tables"], case["computed"], case["layouts"],
                     scale=case["scale"], reserved=case.get("reserved"))
    assert torch.equal(kc, _load(case["name"], "k_after", dt))
    assert torch.equal(vc, _load(case["name"], "v_after", dt))
    expected = _load(case["name"], "o", dt)
    assert torch.equal(out, expected)


FUSED = np.load(GOLDEN / "fused_norm.npz")
FUSED_CASES = ["w2_t5_h64", "w4_t3_h3584", "w8_t2_h896"]


@pytest.mark.parametrize("name", FUSED_CASES)
def test_fused_add_rms_norm_matches_reference(name):
    """Rank sum + ``fused_add_rms_norm`` (_qwen2_kernels.py:145-180)."""

    from oracle import tensor_parallel as otp

    partials = torch.from_numpy(FUSED[f"{name}_partials"])
    residual = torch.from_numpy(FUSED[f"{name}_residual"])
    weight = torch.from_numpy(FUSED[f"{name}_weight"])
    eps = float(FUSED[f"{name}_eps"])
    normed, new_residual = otp.all_reduce_add_rms_norm(list(partials), residual, weight, eps)
    want_res = torch.from_numpy(FUSED[f"{name}_new_residual"])
    want_norm = torch.from_numpy(FUSED[f"{name}_normed"])
    # The residual is the fp16 rounding of an exact fp32 sum of two fp16 values.
    assert torch.equal(new_residual, want_res.half())
    assert torch.equal(normed, want_norm.half())


def test_qwen2_oracle_greedy_matches_reference():
    """The oracle decoder reproduces the reference model's greedy tokens:
    a two-request prefill, then 64 decode steps (tests/golden/qwen2_greedy.npz,
    written by the reference's Qwen2ForCausalLM with the Torch AWQ scheme)."""

    from oracle.qwen2 import Qwen2Oracle

    d = np.load(GOLDEN / "qwen2_greedy.npz")
    cfg = json.loads(bytes(d["config_json"]).decode())
    model = Qwen2Oracle({k[2:]: d[k] for k in d.files if k.startswith("w:")}, cfg)
    prompts = [d["prompt0"].tolist(), d["prompt1"].tolist()]
    nxt, _ = model.step([(p, 0) for p in prompts])
    tokens = [nxt]
    ctx = [len(p) for p in prompts]
    for _ in range(len(d["tokens"]) - 1):
        nxt, _ = model.step([([t], c) for t, c in zip(nxt, ctx)])
        ctx = [c + 1 for c in ctx]
        tokens.append(nxt)
    assert np.array_equal(np.asarray(tokens), d["tokens"])
