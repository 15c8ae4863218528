"""Greedy tokens of the decode kernels that the 7B/72B numbers run, pinned to
the reference's own model.

tests/golden/qwen2_decode_pin.npz holds the greedy tokens that the
reference's ``Qwen2ForCausalLM`` (Torch AWQ scheme, ``TorchPagedAttention``,
fp16, CPU) produced for a random-init AWQ Qwen2 with hidden 2048,
intermediate 8192, 16 query / 2 KV heads, 2 layers and group 128: one
request alone and four requests together, each a prefill plus 64 decode
steps.  The weights are regenerated here from the fixture's seed
(``tests/golden/qwen2_weights.py``, checked against the fixture's digest).

Its MLP projections hold 16 and 8 MiB of int4 codes, so the runner's decode
steps take the paths of the large models: one request runs the one-row dp4a
GEMV for every projection (the down projection with the SiLU-mul fused into
it); four requests run the warp-MMA kernel for every projection (the down
projection after lvb_silu_mul), the routes of the 7B model at 2..16 rows.

The runner is fed the reference's tokens (teacher forcing) and must pick the
reference's token at every step whose reference top-2 logit margin is at
least 0.02 (five fp16 ulps of these logits), and one of the reference's top
two at the few steps below that, eagerly and from a replayed CUDA graph.
Because every input is the reference's, this is the same as identical free
running greedy sequences wherever no step is a near tie.
"""

from __future__ import annotations

import functools
import json
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "qwen2_decode_pin.npz"
MARGIN = 0.02


@functools.lru_cache(maxsize=1)
def _fixture():
    from tests.golden.qwen2_weights import checksum, random_awq_state

    d = np.load(GOLDEN)
    cfg = json.loads(bytes(d["config_json"]).decode())
    state = random_awq_state(cfg, cfg["seed"])
    assert checksum(state) == cfg["weights_sha256"], "weight generator differs from the fixture's"
    prompts = [d[f"prompt{i}"].tolist() for i in range(4)]
    runs = {name: (d[f"{name}_tokens"], d[f"{name}_margins"], d[f"{name}_second"]) for name in ("single", "batch")}
    return cfg, state, prompts, d["tables"], runs


def _decode(run: str, graph: bool) -> np.ndarray:
    from light_vllm_b200 import B200PagedAttentionBackend
    from oracle.paged_cache import model_spec, reference_types

    T = reference_types()
    PagedAttentionMetadata, PagedKVCache, PagedKVCacheConfig = T.PagedAttentionMetadata, T.PagedKVCache, T.PagedKVCacheConfig
    linear_query_layout = T.linear_query_layout
    from light_vllm_b200.qwen2 import Qwen2AWQRunner, Qwen2Shape, StaticDecodeAttention, shard_state_dict

    cfg, state, prompts, all_tables, runs = _fixture()
    ref_tokens = runs[run][0]
    members = (0,) if run == "single" else tuple(range(len(prompts)))
    ps = [prompts[i] for i in members]
    tables = [[int(b) for b in all_tables[i]] for i in members]
    shape = Qwen2Shape.from_mapping(cfg)
    device = torch.device("cuda", torch.cuda.current_device())
    runner = Qwen2AWQRunner(shape, shard_state_dict(state, shape, 0, 1), device, max_tokens=64)
    bs = cfg["block_size"]
    cache = PagedKVCache(model_spec(T, runner.kv_layers()),
                         PagedKVCacheConfig(int(all_tables.size), bs, dtype=torch.float16, device=device))
    backend = B200PagedAttentionBackend()

    def eager_step(ids, computed, lengths):
        used = tuple(tuple(t[: -(-(c + n) // bs)]) for t, c, n in zip(tables, computed, lengths))
        md = PagedAttentionMetadata(block_tables=used, num_computed_tokens=tuple(computed),
                                    query_layouts=tuple(linear_query_layout(n) for n in lengths))
        positions = [c + j for c, n in zip(computed, lengths) for j in range(n)]
        rows = np.cumsum(lengths) - 1
        return runner.forward(torch.tensor(ids, device=device),
                              torch.tensor(positions, dtype=torch.int32, device=device),
                              backend.create(cache, md), torch.tensor(rows, device=device))

    try:
        picks = [eager_step([t for p in ps for t in p], [0] * len(ps), [len(p) for p in ps]).tolist()]
        ctx = [len(p) for p in ps]
        steps = len(ref_tokens) - 1
        if not graph:
            for s in range(steps):
                picks.append(eager_step(ref_tokens[s].tolist(), ctx, [1] * len(ps)).tolist())
                ctx = [c + 1 for c in ctx]
        else:
            attention = StaticDecodeAttention(cache, tables, ctx, device)
            ids = torch.tensor(ref_tokens[0], dtype=torch.int64, device=device)
            step = runner.capture_decode(attention, ids)
            for s in range(steps):
                ids.copy_(torch.from_numpy(ref_tokens[s]))
                step.replay()
                picks.append(ids.tolist())
            del step
        return np.asarray(picks)
    finally:
        torch.cuda.synchronize()
        runner.close()


def _check(run: str, picks: np.ndarray) -> None:
    _, _, _, _, runs = _fixture()
    tokens, margins, second = runs[run]
    assert picks.shape == tokens.shape
    clear = margins >= MARGIN
    assert clear.mean() > 0.9  # the fixture is mostly clear-cut steps
    mismatch = np.argwhere(clear & (picks != tokens))
    assert mismatch.size == 0, f"{run}: differs from the reference at (step, request) {mismatch[:8].tolist()}"
    close = ~clear
    assert np.all((picks[close] == tokens[close]) | (picks[close] == second[close])), run


@pytest.mark.parametrize("graph", [False, True], ids=["eager", "graph"])
@pytest.mark.parametrize("run", ["single", "batch"])
def test_decode_paths_match_reference_greedy(run, graph):
    from light_vllm_b200 import _native

    picks = _decode(run, graph)
    assert _native.device_error() == 0
    _check(run, picks)
