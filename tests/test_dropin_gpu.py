"""The plugins dropped into light-vllm's own model and step handler.

The reference's ``Qwen2ForCausalLM`` (modeling/models/qwen2.py:553-705) is
built with ``AWQLinearMethod(AWQConfig(group_size=128), B200AWQScheme())``
(modeling/quantization/awq.py:506-664: merged QKV and gate/up storage,
``scheme.prepare`` once per merged operation) and prepared for inference;
attention runs through ``B200PagedAttentionBackend().create(...)`` over the
reference's own ``PagedKVCache`` and ``PagedAttentionMetadata``.  Nothing of
this package's runner is involved.  The model decodes the greedy fixture
``tests/golden/qwen2_greedy.npz`` (a prefill of two prompts plus 64 steps,
recorded from the same model on the reference's Torch paths) and must
reproduce all 130 tokens:

* through ``ForwardBatch`` directly (modeling/models/interfaces.py), and
* through ``PagedStepHandler.forward`` (runtime/execution/worker.py:237-304),
  which packs the token-major batch, builds the metadata, calls
  ``backend.create`` and checks that every attention layer ran.

Skipped when light-vllm is not importable (``baseline/_ref`` or
``LIGHT_VLLM_SRC``).
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.paged_cache import reference_types

pytestmark = pytest.mark.gpu
REF = reference_types()
GOLDEN = Path(__file__).resolve().parent / "golden" / "qwen2_greedy.npz"

if REF.source != "light_vllm":
    pytest.skip("light-vllm is not importable (no baseline/_ref, no LIGHT_VLLM_SRC)", allow_module_level=True)


def _model(device):
    from light_vllm.modeling.models.qwen2 import Qwen2Config, Qwen2ForCausalLM
    from light_vllm.modeling.quantization.awq import AWQConfig, AWQLinearMethod
    from light_vllm.modeling.tensor_parallel import TensorParallelContext

    from light_vllm_b200 import B200AWQScheme

    class CountingScheme(B200AWQScheme):
        prepared = 0

        def prepare(self, *args):
            CountingScheme.prepared += 1
            return super().prepare(*args)

    d = np.load(GOLDEN)
    cfg = json.loads(bytes(d["config_json"]).decode())
    names = Qwen2Config.__dataclass_fields__ if hasattr(Qwen2Config, "__dataclass_fields__") else cfg
    qcfg = Qwen2Config(**{k: v for k, v in cfg.items() if k in names and k not in ("group_size", "block_size", "seed")})
    scheme = CountingScheme()
    model = Qwen2ForCausalLM(qcfg, TensorParallelContext(), AWQLinearMethod(AWQConfig(group_size=128), scheme),
                             device=device, dtype=torch.float16)
    with torch.no_grad():
        state = model.state_dict()
        for key in d.files:
            if key.startswith("w:"):
                state[key[2:]].copy_(torch.from_numpy(d[key]))
        model.prepare_for_inference()
    # one prepare per merged QKV, o, merged gate/up and down of each layer
    assert CountingScheme.prepared == 4 * qcfg.num_hidden_layers
    return model, d, cfg


def _check(tokens, d):
    np.testing.assert_array_equal(np.asarray(tokens), d["tokens"])


def test_reference_model_through_forward_batch():
    from light_vllm.modeling.models.interfaces import ForwardBatch

    from light_vllm_b200 import B200PagedAttentionBackend, _native

    device = torch.device("cuda", 0)
    model, d, cfg = _model(device)
    bs = cfg["block_size"]
    cache = REF.PagedKVCache(model.kv_cache_spec, REF.PagedKVCacheConfig(32, bs, dtype=torch.float16, device=device))
    backend = B200PagedAttentionBackend()
    tables = [tuple(int(b) for b in t) for t in d["tables"]]
    prompts = [d["prompt0"].tolist(), d["prompt1"].tolist()]

    def run(ids, positions, computed, lengths):
        starts = [0]
        for n in lengths:
            starts.append(starts[-1] + n)
        used = tuple(t[: -(-(c + n) // bs)] for t, c, n in zip(tables, computed, lengths))
        md = REF.PagedAttentionMetadata(block_tables=used, num_computed_tokens=tuple(computed),
                                        query_layouts=tuple(REF.linear_query_layout(n) for n in lengths))
        attention = backend.create(cache, md)
        batch = ForwardBatch(input_ids=torch.tensor(ids, dtype=torch.long, device=device),
                             positions=torch.tensor(positions, dtype=torch.long, device=device),
                             query_start_loc=tuple(starts), attention=attention,
                             logit_query_indices=tuple(s - 1 for s in starts[1:]))
        with torch.no_grad():
            logits = model(batch).logits
        assert attention.layer_ids == frozenset(layer.layer_id for layer in cache.model_spec.layers)
        return logits.argmax(-1).tolist()

    nxt = run([t for p in prompts for t in p], [i for p in prompts for i in range(len(p))], [0, 0],
              [len(p) for p in prompts])
    tokens = [nxt]
    ctx = [len(p) for p in prompts]
    for _ in range(len(d["tokens"]) - 1):
        nxt = run(nxt, ctx, ctx, [1, 1])
        tokens.append(nxt)
        ctx = [c + 1 for c in ctx]
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    _check(tokens, d)


def test_reference_step_handler_with_b200_backend():
    from light_vllm.runtime.execution.interfaces import ModelStepBatch, ModelStepRequest
    from light_vllm.runtime.execution.worker import PagedStepHandler

    from light_vllm_b200 import B200PagedAttentionBackend, _native

    device = torch.device("cuda", 0)
    model, d, cfg = _model(device)
    bs = cfg["block_size"]
    handler = PagedStepHandler(model, REF.PagedKVCacheConfig(32, bs, dtype=torch.float16, device=device),
                               B200PagedAttentionBackend())
    tables = [tuple(int(b) for b in t) for t in d["tables"]]
    prompts = [d["prompt0"].tolist(), d["prompt1"].tolist()]

    def step(queries, computed):
        requests = []
        for i, (q, c) in enumerate(zip(queries, computed)):
            n = len(q)
            requests.append(ModelStepRequest(
                request_id=f"r{i}", query_token_ids=tuple(q), num_computed_tokens=c, num_reserved_query_tokens=n,
                query_layout=REF.linear_query_layout(n), block_ids=tables[i][: -(-(c + n) // bs)],
                logit_query_indices=(n - 1,)))
        with torch.no_grad():
            out = handler.forward(model, ModelStepBatch(tuple(requests)))
        return [int(out.request_logits(i).argmax(-1).reshape(-1)[-1]) for i in range(len(requests))]

    nxt = step(prompts, [0, 0])
    tokens = [nxt]
    ctx = [len(p) for p in prompts]
    for _ in range(len(d["tokens"]) - 1):
        nxt = step([[t] for t in nxt], ctx)
        tokens.append(nxt)
        ctx = [c + 1 for c in ctx]
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    _check(tokens, d)
