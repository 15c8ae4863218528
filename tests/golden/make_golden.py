"""Generate golden vectors for the hot path by running the reference itself.

Run in a container that has the light-vllm source tree (read-only is fine):

    LIGHT_VLLM_SRC=/path/to/light-vllm/src python tests/golden/make_golden.py

It imports the reference's own correctness implementations (the Torch AWQ
scheme, ``PagedAttentionMetadata`` and ``TorchPagedAttention``), runs them on
seeded inputs and writes the inputs and outputs as small fixtures next to this
script.  The fixtures are committed; the GPU box never needs the reference.

Fixtures:
  awq_golden.npz     pack/unpack vectors, quantize_awq_weight outputs and
                     Torch-scheme linear outputs.
  paged_meta.json    slot mappings, request indices, tree visibility and
                     block-table validation outcomes for metadata cases.
  paged_attn.npz     TorchPagedAttention outputs and post-write cache contents.
  fused_norm.npz     fused_add_rms_norm outputs after a rank sum of fp16
                     partials (the row-parallel epilogue of a Qwen2 block).
  qwen2_greedy.npz   a random-init AWQ Qwen2ForCausalLM (Torch AWQ scheme,
                     TorchPagedAttention, fp16, CPU): its weights, two prompts,
                     the greedy tokens of a prefill plus 64 decode steps and
                     the top-2 logit margin of every step.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _import_reference():
    src = os.environ.get("LIGHT_VLLM_SRC")
    if not src or not Path(src).is_dir():
        raise SystemExit("set LIGHT_VLLM_SRC to the light-vllm 'src' directory")
    sys.path.insert(0, src)
    from light_vllm.modeling.attention import AttentionLayerSpec, ModelKVCacheSpec
    from light_vllm.modeling.quantization import awq
    from light_vllm.runtime.execution.interfaces import QueryLayout
    from light_vllm.runtime.execution.paged_attention import (
        PagedAttentionMetadata,
        TorchPagedAttention,
    )
    from light_vllm.runtime.execution.paged_cache import PagedKVCache, PagedKVCacheConfig
    from light_vllm.modeling.models._qwen2_kernels import fused_add_rms_norm
    from light_vllm.modeling.models.interfaces import ForwardBatch
    from light_vllm.modeling.models.qwen2 import Qwen2Config, Qwen2ForCausalLM
    from light_vllm.modeling.quantization.awq import AWQConfig, AWQLinearMethod
    from light_vllm.modeling.quantization.awq_schemes import TorchAWQScheme
    from light_vllm.modeling.tensor_parallel import TensorParallelContext

    return dict(
        AttentionLayerSpec=AttentionLayerSpec,
        ModelKVCacheSpec=ModelKVCacheSpec,
        awq=awq,
        QueryLayout=QueryLayout,
        PagedAttentionMetadata=PagedAttentionMetadata,
        TorchPagedAttention=TorchPagedAttention,
        PagedKVCache=PagedKVCache,
        PagedKVCacheConfig=PagedKVCacheConfig,
        fused_add_rms_norm=fused_add_rms_norm,
        ForwardBatch=ForwardBatch,
        Qwen2Config=Qwen2Config,
        Qwen2ForCausalLM=Qwen2ForCausalLM,
        AWQConfig=AWQConfig,
        AWQLinearMethod=AWQLinearMethod,
        TorchAWQScheme=TorchAWQScheme,
        TensorParallelContext=TensorParallelContext,
    )


def _as_storable(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def make_awq(ref) -> None:
    awq = ref["awq"]
    out: dict[str, np.ndarray] = {}
    # Known answer from the reference's own test (tests/test_awq.py:149-163).
    values = torch.tensor([[0, 1, 2, 3, 4, 5, 6, 7], [15, 14, 13, 12, 11, 10, 9, 8]],
                          dtype=torch.int32)
    out["pack_small_values"] = values.numpy()
    out["pack_small_packed"] = awq.pack_awq(values).numpy()
    gen = torch.Generator().manual_seed(11)
    values = torch.randint(0, 16, (6, 32), generator=gen, dtype=torch.int32)
    out["pack_rand_values"] = values.numpy()
    out["pack_rand_packed"] = awq.pack_awq(values).numpy()

    cases = [
        ("q16x24g8", (16, 24), 8, 3),
        ("q64x256g32", (64, 256), 32, 5),
        ("q128x384g128", (128, 384), 128, 9),
    ]
    for name, shape, group, seed in cases:
        torch.manual_seed(seed)
        weight = torch.randn(*shape, dtype=torch.float16)
        quant = awq.quantize_awq_weight(weight, group_size=group)
        out[f"{name}_weight"] = weight.numpy()
        out[f"{name}_qweight"] = quant.qweight.numpy()
        out[f"{name}_qzeros"] = quant.qzeros.numpy()
        out[f"{name}_scales"] = quant.scales.numpy()
        out[f"{name}_dequant"] = quant.dequantized.numpy()
        x = torch.randn(5, shape[1], dtype=torch.float16)
        bias = torch.randn(shape[0], dtype=torch.float16)
        y = awq._torch_awq_linear(x, quant.qweight, quant.qzeros, quant.scales, group, bias)
        out[f"{name}_x"] = x.numpy()
        out[f"{name}_bias"] = bias.numpy()
        out[f"{name}_y"] = y.numpy()
        xf = x.float()
        yf = awq._torch_awq_linear(xf, quant.qweight, quant.qzeros, quant.scales, group, None)
        out[f"{name}_y_fp32"] = yf.numpy()
    np.savez_compressed(HERE / "awq_golden.npz", **out)


def _meta_cases(ref):
    QL = ref["QueryLayout"]

    def linear(n):
        return tuple(-1 if i == 0 else i - 1 for i in range(n))

    return [
        # tests/test_paged_attention.py:121-130 known answer [4, 5, 0, 3, 6]
        dict(name="slots_noncontiguous", tables=((2, 0), (1, 3)), computed=(0, 1),
             layouts=(linear(3), linear(2)), num_blocks=4, block_size=2),
        # tests/test_paged_attention.py:149-175 visibility known answer
        dict(name="tree_visibility", tables=((0, 1), (2,)), computed=(0, 0),
             layouts=((-1, 0, 0), linear(2)), num_blocks=3, block_size=2),
        dict(name="lookahead", tables=((0, 1, 2),), computed=(0,), layouts=(linear(1),),
             reserved=(3,), num_blocks=3, block_size=1),
        dict(name="readonly_shared", tables=((0, 1), (0, 2)), computed=(2, 2),
             layouts=(linear(1), linear(1)), readonly=(1, 1), num_blocks=4, block_size=2),
        dict(name="err_not_covered", tables=((0,),), computed=(1,), layouts=(linear(2),),
             num_blocks=4, block_size=2),
        dict(name="err_out_of_range", tables=((4, 0),), computed=(2,), layouts=(linear(1),),
             num_blocks=4, block_size=2),
        dict(name="err_alias_within", tables=((0, 0),), computed=(2,), layouts=(linear(1),),
             num_blocks=4, block_size=2),
        dict(name="err_alias_across", tables=((0,), (0,)), computed=(0, 1),
             layouts=(linear(1), linear(1)), num_blocks=4, block_size=2),
        dict(name="err_one_sided_prefix", tables=((0, 1), (0, 2)), computed=(2, 2),
             layouts=(linear(1), linear(1)), readonly=(1, 0), num_blocks=5, block_size=2),
        dict(name="err_misaligned_prefix", tables=((0, 1, 2), (3, 0, 4)), computed=(4, 4),
             layouts=(linear(1), linear(1)), readonly=(1, 2), num_blocks=5, block_size=2),
        dict(name="err_readonly_beyond", tables=((0,),), computed=(1,), layouts=(linear(1),),
             readonly=(1,), num_blocks=2, block_size=2),
        dict(name="err_unused_trailing_a", tables=((0, 0),), computed=(0,), layouts=(linear(1),),
             num_blocks=4, block_size=2),
        dict(name="err_unused_trailing_b", tables=((0,), (1, 0)), computed=(0, 0),
             layouts=(linear(1), linear(1)), num_blocks=4, block_size=2),
        dict(name="tree_chain", tables=((1, 3, 0, 2),), computed=(2,),
             layouts=((-1, 0, 0, 2, 3),), readonly=(1,), num_blocks=4, block_size=2),
    ], QL


def make_meta(ref) -> None:
    PagedAttentionMetadata = ref["PagedAttentionMetadata"]
    cases, QL = _meta_cases(ref)
    results = []
    for case in cases:
        md = PagedAttentionMetadata(
            block_tables=case["tables"],
            num_computed_tokens=case["computed"],
            query_layouts=tuple(QL(p) for p in case["layouts"]),
            num_reserved_query_tokens=case.get("reserved", ()),
            num_readonly_prefix_blocks=case.get("readonly", ()),
        )
        record = {k: v for k, v in case.items()}
        record["query_start_loc"] = list(md.query_start_loc)
        record["request_indices"] = list(md.request_indices)
        vis, starts = md.visibility_tensor(device=torch.device("cpu"))
        record["visibility"] = [bool(v) for v in vis.tolist()]
        record["visibility_start"] = starts.tolist()
        record["has_only_linear_queries"] = md.has_only_linear_queries
        try:
            md.validate_block_tables(num_blocks=case["num_blocks"], block_size=case["block_size"])
            record["validate_error"] = None
        except Exception as exc:  # the reference raises KVCacheError
            record["validate_error"] = str(exc)
        try:
            record["slot_mapping"] = md.slot_mapping(
                block_size=case["block_size"], device=torch.device("cpu")).tolist()
            record["slot_error"] = None
        except Exception as exc:
            record["slot_mapping"] = None
            record["slot_error"] = str(exc)
        results.append(record)
    (HERE / "paged_meta.json").write_text(json.dumps(results, indent=1) + "\n")


def make_attention(ref) -> None:
    AttentionLayerSpec = ref["AttentionLayerSpec"]
    ModelKVCacheSpec = ref["ModelKVCacheSpec"]
    PagedKVCache = ref["PagedKVCache"]
    PagedKVCacheConfig = ref["PagedKVCacheConfig"]
    PagedAttentionMetadata = ref["PagedAttentionMetadata"]
    TorchPagedAttention = ref["TorchPagedAttention"]
    QL = ref["QueryLayout"]

    def linear(n):
        return tuple(-1 if i == 0 else i - 1 for i in range(n))

    cases = [
        dict(name="gqa_prefill_f32", dtype=torch.float32, hq=4, hkv=2, d=8, bs=4, nb=16,
             tables=((7, 1), (4,)), computed=(0, 0), layouts=(linear(6), linear(3))),
        dict(name="tree_f16", dtype=torch.float16, hq=4, hkv=2, d=16, bs=2, nb=16,
             tables=((7, 1), (4, 6)), computed=(0, 0), layouts=((-1, 0, 0, 2), (-1, 0, 0))),
        dict(name="history_bf16", dtype=torch.bfloat16, hq=28, hkv=4, d=32, bs=16, nb=12,
             tables=(tuple(range(9)),), computed=(130,), layouts=(linear(1),), prefix=130),
        dict(name="lookahead_f16", dtype=torch.float16, hq=4, hkv=2, d=16, bs=2, nb=16,
             tables=((8, 3, 12), (10, 14)), computed=(0, 0), layouts=(linear(3), linear(1)),
             reserved=(5, 4)),
        dict(name="readonly_prefix_f16", dtype=torch.float16, hq=4, hkv=2, d=16, bs=2, nb=16,
             tables=((0, 5), (0, 7)), computed=(2, 2), layouts=(linear(1), linear(1)),
             readonly=(1, 1), prefix=2),
        dict(name="mixed_decode_prefill_f32", dtype=torch.float32, hq=6, hkv=2, d=8, bs=4, nb=20,
             tables=((3, 9, 1), (5,), (11, 2, 0, 17)), computed=(9, 0, 13),
             layouts=(linear(1), linear(3), linear(2))),
    ]
    out: dict[str, np.ndarray] = {}
    index = []
    for ci, case in enumerate(cases):
        torch.manual_seed(1000 + ci)
        spec = ModelKVCacheSpec((AttentionLayerSpec("attention", case["hq"], case["hkv"], case["d"]),))
        cache = PagedKVCache(spec, PagedKVCacheConfig(case["nb"], case["bs"], dtype=case["dtype"]))
        layer = cache.layer("attention")
        layer.keys.copy_(torch.randn(layer.keys.shape).to(case["dtype"]))
        layer.values.copy_(torch.randn(layer.values.shape).to(case["dtype"]))
        before_k = layer.keys.clone()
        before_v = layer.values.clone()
        md = PagedAttentionMetadata(
            block_tables=case["tables"],
            num_computed_tokens=case["computed"],
            query_layouts=tuple(QL(p) for p in case["layouts"]),
            num_reserved_query_tokens=case.get("reserved", ()),
            num_readonly_prefix_blocks=case.get("readonly", ()),
        )
        t = md.num_query_tokens
        q = torch.randn(t, case["hq"], case["d"]).to(case["dtype"])
        k = torch.randn(t, case["hkv"], case["d"]).to(case["dtype"])
        v = torch.randn(t, case["hkv"], case["d"]).to(case["dtype"])
        scale = 1.0 / case["d"] ** 0.5
        o = TorchPagedAttention(cache, md).forward("attention", q, k, v, scale=scale)
        name = case["name"]
        for key, tensor in (("q", q), ("k", k), ("v", v), ("o", o), ("k_before", before_k),
                            ("v_before", before_v), ("k_after", layer.keys),
                            ("v_after", layer.values)):
            out[f"{name}_{key}"] = _as_storable(tensor)
        meta = {kk: vv for kk, vv in case.items() if kk != "dtype"}
        meta["dtype"] = str(case["dtype"]).replace("torch.", "")
        meta["scale"] = scale
        index.append(meta)
    out["index_json"] = np.frombuffer(json.dumps(index).encode(), dtype=np.uint8)
    np.savez_compressed(HERE / "paged_attn.npz", **out)


def make_fused_norm(ref) -> None:
    """Rank sums of fp16 partials, then the reference's ``fused_add_rms_norm``.

    The all-reduced tensor is the fp16 rounding of the fp32 rank sum.  The
    reference function runs on fp32 copies of the fp16 inputs: on CPU that is
    its ``hidden + residual`` / ``F.rms_norm`` path in fp32, the arithmetic its
    Triton kernel performs on GPUs before storing fp16.
    """

    out: dict[str, np.ndarray] = {}
    cases = [("w2_t5_h64", 2, 5, 64, 1e-6), ("w4_t3_h3584", 4, 3, 3584, 1e-6),
             ("w8_t2_h896", 8, 2, 896, 1e-5)]
    for ci, (name, world, tokens, hidden, eps) in enumerate(cases):
        g = torch.Generator().manual_seed(3000 + ci)
        partials = (torch.randn(world, tokens, hidden, generator=g) * 4).half()
        residual = (torch.randn(tokens, hidden, generator=g) * 8).half()
        weight = (torch.rand(hidden, generator=g) * 2).half()
        reduced = partials.float().sum(0).half()
        normed, new_residual = ref["fused_add_rms_norm"](reduced.float(), residual.float(), weight.float(), eps)
        for key, tensor in (("partials", partials), ("residual", residual), ("weight", weight),
                            ("normed", normed), ("new_residual", new_residual)):
            out[f"{name}_{key}"] = _as_storable(tensor)
        out[f"{name}_eps"] = np.array(eps, dtype=np.float64)
    np.savez_compressed(HERE / "fused_norm.npz", **out)


QWEN2_TINY = dict(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                  num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=256,
                  rms_norm_eps=1e-6, rope_theta=1e6)
QWEN2_PROMPTS = (7, 12)
QWEN2_STEPS = 64
QWEN2_BLOCK = 16


QWEN2_SEED = 16


def make_qwen2(ref, seed: int = QWEN2_SEED, write: bool = True) -> float:
    """Greedy decoding of a seeded random-init AWQ Qwen2 through the reference.

    The seed is one whose every step has a top-2 logit margin far above fp16
    rounding noise, so greedy identity is decided by the arithmetic, not by
    ties.  Returns that smallest margin.
    """

    awq = ref["awq"]
    cfg = ref["Qwen2Config"](**QWEN2_TINY)
    method = ref["AWQLinearMethod"](ref["AWQConfig"](group_size=128), ref["TorchAWQScheme"]())
    model = ref["Qwen2ForCausalLM"](cfg, ref["TensorParallelContext"](), method, device="cpu",
                                    dtype=torch.float16)
    g = torch.Generator().manual_seed(seed)
    out: dict[str, np.ndarray] = {}
    with torch.no_grad():
        for name, module in model.named_modules():
            if hasattr(module, "qweight") and hasattr(module, "qzeros"):
                k, n8 = module.qweight.shape
                groups = module.qzeros.shape[0]
                q = torch.randint(0, 16, (k, n8 * 8), generator=g, dtype=torch.int32)
                z = torch.randint(0, 16, (groups, n8 * 8), generator=g, dtype=torch.int32)
                module.qweight.copy_(awq.pack_awq(q))
                module.qzeros.copy_(awq.pack_awq(z))
                module.scales.copy_((torch.rand(groups, n8 * 8, generator=g) * 0.018 + 0.002).half())
                if module.bias is not None:
                    module.bias.copy_((torch.randn(module.bias.shape, generator=g) * 0.1).half())
            elif name.endswith("layernorm") or name.endswith(".norm"):
                module.weight.copy_((torch.rand(module.weight.shape, generator=g) + 0.5).half())
        model.model.embed_tokens.weight.copy_((torch.randn(model.model.embed_tokens.weight.shape,
                                                           generator=g) * 0.5).half())
        model.lm_head.weight.copy_((torch.randn(model.lm_head.weight.shape, generator=g) * 0.05).half())
        for key, tensor in model.state_dict().items():
            out[f"w:{key}"] = _as_storable(tensor)
        model.prepare_for_inference()

        spec = model.kv_cache_spec
        cache = ref["PagedKVCache"](spec, ref["PagedKVCacheConfig"](32, QWEN2_BLOCK, dtype=torch.float16))
        prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g) for n in QWEN2_PROMPTS]
        per_seq = -(-(max(QWEN2_PROMPTS) + QWEN2_STEPS) // QWEN2_BLOCK)
        tables = tuple(tuple(range(i * per_seq, (i + 1) * per_seq)) for i in range(len(prompts)))
        QL = ref["QueryLayout"]

        def linear(n):
            return QL(tuple(-1 if i == 0 else i - 1 for i in range(n)))

        def run(ids, positions, computed, lengths):
            starts = [0]
            for n in lengths:
                starts.append(starts[-1] + n)
            # A table covers exactly the blocks its tokens use.
            used = tuple(t[: -(-(c + n) // QWEN2_BLOCK)] for t, c, n in zip(tables, computed, lengths))
            md = ref["PagedAttentionMetadata"](block_tables=used, num_computed_tokens=tuple(computed),
                                               query_layouts=tuple(linear(n) for n in lengths))
            batch = ref["ForwardBatch"](input_ids=torch.tensor(ids, dtype=torch.long),
                                        positions=torch.tensor(positions, dtype=torch.long),
                                        query_start_loc=tuple(starts),
                                        attention=ref["TorchPagedAttention"](cache, md),
                                        logit_query_indices=tuple(s - 1 for s in starts[1:]))
            logits = model(batch).logits.float()
            top2 = logits.topk(2, dim=-1).values
            return logits.argmax(-1).tolist(), (top2[:, 0] - top2[:, 1]).tolist()

        ids = [t for p in prompts for t in p.tolist()]
        positions = [i for p in prompts for i in range(len(p))]
        tokens, margins = [], []
        nxt, marg = run(ids, positions, [0] * len(prompts), [len(p) for p in prompts])
        tokens.append(nxt)
        margins.append(marg)
        ctx = [len(p) for p in prompts]
        for _ in range(QWEN2_STEPS):
            nxt, marg = run(nxt, ctx, ctx, [1] * len(prompts))
            tokens.append(nxt)
            margins.append(marg)
            ctx = [c + 1 for c in ctx]
    for i, p in enumerate(prompts):
        out[f"prompt{i}"] = p.numpy().astype(np.int64)
    out["tables"] = np.asarray(tables, dtype=np.int32)
    out["tokens"] = np.asarray(tokens, dtype=np.int64)      # [1 + steps, requests]
    out["margins"] = np.asarray(margins, dtype=np.float32)
    out["config_json"] = np.frombuffer(json.dumps(dict(QWEN2_TINY, group_size=128, block_size=QWEN2_BLOCK,
                                                       seed=seed)).encode(), dtype=np.uint8)
    if write:
        np.savez_compressed(HERE / "qwen2_greedy.npz", **out)
    return float(np.min(out["margins"]))


QWEN2_PIN = dict(vocab_size=512, hidden_size=2048, intermediate_size=8192, num_hidden_layers=2,
                 num_attention_heads=16, num_key_value_heads=2, max_position_embeddings=512,
                 rms_norm_eps=1e-6, rope_theta=1e6)
QWEN2_PIN_PROMPTS = (6, 11, 17, 23)
QWEN2_PIN_STEPS = 64
QWEN2_PIN_MARGIN = 0.02
QWEN2_PIN_SEED = 1


def make_qwen2_pin(ref, seed: int = QWEN2_PIN_SEED, threshold: float = float("-inf"),
                   write: bool = True) -> float | None:
    """Greedy tokens of a random-init AWQ Qwen2 whose MLP projections are
    large enough (>= 8 MiB of int4 codes) for the B200 decode paths that the
    7B/72B numbers run: one request alone (one-row decode) and four requests
    together (small-batch decode), each a prefill plus 64 decode steps,
    through the reference's own ``Qwen2ForCausalLM`` with the Torch AWQ scheme
    and ``TorchPagedAttention`` (fp16, CPU).

    Only the seed, prompts, tables, tokens, runner-up tokens and top-2 logit
    margins are stored; the weights come from
    ``qwen2_weights.random_awq_state``.  A model this size has steps whose
    top-2 margin is one fp16 ulp of the logits, so the GPU test feeds the
    reference's tokens back (teacher forcing) and requires its greedy pick to
    equal the reference's at every step whose margin is at least
    ``QWEN2_PIN_MARGIN`` and to be one of the reference's top two at the
    others.  Returns the smallest margin (None if ``threshold`` is given and a
    step falls below it).
    """

    sys.path.insert(0, str(HERE.parent.parent))
    from tests.golden.qwen2_weights import checksum, random_awq_state

    cfg = ref["Qwen2Config"](**QWEN2_PIN)
    method = ref["AWQLinearMethod"](ref["AWQConfig"](group_size=128), ref["TorchAWQScheme"]())
    model = ref["Qwen2ForCausalLM"](cfg, ref["TensorParallelContext"](), method, device="cpu",
                                    dtype=torch.float16)
    state = random_awq_state(QWEN2_PIN, seed)
    out: dict[str, np.ndarray] = {}
    with torch.no_grad():
        sd = model.state_dict()
        if set(sd) != set(state):
            raise SystemExit(f"state dict keys differ: {sorted(set(sd) ^ set(state))[:8]}")
        for key, tensor in state.items():
            sd[key].copy_(tensor)
        model.prepare_for_inference()
        g = torch.Generator().manual_seed(seed + 7919)
        prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in QWEN2_PIN_PROMPTS]
        per_seq = -(-(max(QWEN2_PIN_PROMPTS) + QWEN2_PIN_STEPS) // QWEN2_BLOCK)
        tables = tuple(tuple(range(i * per_seq, (i + 1) * per_seq)) for i in range(len(prompts)))
        QL = ref["QueryLayout"]

        def linear(n):
            return QL(tuple(-1 if i == 0 else i - 1 for i in range(n)))

        smallest = float("inf")
        for run_name, members in (("single", (0,)), ("batch", tuple(range(len(prompts))))):
            cache = ref["PagedKVCache"](model.kv_cache_spec,
                                        ref["PagedKVCacheConfig"](len(prompts) * per_seq, QWEN2_BLOCK,
                                                                  dtype=torch.float16))
            run_tables = [tables[i] for i in members]

            def run(ids, positions, computed, lengths):
                starts = [0]
                for n in lengths:
                    starts.append(starts[-1] + n)
                used = tuple(t[: -(-(c + n) // QWEN2_BLOCK)] for t, c, n in zip(run_tables, computed, lengths))
                md = ref["PagedAttentionMetadata"](block_tables=used, num_computed_tokens=tuple(computed),
                                                   query_layouts=tuple(linear(n) for n in lengths))
                batch = ref["ForwardBatch"](input_ids=torch.tensor(ids, dtype=torch.long),
                                            positions=torch.tensor(positions, dtype=torch.long),
                                            query_start_loc=tuple(starts),
                                            attention=ref["TorchPagedAttention"](cache, md),
                                            logit_query_indices=tuple(s - 1 for s in starts[1:]))
                logits = model(batch).logits.float()
                top2 = logits.topk(2, dim=-1)
                second.append(top2.indices[:, 1].tolist())
                return logits.argmax(-1).tolist(), (top2.values[:, 0] - top2.values[:, 1]).tolist()

            second: list[list[int]] = []
            ps = [prompts[i] for i in members]
            nxt, marg = run([t for p in ps for t in p], [i for p in ps for i in range(len(p))],
                            [0] * len(ps), [len(p) for p in ps])
            tokens, margins = [nxt], [marg]
            ctx = [len(p) for p in ps]
            for _ in range(QWEN2_PIN_STEPS):
                if min(marg) < threshold:
                    return None
                nxt, marg = run(nxt, ctx, ctx, [1] * len(ps))
                tokens.append(nxt)
                margins.append(marg)
                ctx = [c + 1 for c in ctx]
            out[f"{run_name}_second"] = np.asarray(second, dtype=np.int64)
            if min(marg) < threshold:
                return None
            smallest = min(smallest, float(np.min(margins)))
            out[f"{run_name}_tokens"] = np.asarray(tokens, dtype=np.int64)   # [1 + steps, requests]
            out[f"{run_name}_margins"] = np.asarray(margins, dtype=np.float32)
    for i, p in enumerate(prompts):
        out[f"prompt{i}"] = np.asarray(p, dtype=np.int64)
    out["tables"] = np.asarray(tables, dtype=np.int32)
    out["config_json"] = np.frombuffer(json.dumps(dict(QWEN2_PIN, group_size=128, block_size=QWEN2_BLOCK,
                                                       seed=seed, weights_sha256=checksum(state))).encode(),
                                       dtype=np.uint8)
    if write:
        np.savez_compressed(HERE / "qwen2_decode_pin.npz", **out)
    return smallest


def main() -> None:
    torch.set_num_threads(1)
    ref = _import_reference()
    make_awq(ref)
    make_meta(ref)
    make_attention(ref)
    make_fused_norm(ref)
    make_qwen2(ref)
    make_qwen2_pin(ref)
    for name in ("awq_golden.npz", "paged_meta.json", "paged_attn.npz", "fused_norm.npz", "qwen2_greedy.npz",
                 "qwen2_decode_pin.npz"):
        print(name, (HERE / name).stat().st_size, "bytes")


if __name__ == "__main__":
    main()
