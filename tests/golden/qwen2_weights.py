"""Seeded random-init AWQ Qwen2 weights, regenerated identically on any host.

Test infrastructure.  ``random_awq_state(config, seed)`` returns the
state dict of a random-init AWQ ``Qwen2ForCausalLM`` (the reference's key
names, modeling/models/qwen2.py, before ``prepare_for_inference`` merges the
projections) drawn from one CPU ``torch.Generator`` in a fixed order that
depends only on the configuration.  ``make_golden.py`` loads it into the
reference's own model to record greedy tokens; the GPU tests regenerate the
same tensors from the seed, so fixtures for multi-megabyte models carry only
the seed, the prompts and the tokens.

Distributions: int4 codes and zero points uniform in
0..15 packed in the AutoAWQ order (``oracle.awq.pack``, pinned bit-exactly
to the reference's ``pack_awq``), fp16 scales uniform in [0.002, 0.02], QKV
biases N(0, 0.1), norm weights U[0.5, 1.5], embeddings N(0, 0.5) and the
lm_head N(0, ``lm_head_std``).
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import awq as oawq


def projection_shapes(cfg: dict) -> list[tuple[str, int, int, bool]]:
    """(module name, in_features, out_features, has_bias) of every AWQ
    projection in state-dict order."""

    hidden = cfg["hidden_size"]
    inter = cfg["intermediate_size"]
    head = hidden // cfg["num_attention_heads"]
    kv = cfg["num_key_value_heads"] * head
    out = []
    for layer in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{layer}"
        out += [(f"{p}.self_attn.q_proj", hidden, hidden, True),
                (f"{p}.self_attn.k_proj", hidden, kv, True),
                (f"{p}.self_attn.v_proj", hidden, kv, True),
                (f"{p}.self_attn.o_proj", hidden, hidden, False),
                (f"{p}.mlp.gate_proj", hidden, inter, False),
                (f"{p}.mlp.up_proj", hidden, inter, False),
                (f"{p}.mlp.down_proj", inter, hidden, False)]
    return out


def random_awq_state(cfg: dict, seed: int, *, group_size: int = 128,
                     lm_head_std: float = 0.05) -> dict[str, torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    state: dict[str, torch.Tensor] = {}
    hidden = cfg["hidden_size"]
    for name, k, n, bias in projection_shapes(cfg):
        groups = k // group_size
        codes = torch.randint(0, 16, (k, n), generator=g, dtype=torch.int32).numpy()
        zeros = torch.randint(0, 16, (groups, n), generator=g, dtype=torch.int32).numpy()
        state[f"{name}.qweight"] = torch.from_numpy(oawq.pack(codes))
        state[f"{name}.qzeros"] = torch.from_numpy(oawq.pack(zeros))
        state[f"{name}.scales"] = (torch.rand(groups, n, generator=g) * 0.018 + 0.002).half()
        if bias:
            state[f"{name}.bias"] = (torch.randn(n, generator=g) * 0.1).half()
    for layer in range(cfg["num_hidden_layers"]):
        for norm in ("input_layernorm", "post_attention_layernorm"):
            state[f"model.layers.{layer}.{norm}.weight"] = (torch.rand(hidden, generator=g) + 0.5).half()
    state["model.norm.weight"] = (torch.rand(hidden, generator=g) + 0.5).half()
    vocab = cfg["vocab_size"]
    state["model.embed_tokens.weight"] = (torch.randn(vocab, hidden, generator=g) * 0.5).half()
    state["lm_head.weight"] = (torch.randn(vocab, hidden, generator=g) * lm_head_std).half()
    return state


def checksum(state: dict[str, torch.Tensor]) -> str:
    """Order-independent digest of a state dict (guards against a changed
    generator between the fixture's host and the test's)."""

    import hashlib

    h = hashlib.sha256()
    for key in sorted(state):
        h.update(key.encode())
        h.update(np.ascontiguousarray(state[key].numpy()).tobytes())
    return h.hexdigest()
