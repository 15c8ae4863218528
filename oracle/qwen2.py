"""CPU restatement of the Qwen2 AWQ decoder step (test oracle).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.

Follows the reference model's forward (modeling/models/qwen2.py):
  embedding -> [layer 0: residual = x, x = RMSNorm(x)]
  per layer (qwen2.py:497-514):
    qkv = AWQ(x) + bias, split, RoPE on q and k        (qwen2.py:369-411)
    attention over the request's cached K/V + this step  (paged_attention.py:337-380)
    x, residual = add_rms_norm(o_proj(attn), residual)  (_qwen2_kernels.py:20-43)
    x = down(silu(gate) * up)                           (qwen2.py:233-253)
    x, residual = add_rms_norm(x, residual, next norm)
  final add_rms_norm with model.norm, lm_head, greedy argmax (sampling.py:103-112)
with the arithmetic of the kernels the reference runs on GPUs: fp16 tensors
between steps, fp32 inside each step (projections accumulate in fp32 and
round once with the bias; RoPE, SiLU-mul and the fused norm compute in fp32
and round once).  RoPE tables are fp32 angles rounded to fp16 cos/sin
(qwen2.py:676-705).  K/V are kept per request as contiguous fp16 rows; the
paged layout does not change the arithmetic.
"""

from __future__ import annotations

import numpy as np
import torch
from torch.nn import functional as F

from oracle import awq as oawq


def rope_tables(max_positions: int, head_size: int, theta: float) -> tuple[torch.Tensor, torch.Tensor]:
    """fp16 cos/sin [max_positions, head_size] (qwen2.py:683-705)."""

    positions = torch.arange(max_positions, dtype=torch.float32)
    freqs = 1.0 / (theta ** (torch.arange(0, head_size, 2, dtype=torch.float32) / head_size))
    angles = torch.outer(positions, freqs)
    emb = torch.cat((angles, angles), dim=-1)
    return emb.cos().half(), emb.sin().half()


def add_rms_norm(x: torch.Tensor, residual: torch.Tensor | None, weight: torch.Tensor,
                 eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """``fused_add_rms_norm`` (fp32, both results rounded to fp16); without a
    residual the input itself becomes the residual (qwen2.py:497-503)."""

    v = x.float() if residual is None else x.float() + residual.float()
    normed = F.rms_norm(v, (v.shape[-1],), weight.float(), eps)
    return normed.half(), v.half()


def apply_rope(x: torch.Tensor, positions: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Half rotation on [T, heads, D] fp16 (_qwen2_kernels.py:66-133)."""

    half = x.shape[-1] // 2
    xf = x.float()
    rotated = torch.cat((-xf[..., half:], xf[..., :half]), dim=-1)
    c = cos[positions].float().unsqueeze(1)
    s = sin[positions].float().unsqueeze(1)
    return (xf * c + rotated * s).half()


class Projection:
    """An AWQ projection dequantised once: y = fp16(x @ W + bias) in fp32."""

    def __init__(self, qweight, qzeros, scales, group_size: int, bias=None):
        self.weight = torch.from_numpy(
            oawq.dequantize(np.asarray(qweight), np.asarray(qzeros), np.asarray(scales), group_size)
        ).float()
        self.bias = None if bias is None else torch.as_tensor(np.asarray(bias)).float()

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        y = x.float() @ self.weight
        if self.bias is not None:
            y = y + self.bias
        return y.half()


def _cat_awq(parts, group_size):
    qweight = np.concatenate([p[0] for p in parts], axis=1)
    qzeros = np.concatenate([p[1] for p in parts], axis=1)
    scales = np.concatenate([p[2] for p in parts], axis=1)
    biases = [p[3] for p in parts]
    bias = None if biases[0] is None else np.concatenate(biases)
    return Projection(qweight, qzeros, scales, group_size, bias)


class Qwen2Oracle:
    """Greedy decoding of a Qwen2 AWQ model from a state dict (numpy arrays
    keyed like the reference's ``state_dict``)."""

    def __init__(self, weights: dict, config: dict):
        c = config
        self.hidden = c["hidden_size"]
        self.hq = c["num_attention_heads"]
        self.hkv = c["num_key_value_heads"]
        self.head = self.hidden // self.hq
        self.eps = c["rms_norm_eps"]
        self.layers_n = c["num_hidden_layers"]
        g = c["group_size"]

        def t(key):
            return torch.as_tensor(np.asarray(weights[key]))

        def awq(prefix, bias=False):
            return (weights[f"{prefix}.qweight"], weights[f"{prefix}.qzeros"], weights[f"{prefix}.scales"],
                    weights[f"{prefix}.bias"] if bias else None)

        self.embed = t("model.embed_tokens.weight")
        self.lm_head = t("lm_head.weight").float()
        self.final_norm = t("model.norm.weight")
        self.layers = []
        for i in range(self.layers_n):
            p = f"model.layers.{i}"
            self.layers.append(dict(
                qkv=_cat_awq([awq(f"{p}.self_attn.{n}_proj", True) for n in ("q", "k", "v")], g),
                o=_cat_awq([awq(f"{p}.self_attn.o_proj")], g),
                gate_up=_cat_awq([awq(f"{p}.mlp.{n}_proj") for n in ("gate", "up")], g),
                down=_cat_awq([awq(f"{p}.mlp.down_proj")], g),
                ln_in=t(f"{p}.input_layernorm.weight"),
                ln_post=t(f"{p}.post_attention_layernorm.weight"),
            ))
        self.cos, self.sin = rope_tables(c["max_position_embeddings"], self.head, c["rope_theta"])
        self.kv: dict[int, list[list[torch.Tensor]]] = {}

    def _attend(self, layer: int, request: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        cache = self.kv.setdefault(request, [[None, None] for _ in range(self.layers_n)])[layer]
        cache[0] = k if cache[0] is None else torch.cat((cache[0], k))
        cache[1] = v if cache[1] is None else torch.cat((cache[1], v))
        keys, values = cache[0].float(), cache[1].float()
        total = keys.shape[0]
        n = q.shape[0]
        group = self.hq // self.hkv
        keys = keys.repeat_interleave(group, dim=1)
        values = values.repeat_interleave(group, dim=1)
        scores = torch.einsum("qhd,khd->hqk", q.float(), keys) / self.head ** 0.5
        # query token j sits at position total - n + j and sees keys up to it
        mask = torch.arange(total).unsqueeze(0) > (total - n + torch.arange(n)).unsqueeze(1)
        scores = scores.masked_fill(mask.unsqueeze(0), float("-inf"))
        probs = torch.softmax(scores, dim=-1)
        return torch.einsum("hqk,khd->qhd", probs, values).half()

    def step(self, requests: list[tuple[list[int], int]]) -> tuple[list[int], torch.Tensor]:
        """Run one step; ``requests`` = [(token ids, position of the first)].
        Returns each request's greedy next token and the last-token logits."""

        ids = torch.tensor([t for toks, _ in requests for t in toks], dtype=torch.long)
        positions = torch.tensor([p0 + j for toks, p0 in requests for j in range(len(toks))], dtype=torch.long)
        bounds = np.cumsum([0] + [len(toks) for toks, _ in requests])
        x = self.embed[ids]
        x, residual = add_rms_norm(x, None, self.layers[0]["ln_in"], self.eps)
        qd, kd = self.hq * self.head, self.hkv * self.head
        for li, L in enumerate(self.layers):
            qkv = L["qkv"](x)
            q = qkv[:, :qd].reshape(-1, self.hq, self.head)
            k = qkv[:, qd:qd + kd].reshape(-1, self.hkv, self.head)
            v = qkv[:, qd + kd:].reshape(-1, self.hkv, self.head)
            q = apply_rope(q, positions, self.cos, self.sin)
            k = apply_rope(k, positions, self.cos, self.sin)
            attn = torch.cat([self._attend(li, r, q[bounds[r]:bounds[r + 1]], k[bounds[r]:bounds[r + 1]],
                                           v[bounds[r]:bounds[r + 1]]) for r in range(len(requests))])
            x, residual = add_rms_norm(L["o"](attn.reshape(-1, qd)), residual, L["ln_post"], self.eps)
            gu = L["gate_up"](x).float()
            inter = gu.shape[1] // 2
            act = (F.silu(gu[:, :inter]) * gu[:, inter:]).half()
            nxt = self.layers[li + 1]["ln_in"] if li + 1 < self.layers_n else self.final_norm
            x, residual = add_rms_norm(L["down"](act), residual, nxt, self.eps)
        last = torch.tensor(bounds[1:] - 1, dtype=torch.long)
        logits = (x[last].float() @ self.lm_head.t()).half()
        return logits.float().argmax(-1).tolist(), logits
