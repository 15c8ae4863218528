"""Qwen2 AWQ decoder stack on the sm_100a kernels (the callers of the hot path).

Restates the reference model's per-step dataflow (modeling/models/qwen2.py:
Qwen2MLP.forward 233-253, Qwen2Attention.forward 369-433,
Qwen2DecoderLayer.forward 497-514, Qwen2ForCausalLM.forward 636-673, RoPE
tables 676-705) over this package's operators, with tensor parallelism laid
out like the reference (column-parallel QKV and gate/up, row-parallel o/down,
vocab-parallel embedding and lm_head, KV heads replicated when there are
fewer than ranks: qwen2.py:290-318, tensor_parallel.py:248-330):

  x = embed(ids)                          lvb_embedding, masked per vocab shard
  x, residual = allreduce_add_rmsnorm(x, 0, input_layernorm)
  per layer:
    qkv  = AWQ(x) + bias                  B200AWQScheme, merged QKV; at one row the
    rope(q, k) + K/V write                RoPE and K/V write run in the QKV GEMV's
                                          epilogue (lvb_awq_qkv_rope_packed), else
                                          lvb_rope_kv_write (q in place, k, v to the pages)
    attn = attention.forward(q, ...)      B200PagedAttention (K/V already written)
    x, residual = allreduce_add_rmsnorm(AWQ_o(attn), residual, post_norm)
    x, residual = allreduce_add_rmsnorm(AWQ_down(silu(gate) * up), residual, next norm)
                                          (the SiLU-mul inside the down projection's
                                          activation prologue at decode sizes)
  next   = greedy over the full vocabulary   lvb_lm_head_argmax at <= 4 rows (no logits
                                          written), else cuBLAS logits + argmax;
                                          per-shard (max, index) gathered under TP

Every row-parallel sum, the residual add and the following RMSNorm are one
launch of ``lvb_allreduce_add_rmsnorm`` over NVLink peer memory (a single
rank runs the same kernel without peers).  The decode step takes no host
synchronisation, so ``capture_decode`` records it, with the greedy feedback
of the next token and the advance of every request's position, as one CUDA
graph.
"""

from __future__ import annotations

from dataclasses import dataclass
from collections.abc import Mapping

import torch
import torch.distributed as dist
from torch import Tensor

from light_vllm_b200 import _native
from light_vllm_b200.awq import B200AWQScheme
from light_vllm_b200.collectives import (
    PeerWorkspace,
    all_reduce_add_rms_norm,
    awq_column_shard,
    awq_row_shard,
    partition_dimension,
)
from light_vllm_b200.kv_cache import KVCacheError
from light_vllm_b200.paged_attention import _heads_contiguous, _rope_write_kv


@dataclass(frozen=True, slots=True)
class Qwen2Shape:
    """The Qwen2 configuration fields the decoder step uses (qwen2.py:43-140)."""

    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    max_position_embeddings: int = 32768
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    group_size: int = 128

    @property
    def head_size(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @classmethod
    def from_mapping(cls, values: Mapping[str, object]) -> "Qwen2Shape":
        names = cls.__dataclass_fields__
        return cls(**{k: v for k, v in values.items() if k in names})


@dataclass(frozen=True, slots=True)
class RankLayout:
    """What one tensor-parallel rank holds (qwen2.py:290-318)."""

    rank: int
    world: int
    q_heads: int
    kv_heads: int
    q_part: object
    kv_part: object
    inter_part: object
    vocab_part: object

    @classmethod
    def of(cls, shape: Qwen2Shape, rank: int, world: int) -> "RankLayout":
        hq, hkv, d = shape.num_attention_heads, shape.num_key_value_heads, shape.head_size
        if hq % world:
            raise ValueError("Qwen2 query heads must be divisible by tensor parallel size")
        if hkv >= world:
            if hkv % world:
                raise ValueError("Qwen2 KV heads must be divisible by tensor parallel size")
            kv_rank, kv_world = rank, world
        else:
            if world % hkv:
                raise ValueError("tensor parallel size must be divisible by Qwen2 KV heads when replicating")
            kv_rank, kv_world = rank // (world // hkv), hkv
        if shape.intermediate_size % world:
            raise ValueError("Qwen2 intermediate size must be divisible by tensor parallel size")
        return cls(rank, world, hq // world, max(1, hkv // world),
                   partition_dimension(hq * d, rank, world),
                   partition_dimension(hkv * d, kv_rank, kv_world),
                   partition_dimension(shape.intermediate_size, rank, world),
                   partition_dimension(shape.vocab_size, rank, world))


def shard_state_dict(weights: Mapping[str, Tensor], shape: Qwen2Shape, rank: int, world: int) -> dict:
    """This rank's slice of a full checkpoint state dict, keyed like the
    reference's (``checkpoint_shards`` of the AWQ and vocab-parallel layers,
    awq.py:165-198, 272-297, tensor_parallel.py:277-279)."""

    lay = RankLayout.of(shape, rank, world)
    g = shape.group_size
    out: dict[str, Tensor] = {}
    for i in range(shape.num_hidden_layers):
        p = f"model.layers.{i}"
        for name, part in (("q", lay.q_part), ("k", lay.kv_part), ("v", lay.kv_part)):
            key = f"{p}.self_attn.{name}_proj"
            qw, qz, sc, b = awq_column_shard(weights[f"{key}.qweight"], weights[f"{key}.qzeros"],
                                             weights[f"{key}.scales"], weights[f"{key}.bias"], part)
            out.update({f"{key}.qweight": qw, f"{key}.qzeros": qz, f"{key}.scales": sc, f"{key}.bias": b})
        for key, part in ((f"{p}.mlp.gate_proj", lay.inter_part), (f"{p}.mlp.up_proj", lay.inter_part)):
            qw, qz, sc, _ = awq_column_shard(weights[f"{key}.qweight"], weights[f"{key}.qzeros"],
                                             weights[f"{key}.scales"], None, part)
            out.update({f"{key}.qweight": qw, f"{key}.qzeros": qz, f"{key}.scales": sc})
        for key, part in ((f"{p}.self_attn.o_proj", lay.q_part), (f"{p}.mlp.down_proj", lay.inter_part)):
            qw, qz, sc = awq_row_shard(weights[f"{key}.qweight"], weights[f"{key}.qzeros"],
                                       weights[f"{key}.scales"], g, part)
            out.update({f"{key}.qweight": qw, f"{key}.qzeros": qz, f"{key}.scales": sc})
        for n in ("input_layernorm", "post_attention_layernorm"):
            out[f"{p}.{n}.weight"] = weights[f"{p}.{n}.weight"]
    vp = lay.vocab_part
    out["model.embed_tokens.weight"] = weights["model.embed_tokens.weight"][vp.start:vp.end].contiguous()
    out["lm_head.weight"] = weights["lm_head.weight"][vp.start:vp.end].contiguous()
    out["model.norm.weight"] = weights["model.norm.weight"]
    return out


def rope_tables(shape: Qwen2Shape, device: torch.device) -> tuple[Tensor, Tensor]:
    """fp16 cos/sin [max_positions, head_size], computed like
    ``prepare_for_inference`` (qwen2.py:683-705) on the model's device."""

    d = shape.head_size
    positions = torch.arange(shape.max_position_embeddings, dtype=torch.float32, device=device)
    freqs = 1.0 / (shape.rope_theta ** (torch.arange(0, d, 2, dtype=torch.float32, device=device) / d))
    angles = torch.outer(positions, freqs)
    emb = torch.cat((angles, angles), dim=-1)
    return emb.cos().half().contiguous(), emb.sin().half().contiguous()


class _Layer:
    __slots__ = ("layer_id", "qkv", "o", "gate_up", "down", "ln_in", "ln_post")


class Qwen2AWQRunner:
    """One rank's Qwen2 AWQ decoder stack (fp16 activations).

    ``weights`` is this rank's shard (``shard_state_dict``), keyed like the
    reference's state dict.  With ``world > 1`` a ``torch.distributed``
    process group must be initialised (the peer workspace exchanges CUDA IPC
    handles over it; the vocab-parallel greedy pick gathers over it).
    ``max_tokens`` bounds the tokens of one step.
    """

    def __init__(self, shape: Qwen2Shape, weights: Mapping[str, Tensor], device: torch.device, *,
                 rank: int = 0, world: int = 1, group: dist.ProcessGroup | None = None,
                 max_tokens: int = 256) -> None:
        self.shape = shape
        self.device = torch.device(device)
        self.rank, self.world, self.group = rank, world, group
        self.layout = RankLayout.of(shape, rank, world)
        self.max_tokens = int(max_tokens)
        scheme = B200AWQScheme()
        g = shape.group_size

        def dev(t):
            return t.to(self.device, non_blocking=True)

        def merged(keys, bias):
            qw = torch.cat([dev(weights[f"{k}.qweight"]) for k in keys], dim=1).contiguous()
            qz = torch.cat([dev(weights[f"{k}.qzeros"]) for k in keys], dim=1).contiguous()
            sc = torch.cat([dev(weights[f"{k}.scales"]) for k in keys], dim=1).contiguous()
            b = torch.cat([dev(weights[f"{k}.bias"]) for k in keys]).contiguous() if bias else None
            return scheme.prepare(qw, qz, sc, g, b)

        self.layers: list[_Layer] = []
        for i in range(shape.num_hidden_layers):
            p = f"model.layers.{i}"
            L = _Layer()
            L.layer_id = f"{p}.self_attn"
            L.qkv = merged([f"{p}.self_attn.{n}_proj" for n in ("q", "k", "v")], True)
            L.o = merged([f"{p}.self_attn.o_proj"], False)
            L.gate_up = merged([f"{p}.mlp.gate_proj", f"{p}.mlp.up_proj"], False)
            L.down = merged([f"{p}.mlp.down_proj"], False)
            L.ln_in = dev(weights[f"{p}.input_layernorm.weight"]).half().contiguous()
            L.ln_post = dev(weights[f"{p}.post_attention_layernorm.weight"]).half().contiguous()
            self.layers.append(L)
        self.embed = dev(weights["model.embed_tokens.weight"]).half().contiguous()
        self.lm_head = dev(weights["lm_head.weight"]).half().contiguous()
        self.final_norm = dev(weights["model.norm.weight"]).half().contiguous()
        self.cos, self.sin = rope_tables(shape, self.device)
        self.workspace = PeerWorkspace(self.max_tokens, shape.hidden_size, self.device, group,
                                       distributed=world > 1)
        self.scale = 1.0 / shape.head_size ** 0.5
        self._lib = _native.library()
        # zero-filled once; every lvb_lm_head_argmax call leaves it zero
        self.head_workspace = torch.zeros(int(self._lib.lvb_lm_head_workspace_bytes()), dtype=torch.uint8,
                                          device=self.device)

    # ------------------------------------------------------------------ specs
    def kv_layers(self) -> tuple[tuple[str, int, int, int], ...]:
        """Per-layer K/V geometry of this rank, (layer_id, query heads, KV
        heads, head size) -- the fields of the reference's
        ``AttentionLayerSpec`` entries of ``kv_cache_spec`` (qwen2.py:597-611);
        build the cache's ``ModelKVCacheSpec`` from them."""

        return tuple((L.layer_id, self.layout.q_heads, self.layout.kv_heads, self.shape.head_size)
                     for L in self.layers)

    def close(self) -> None:
        self.workspace.close()

    # ---------------------------------------------------------------- forward
    def _embed(self, ids: Tensor) -> Tensor:
        """Masked lookup of this rank's vocabulary rows (``lvb_embedding``;
        rows of other shards are zero and the following all-reduce sums
        them, tensor_parallel.py:296-306)."""

        vp = self.layout.vocab_part
        out = torch.empty((ids.shape[0], self.shape.hidden_size), dtype=torch.float16, device=self.device)
        ids = ids if ids.dtype == torch.int64 else ids.to(torch.int64)
        _native.check(self._lib.lvb_embedding(
            ids.data_ptr(), ids.shape[0], self.embed.data_ptr(), vp.start, vp.end, self.shape.hidden_size,
            out.data_ptr(), out.stride(0), _native.stream_handle(self.device)), "lvb_embedding")
        return out

    def _rope(self, qkv: Tensor, positions: Tensor) -> None:
        s = self.shape
        _native.check(self._lib.lvb_rope_qk(
            qkv.data_ptr(), qkv.stride(0), qkv.shape[0], self.layout.q_heads, self.layout.kv_heads, s.head_size,
            positions.data_ptr(), self.cos.data_ptr(), self.sin.data_ptr(), self.cos.shape[0],
            _native.stream_handle(self.device)), "lvb_rope_qk")

    def _greedy(self, hidden: Tensor) -> Tensor:
        """Greedy next token of each row (qwen2.py:665-673, sampling.py:103-112).
        Up to four rows: ``lvb_lm_head_argmax`` streams the head once and
        keeps per row the (maximum fp16 logit, lowest index) without writing
        logits; larger batches: cuBLAS logits and argmax."""

        t = hidden.shape[0]
        vp = self.layout.vocab_part
        if t <= 4:
            index = torch.empty(t, dtype=torch.int64, device=self.device)
            values = torch.empty(t, dtype=torch.float32, device=self.device) if self.world > 1 else None
            hidden = hidden if hidden.is_contiguous() else hidden.contiguous()
            _native.check(self._lib.lvb_lm_head_argmax(
                hidden.data_ptr(), hidden.stride(0), t, self.lm_head.data_ptr(), self.lm_head.shape[0],
                self.shape.hidden_size, vp.start, index.data_ptr(), None if values is None else values.data_ptr(),
                self.head_workspace.data_ptr(), _native.stream_handle(self.device)), "lvb_lm_head_argmax")
            if self.world == 1:
                return index
        else:
            logits = torch.mm(hidden, self.lm_head.t())
            if self.world == 1:
                return logits.argmax(dim=-1)
            values, index = logits.max(dim=-1)
            index = index + vp.start
        gv = torch.empty((self.world,) + tuple(values.shape), dtype=values.dtype, device=self.device)
        gi = torch.empty((self.world,) + tuple(index.shape), dtype=index.dtype, device=self.device)
        dist.all_gather_into_tensor(gv, values, group=self.group)
        dist.all_gather_into_tensor(gi, index, group=self.group)
        best = gv.argmax(dim=0)  # first maximum: the lowest vocabulary shard
        return gi.gather(0, best.unsqueeze(0)).squeeze(0)

    def forward(self, input_ids: Tensor, positions: Tensor, attention, logit_rows: Tensor | None = None) -> Tensor:
        """One model step over a token-major batch; returns the greedy next
        token of each row in ``logit_rows`` (every row when None).

        ``positions`` are int32 on the device; ``attention`` is an attention
        context (``B200PagedAttention`` or ``StaticDecodeAttention``)."""

        s, lay = self.shape, self.layout
        t = input_ids.shape[0]
        if t > self.max_tokens:
            raise ValueError(f"{t} tokens exceed the runner's max_tokens={self.max_tokens}")
        if positions.dtype != torch.int32:
            raise ValueError("positions must be int32")
        ws = self.workspace
        eps = s.rms_norm_eps
        qd, kd = lay.q_heads * s.head_size, lay.kv_heads * s.head_size
        fused_rope = s.head_size % 16 == 0 and hasattr(attention, "rope_write_kv")
        residual = torch.zeros((t, s.hidden_size), dtype=torch.float16, device=self.device)
        x, residual = all_reduce_add_rms_norm(ws, self._embed(input_ids), residual, self.layers[0].ln_in, eps)
        for i, L in enumerate(self.layers):
            qkv = None
            if fused_rope and t == 1 and hasattr(attention, "kv_write_args"):
                # One-row decode: RoPE and the K/V write run in the QKV
                # projection's own epilogue (qwen2.py:380-411).
                kv_args = attention.kv_write_args(L.layer_id)
                if kv_args is not None:
                    qkv = L.qkv.qkv_rope(x, positions, self.cos, self.sin, kv_args, lay.q_heads, lay.kv_heads,
                                         s.head_size)
                rope_done = qkv is not None
            else:
                rope_done = False
            if qkv is None:
                qkv = L.qkv(x)
            q = qkv[:, :qd].view(t, lay.q_heads, s.head_size)
            k = qkv[:, qd:qd + kd].view(t, lay.kv_heads, s.head_size)
            v = qkv[:, qd + kd:qd + 2 * kd].view(t, lay.kv_heads, s.head_size)
            if fused_rope:
                # RoPE fused with the K/V write (the QKV epilogue of qwen2.py:380-411)
                if not rope_done:
                    attention.rope_write_kv(L.layer_id, qkv, lay.q_heads, lay.kv_heads, positions, self.cos,
                                            self.sin)
                attn = attention.forward(L.layer_id, q, k, v, scale=self.scale, write_kv=False)
            else:
                self._rope(qkv, positions)
                attn = attention.forward(L.layer_id, q, k, v, scale=self.scale)
            x, residual = all_reduce_add_rms_norm(ws, L.o(attn.reshape(t, qd)), residual, L.ln_post, eps)
            # SiLU-mul runs inside the down projection's activation prologue
            # at decode batch sizes (lvb_awq_silu_linear_packed).
            down = L.down.silu_mul_linear(L.gate_up(x))
            nxt = self.layers[i + 1].ln_in if i + 1 < len(self.layers) else self.final_norm
            x, residual = all_reduce_add_rms_norm(ws, down, residual, nxt, eps)
        if logit_rows is not None:
            x = x.index_select(0, logit_rows)
        return self._greedy(x)

    # ------------------------------------------------------------ CUDA graph
    def capture_decode(self, attention: "StaticDecodeAttention", ids: Tensor) -> "DecodeGraph":
        """Record one decode step of every request in ``attention`` as a CUDA
        graph: forward, next token fed back into ``ids`` (int64, one per
        request) and every position advanced by one."""

        if ids.dtype != torch.int64 or ids.shape != (attention.num_seqs,):
            raise ValueError("ids must be an int64 tensor with one token per request")
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            # Warm-up: the same forward the first replay runs (same K/V slots,
            # same tokens), without feeding back or advancing.
            self.forward(ids, attention.computed, attention)
            torch.cuda.synchronize(self.device)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                nxt = self.forward(ids, attention.computed, attention)
                ids.copy_(nxt)
                attention.advance()
        torch.cuda.current_stream(self.device).wait_stream(stream)
        return DecodeGraph(graph, ids, attention)


class DecodeGraph:
    """A captured decode step; ``replay`` runs one step of every request."""

    def __init__(self, graph: torch.cuda.CUDAGraph, ids: Tensor, attention: "StaticDecodeAttention") -> None:
        self.graph = graph
        self.ids = ids
        self.attention = attention

    def replay(self) -> None:
        self.attention.reserve_step()
        self.graph.replay()


class StaticDecodeAttention:
    """Decode-only attention context whose metadata lives in fixed device
    buffers, so a step can be replayed from a CUDA graph.

    Each request owns a full block table reserved up front (``tables``, equal
    lengths), its current context length in ``computed`` (int32, also the
    position of its next token) and one query token per step.  The kernels
    read only the blocks the context uses.  ``advance`` moves every request
    one token on, on the device; the host counts steps so that no request
    outgrows its table."""

    def __init__(self, cache, tables, computed, device: torch.device) -> None:
        tables = [list(t) for t in tables]
        if not tables or len({len(t) for t in tables}) != 1:
            raise KVCacheError("static decode tables must be non-empty and of equal length")
        config = cache.config
        flat = [b for t in tables for b in t]
        if any(b < 0 or b >= config.num_blocks for b in flat):
            raise KVCacheError("block table references a block outside the KV cache")
        if len(set(flat)) != len(flat):
            raise KVCacheError("static decode block tables must not share blocks")
        if len(computed) != len(tables):
            raise KVCacheError("one context length per request is required")
        self.cache = cache
        self.device = torch.device(device)
        self.num_seqs = len(tables)
        self.stride = len(tables[0])
        self.capacity = self.stride * config.block_size
        if max(computed) >= self.capacity:
            raise KVCacheError("a request's context already fills its block table")
        self.tables = torch.tensor(tables, dtype=torch.int32, device=self.device)
        self.computed = torch.tensor(list(computed), dtype=torch.int32, device=self.device)
        self.query_start = torch.arange(self.num_seqs + 1, dtype=torch.int32, device=self.device)
        self.request_indices = torch.arange(self.num_seqs, dtype=torch.int32, device=self.device)
        self._host_max = max(computed)
        lib = _native.library()
        self._lib = lib
        spec = cache.model_spec.layers[0]
        need = int(lib.lvb_paged_attention_workspace_bytes(self.num_seqs, spec.num_query_heads, spec.num_kv_heads,
                                                            spec.head_size, self.capacity))
        # zeroed once: the split-merge semaphores start at zero and every call leaves them zero
        self.workspace = torch.zeros(max(need, 1 << 20), dtype=torch.uint8, device=self.device)

    def reserve_step(self) -> None:
        """Host check before a step: every request keeps a free slot."""

        if self._host_max + 1 > self.capacity:
            raise KVCacheError("a request would outgrow its reserved block table")
        self._host_max += 1

    def advance(self) -> None:
        self.computed.add_(1)

    def kv_write_args(self, layer_id: str) -> tuple | None:
        """Device addresses for a projection epilogue's K/V write (fp16 caches)."""

        if self.cache.config.dtype != torch.float16:
            return None
        layer = self.cache.layer(layer_id)
        return (layer.keys.data_ptr(), layer.values.data_ptr(), self.tables.data_ptr(), self.stride,
                self.computed.data_ptr(), self.query_start.data_ptr(), self.request_indices.data_ptr(),
                self.cache.config.block_size)

    def rope_write_kv(self, layer_id: str, qkv: Tensor, q_heads: int, kv_heads: int, positions: Tensor,
                      cos: Tensor, sin: Tensor) -> None:
        """RoPE fused with this step's K/V write (``lvb_rope_kv_write``)."""

        _rope_write_kv(self.cache, layer_id, qkv, q_heads, kv_heads, positions, cos, sin, self.tables.data_ptr(),
                       self.stride, self.computed.data_ptr(), self.query_start.data_ptr(),
                       self.request_indices.data_ptr(), self.device)

    def forward(self, layer_id: str, query: Tensor, key: Tensor, value: Tensor, *, scale: float,
                write_kv: bool = True) -> Tensor:
        spec = self.cache.layer_spec(layer_id)
        config = self.cache.config
        layer = self.cache.layer(layer_id)
        stream = _native.stream_handle(self.device)
        dtype_code = _native.DTYPE_BF16 if config.dtype == torch.bfloat16 else _native.DTYPE_F16
        query = _heads_contiguous(query, align=2)
        if write_kv:
            key = _heads_contiguous(key, align=8)
            value = _heads_contiguous(value, align=8)
            _native.check(self._lib.lvb_paged_kv_write(
                key.data_ptr(), key.stride(0), value.data_ptr(), value.stride(0),
                layer.keys.data_ptr(), layer.values.data_ptr(), self.tables.data_ptr(), self.stride,
                self.computed.data_ptr(), self.query_start.data_ptr(), self.request_indices.data_ptr(),
                self.num_seqs, spec.num_kv_heads, spec.head_size, config.block_size, dtype_code, stream),
                "lvb_paged_kv_write")
        out = torch.empty((self.num_seqs, spec.num_query_heads, spec.head_size), dtype=query.dtype,
                          device=self.device)
        _native.check(self._lib.lvb_paged_attention(
            query.data_ptr(), query.stride(0), layer.keys.data_ptr(), layer.values.data_ptr(),
            out.data_ptr(), out.stride(0), self.tables.data_ptr(), self.stride, self.computed.data_ptr(),
            self.query_start.data_ptr(), self.request_indices.data_ptr(), None, None, None,
            self.num_seqs, self.num_seqs, self.num_seqs, 1, self.capacity, spec.num_query_heads, spec.num_kv_heads,
            spec.head_size, config.block_size, config.num_blocks, float(scale), dtype_code,
            self.workspace.data_ptr(), self.workspace.numel(), stream), "lvb_paged_attention")
        return out


def random_shard(shape: Qwen2Shape, rank: int, world: int, device: torch.device, *, seed: int = 0) -> dict:
    """A seeded random-init AWQ checkpoint shard for this rank, generated on
    the device (the benchmark models: no checkpoint is read).  Packed codes
    and zero points are uniform int4, scales uniform in [0.002, 0.02], QKV
    biases N(0, 0.02), embedding / lm_head N(0, 0.02), norms one."""

    lay = RankLayout.of(shape, rank, world)
    g = shape.group_size
    h, d = shape.hidden_size, shape.head_size
    gen = torch.Generator(device=device)
    gen.manual_seed(seed * 1009 + rank)

    def codes(rows, cols):
        return torch.randint(-(2 ** 31), 2 ** 31 - 1, (rows, cols // 8), dtype=torch.int32, device=device,
                             generator=gen)

    def awq(k, n, bias=False):
        sc = (torch.rand((k // g, n), device=device, generator=gen) * 0.018 + 0.002).half()
        out = {"qweight": codes(k, n), "qzeros": codes(k // g, n), "scales": sc}
        if bias:
            out["bias"] = (torch.randn(n, device=device, generator=gen) * 0.02).half()
        return out

    w: dict[str, Tensor] = {}
    for i in range(shape.num_hidden_layers):
        p = f"model.layers.{i}"
        parts = {f"{p}.self_attn.q_proj": awq(h, lay.q_part.local_size, True),
                 f"{p}.self_attn.k_proj": awq(h, lay.kv_part.local_size, True),
                 f"{p}.self_attn.v_proj": awq(h, lay.kv_part.local_size, True),
                 f"{p}.self_attn.o_proj": awq(lay.q_part.local_size, h),
                 f"{p}.mlp.gate_proj": awq(h, lay.inter_part.local_size),
                 f"{p}.mlp.up_proj": awq(h, lay.inter_part.local_size),
                 f"{p}.mlp.down_proj": awq(lay.inter_part.local_size, h)}
        for key, tensors in parts.items():
            for name, t in tensors.items():
                w[f"{key}.{name}"] = t
        w[f"{p}.input_layernorm.weight"] = torch.ones(h, dtype=torch.float16, device=device)
        w[f"{p}.post_attention_layernorm.weight"] = torch.ones(h, dtype=torch.float16, device=device)
    v = lay.vocab_part.local_size
    w["model.embed_tokens.weight"] = (torch.randn((v, h), device=device, generator=gen) * 0.02).half()
    w["lm_head.weight"] = (torch.randn((v, h), device=device, generator=gen) * 0.02).half()
    w["model.norm.weight"] = torch.ones(h, dtype=torch.float16, device=device)
    del d
    return w
