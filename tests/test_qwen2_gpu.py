"""Qwen2 AWQ decoder stack on B200 against the reference's greedy tokens.

tests/golden/qwen2_greedy.npz holds a seeded random-init AWQ Qwen2 (2 layers,
hidden 256, 4 query / 2 KV heads, vocabulary 512, group 128) and the tokens
the reference's own Qwen2ForCausalLM produced greedily on CPU: a two-request
prefill (prompts of 7 and 12 tokens) and 64 decode steps.  The model seed was
chosen so that every step's top-2 logit margin is at least 0.0098 (5 fp16
ulps at the logits' scale): token identity is then decided by the arithmetic,
not by rounding ties.  The runner must reproduce every token exactly: eager
steps through ``B200PagedAttentionBackend``, graph-replayed decode steps
through ``StaticDecodeAttention``, and the same model split over two ranks.
"""

from __future__ import annotations

import datetime
import json
import os
import socket
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "qwen2_greedy.npz"


def _fixture():
    d = np.load(GOLDEN)
    cfg = json.loads(bytes(d["config_json"]).decode())
    weights = {k[2:]: torch.from_numpy(d[k]) for k in d.files if k.startswith("w:")}
    prompts = [d["prompt0"].tolist(), d["prompt1"].tolist()]
    return d, cfg, weights, prompts


def _generate(rank: int, world: int, graph: bool, group=None) -> np.ndarray:
    from light_vllm_b200 import B200PagedAttentionBackend
    from oracle.paged_cache import model_spec, reference_types

    T = reference_types()
    PagedAttentionMetadata, PagedKVCache, PagedKVCacheConfig = T.PagedAttentionMetadata, T.PagedKVCache, T.PagedKVCacheConfig
    linear_query_layout = T.linear_query_layout
    from light_vllm_b200.qwen2 import Qwen2AWQRunner, Qwen2Shape, StaticDecodeAttention, shard_state_dict

    d, cfg, weights, prompts = _fixture()
    shape = Qwen2Shape.from_mapping(cfg)
    device = torch.device("cuda", torch.cuda.current_device())
    runner = Qwen2AWQRunner(shape, shard_state_dict(weights, shape, rank, world), device,
                            rank=rank, world=world, group=group, max_tokens=64)
    bs = cfg["block_size"]
    tables = [[int(b) for b in t] for t in d["tables"]]
    cache = PagedKVCache(model_spec(T, runner.kv_layers()), PagedKVCacheConfig(32, bs, dtype=torch.float16, device=device))
    backend = B200PagedAttentionBackend()
    steps = len(d["tokens"]) - 1

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
        nxt = eager_step([t for p in prompts for t in p], [0, 0], [len(p) for p in prompts])
        tokens = [nxt.tolist()]
        ctx = [len(p) for p in prompts]
        if not graph:
            for _ in range(steps):
                nxt = eager_step(nxt.tolist(), ctx, [1, 1])
                ctx = [c + 1 for c in ctx]
                tokens.append(nxt.tolist())
        else:
            attention = StaticDecodeAttention(cache, tables, ctx, device)
            ids = nxt.clone()
            step = runner.capture_decode(attention, ids)
            for _ in range(steps):
                step.replay()
                tokens.append(ids.tolist())
            del step
        return np.asarray(tokens)
    finally:
        torch.cuda.synchronize()
        runner.close()


def test_eager_greedy_matches_reference():
    from light_vllm_b200 import _native

    d, *_ = _fixture()
    got = _generate(0, 1, graph=False)
    assert _native.device_error() == 0
    np.testing.assert_array_equal(got, d["tokens"])


def test_graph_decode_matches_reference():
    from light_vllm_b200 import _native

    d, *_ = _fixture()
    got = _generate(0, 1, graph=True)
    assert _native.device_error() == 0
    np.testing.assert_array_equal(got, d["tokens"])


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_worker(rank: int, world: int, port: int, results) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=60),
                                         device_id=torch.device("cuda", rank))
    try:
        from light_vllm_b200 import _native

        got = _generate(rank, world, graph=True)
        results[rank] = ("ok", got.tolist(), _native.device_error())
    except Exception as exc:  # reported to the parent
        results[rank] = ("error", repr(exc), -1)
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_tensor_parallel_greedy_matches_reference(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    d, *_ = _fixture()
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        port = _free_port()
        procs = [ctx.Process(target=_tp_worker, args=(r, world, port, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
        for p in procs:
            if p.is_alive():
                p.kill()
        got = dict(results)
    for r in range(world):
        status, tokens, err = got.get(r, ("missing", None, None))
        assert status == "ok", f"rank {r}: {tokens}"
        assert err == 0
        np.testing.assert_array_equal(np.asarray(tokens), d["tokens"])


@pytest.mark.parametrize("head_size,hq,hkv,stride_pad", [(128, 28, 4, 0), (64, 4, 2, 0), (80, 8, 2, 0), (128, 7, 1, 8)])
def test_rope_matches_oracle(head_size, hq, hkv, stride_pad):
    """lvb_rope_qk against the oracle's half rotation (fp32 from fp16, one
    rounding): within one fp16 ulp; positions up to the table end."""

    from light_vllm_b200 import _native
    from oracle.qwen2 import apply_rope, rope_tables

    g = torch.Generator().manual_seed(head_size + hq)
    tokens = 37
    width = (hq + 2 * hkv) * head_size + stride_pad
    qkv = torch.randn(tokens, width, generator=g).half()
    positions = torch.randint(0, 4096, (tokens,), generator=g, dtype=torch.int32)
    positions[0] = 4095
    cos, sin = rope_tables(4096, head_size, 1e6)
    q = qkv[:, :hq * head_size].reshape(tokens, hq, head_size)
    k = qkv[:, hq * head_size:(hq + hkv) * head_size].reshape(tokens, hkv, head_size)
    want_q = apply_rope(q, positions.long(), cos, sin)
    want_k = apply_rope(k, positions.long(), cos, sin)
    dev = qkv.cuda()
    pos_d, cos_d, sin_d = positions.cuda(), cos.cuda(), sin.cuda()  # held until the kernel ran
    lib = _native.library()
    _native.check(lib.lvb_rope_qk(dev.data_ptr(), dev.stride(0), tokens, hq, hkv, head_size,
                                  pos_d.data_ptr(), cos_d.data_ptr(), sin_d.data_ptr(),
                                  4096, torch.cuda.current_stream().cuda_stream), "rope")
    got = dev.cpu()
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    for got_part, want in ((got[:, :hq * head_size].reshape(want_q.shape), want_q),
                           (got[:, hq * head_size:(hq + hkv) * head_size].reshape(want_k.shape), want_k)):
        ulp = torch.clamp(want.float().abs(), min=2.0**-14) * 2.0**-10
        assert float(((got_part.float() - want.float()).abs() / ulp).max()) <= 1.0
    # V columns and padding are untouched
    assert torch.equal(got[:, (hq + hkv) * head_size:], qkv[:, (hq + hkv) * head_size:])


def test_silu_mul_matches_fp32_reference():
    from light_vllm_b200 import _native

    g = torch.Generator().manual_seed(5)
    gate_up = (torch.randn(19, 2 * 1024, generator=g) * 3).half()
    want = (torch.nn.functional.silu(gate_up[:, :1024].float()) * gate_up[:, 1024:].float()).half()
    dev = gate_up.cuda()
    out = torch.empty(19, 1024, dtype=torch.float16, device="cuda")
    _native.check(_native.library().lvb_silu_mul(dev.data_ptr(), dev.stride(0), 19, 1024, out.data_ptr(),
                                                 out.stride(0), torch.cuda.current_stream().cuda_stream), "silu")
    ulp = torch.clamp(want.float().abs(), min=2.0**-14) * 2.0**-10
    assert float(((out.cpu().float() - want.float()).abs() / ulp).max()) <= 1.0


def test_rope_kv_write_equals_rope_then_write():
    """lvb_rope_kv_write is bit-identical to lvb_rope_qk followed by
    lvb_paged_kv_write: rotated queries in place, rotated keys and the values
    in the tokens' cache slots (two requests, mixed query lengths)."""

    from light_vllm_b200 import _native
    from oracle.qwen2 import rope_tables

    lib = _native.library()
    hq, hkv, d, bs, nb = 7, 1, 128, 16, 12
    g = torch.Generator().manual_seed(11)
    tokens = 5
    qkv = torch.randn(tokens, (hq + 2 * hkv) * d, generator=g).half().cuda()
    cos, sin = (t.cuda() for t in rope_tables(512, d, 1e6))
    tables = torch.tensor([[3, 7, 1], [9, 0, 5]], dtype=torch.int32, device="cuda")
    computed = torch.tensor([20, 40], dtype=torch.int32, device="cuda")
    qsl = torch.tensor([0, 3, 5], dtype=torch.int32, device="cuda")
    req = torch.tensor([0, 0, 0, 1, 1], dtype=torch.int32, device="cuda")
    positions = torch.tensor([20, 21, 22, 40, 41], dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    caches = []
    outs = []
    for fused in (False, True):
        kc = torch.zeros(nb, bs, hkv, d, dtype=torch.float16, device="cuda")
        vc = torch.zeros_like(kc)
        x = qkv.clone()
        if fused:
            _native.check(lib.lvb_rope_kv_write(x.data_ptr(), x.stride(0), tokens, hq, hkv, d, positions.data_ptr(),
                                                cos.data_ptr(), sin.data_ptr(), cos.shape[0], kc.data_ptr(),
                                                vc.data_ptr(), tables.data_ptr(), 3, computed.data_ptr(),
                                                qsl.data_ptr(), req.data_ptr(), bs, stream), "rope_kv_write")
        else:
            _native.check(lib.lvb_rope_qk(x.data_ptr(), x.stride(0), tokens, hq, hkv, d, positions.data_ptr(),
                                          cos.data_ptr(), sin.data_ptr(), cos.shape[0], stream), "rope")
            k = x[:, hq * d:(hq + hkv) * d]
            v = x[:, (hq + hkv) * d:]
            _native.check(lib.lvb_paged_kv_write(k.data_ptr(), x.stride(0), v.data_ptr(), x.stride(0), kc.data_ptr(),
                                                 vc.data_ptr(), tables.data_ptr(), 3, computed.data_ptr(),
                                                 qsl.data_ptr(), req.data_ptr(), tokens, hkv, d, bs,
                                                 _native.DTYPE_F16, stream), "kv_write")
        torch.cuda.synchronize()
        caches.append((kc, vc))
        outs.append(x[:, :hq * d].clone())
    assert _native.device_error() == 0
    assert torch.equal(outs[0], outs[1])
    assert torch.equal(caches[0][0], caches[1][0]) and torch.equal(caches[0][1], caches[1][1])
    assert bool(caches[1][0].abs().sum() > 0)


@pytest.mark.parametrize("hidden,hq,hkv,d,position", [(3584, 28, 4, 128, 1037), (896, 14, 2, 64, 5), (2048, 16, 2, 128, 0)])
def test_qkv_rope_gemv_equals_projection_then_rope_kv_write(hidden, hq, hkv, d, position):
    """lvb_awq_qkv_rope_packed (one-row QKV GEMV with the RoPE / K/V-write
    epilogue) is bit-identical to lvb_awq_linear_packed followed by
    lvb_rope_kv_write: rotated queries in y, unrotated keys and values in y,
    rotated keys and the values in the token's cache slot, nothing else of
    the cache touched (Qwen2.5-7B, 0.5B and the pinned model's shapes)."""

    from light_vllm_b200 import _native
    from light_vllm_b200.awq import pack_awq_decode_layout
    from oracle import awq as oawq
    from oracle.qwen2 import rope_tables

    lib = _native.library()
    n, g, bs, nb = (hq + 2 * hkv) * d, 128, 16, 80
    qweight, qzeros, scales = oawq.random_checkpoint(hidden, n, g, seed=hidden + d)
    rng = np.random.default_rng(position)
    x = torch.from_numpy(rng.standard_normal((1, hidden)).astype(np.float16)).cuda()
    bias = torch.from_numpy(rng.standard_normal(n).astype(np.float16)).cuda()
    codes, groups = pack_awq_decode_layout(*(torch.from_numpy(a).cuda() for a in (qweight, qzeros, scales)), g)
    cos, sin = (t.cuda() for t in rope_tables(2048, d, 1e6))
    # one request whose token sits at `position` in its table
    tables = torch.tensor([list(range(nb - 1, -1, -1))], dtype=torch.int32, device="cuda")
    computed = torch.tensor([position], dtype=torch.int32, device="cuda")
    qsl = torch.tensor([0, 1], dtype=torch.int32, device="cuda")
    req = torch.zeros(1, dtype=torch.int32, device="cuda")
    positions = torch.tensor([position], dtype=torch.int32, device="cuda")
    ws = torch.zeros(max(int(lib.lvb_awq_workspace_bytes(1, hidden, n, g)), 256), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    results = []
    for fused in (False, True):
        kc = torch.full((nb, bs, hkv, d), 7.0, dtype=torch.float16, device="cuda")
        vc = torch.full_like(kc, -3.0)
        y = torch.empty(1, n, dtype=torch.float16, device="cuda")
        if fused:
            _native.check(lib.lvb_awq_qkv_rope_packed(
                x.data_ptr(), codes.data_ptr(), groups.data_ptr(), bias.data_ptr(), y.data_ptr(), 1, hidden, n, g,
                ws.data_ptr(), ws.numel(), positions.data_ptr(), cos.data_ptr(), sin.data_ptr(), cos.shape[0],
                kc.data_ptr(), vc.data_ptr(), tables.data_ptr(), nb, computed.data_ptr(), qsl.data_ptr(),
                req.data_ptr(), hq, hkv, d, bs, stream), "qkv_rope")
            plain = y
        else:
            _native.check(lib.lvb_awq_linear_packed(x.data_ptr(), codes.data_ptr(), groups.data_ptr(),
                                                    bias.data_ptr(), y.data_ptr(), 1, hidden, n, g, ws.data_ptr(),
                                                    ws.numel(), stream), "linear")
            plain = y.clone()  # the projection before RoPE: its k and v columns
            _native.check(lib.lvb_rope_kv_write(y.data_ptr(), n, 1, hq, hkv, d, positions.data_ptr(), cos.data_ptr(),
                                                sin.data_ptr(), cos.shape[0], kc.data_ptr(), vc.data_ptr(),
                                                tables.data_ptr(), nb, computed.data_ptr(), qsl.data_ptr(),
                                                req.data_ptr(), bs, stream), "rope_kv_write")
        torch.cuda.synchronize()
        results.append((y[:, :hq * d].clone(), plain[:, hq * d:].clone(), kc, vc))
    assert _native.device_error() == 0
    (q0, kv0, k0, v0), (q1, kv1, k1, v1) = results
    assert torch.equal(q0, q1), "rotated queries differ"
    assert torch.equal(kv0, kv1), "unrotated k/v columns differ"
    assert torch.equal(k0, k1) and torch.equal(v0, v1), "cache contents differ"
    slot_block = int(tables[0, position // bs])
    assert int((k1 != 7.0).sum()) > 0 and bool((k1[slot_block, position % bs] != 7.0).any())
    others = torch.ones(nb, bs, dtype=torch.bool, device="cuda")
    others[slot_block, position % bs] = False
    assert bool((k1[others] == 7.0).all()) and bool((v1[others] == -3.0).all())


@pytest.mark.parametrize("tokens,vocab,hidden", [(1, 152064, 3584), (2, 4099, 256), (3, 1000, 8192), (4, 77, 5120)])
def test_lm_head_argmax_matches_fp16_logits(tokens, vocab, hidden):
    """lvb_lm_head_argmax against argmax over fp16 logits computed in float64
    (the reference's F.linear output rounded to fp16), including planted
    exact ties (equal rows: the lowest index wins, as torch.argmax), twice in
    a row on one workspace (it must be left zero)."""

    from light_vllm_b200 import _native

    g = torch.Generator().manual_seed(tokens * 7 + vocab)
    w = (torch.randn(vocab, hidden, generator=g) * 0.05).half()
    h = torch.randn(tokens, hidden, generator=g).half()
    # tie: the best row of token 0 duplicated at a higher and a lower index
    logits64 = h.double() @ w.double().t()
    best0 = int(logits64[0].argmax())
    lo = max(0, best0 - 3)
    w[lo] = w[best0]
    if best0 + 5 < vocab:
        w[best0 + 5] = w[best0]
    want = (h.double() @ w.double().t()).half().float()
    want_idx = want.argmax(dim=-1)
    want_val = want.max(dim=-1).values
    lib = _native.library()
    ws = torch.zeros(int(lib.lvb_lm_head_workspace_bytes()), dtype=torch.uint8, device="cuda")
    wd, hd = w.cuda(), h.cuda()
    for _ in range(2):
        idx = torch.full((tokens,), -1, dtype=torch.int64, device="cuda")
        val = torch.empty(tokens, dtype=torch.float32, device="cuda")
        _native.check(lib.lvb_lm_head_argmax(hd.data_ptr(), hd.stride(0), tokens, wd.data_ptr(), vocab, hidden, 1000,
                                             idx.data_ptr(), val.data_ptr(), ws.data_ptr(),
                                             torch.cuda.current_stream().cuda_stream), "lm_head")
        torch.cuda.synchronize()
        assert _native.device_error() == 0
        # fp32 accumulation may round a logit to the neighbouring fp16 value; the pick
        # must then still hold the maximum up to one fp16 ulp
        got = idx.cpu() - 1000
        assert torch.equal(got, want_idx) or all(
            float(want[t, got[t]]) >= float(want_val[t]) - float(want_val[t].abs()) * 2.0**-10 for t in range(tokens))
        assert int(got[0]) == min(lo, int(want_idx[0]))  # exact tie of equal rows: the lowest index
        assert torch.allclose(val.cpu(), want[torch.arange(tokens), got], rtol=0, atol=0)
        assert int(ws.cpu().sum()) == 0


def test_embedding_masks_rows_of_other_shards():
    from light_vllm_b200 import _native

    table = torch.randn(50, 64).half().cuda()
    ids = torch.tensor([100, 149, 99, 150, 120], dtype=torch.int64, device="cuda")
    out = torch.full((5, 64), 7.0, dtype=torch.float16, device="cuda")
    _native.check(_native.library().lvb_embedding(ids.data_ptr(), 5, table.data_ptr(), 100, 150, 64, out.data_ptr(),
                                                  out.stride(0), torch.cuda.current_stream().cuda_stream), "embed")
    torch.cuda.synchronize()
    want = torch.zeros(5, 64, dtype=torch.float16)
    for i, v in enumerate(ids.tolist()):
        if 100 <= v < 150:
            want[i] = table[v - 100].cpu()
    assert torch.equal(out.cpu(), want)
