#!/usr/bin/env python
"""Benchmark of the light-vllm hot path on B200.

Workload: one paged-attention decode step of the
Qwen2.5-7B head geometry -- 64 sequences, one query token each, contexts
uniform in [512, 4096], 28 query / 4 KV heads, head_dim 128, bf16 K/V pages
N(0, 1), block_size 16, block tables carved from a random permutation of a
40,000-block pool, softmax scale 1/sqrt(128).  A step is the K/V write of the
64 new tokens plus the attention over every page.

Reported (one JSON line on rank 0):
  value      attention HBM GB/s over the whole job: algorithmic bytes (K and V
             pages read, Q read, O written, block tables, new K/V rows written)
             / device time of K steps replayed back to back from a CUDA graph,
             inputs resident in HBM.  The 302 MB of K/V per step exceed the
             126 MB L2, so no flush is needed between steps.
  e2e        the same bytes / time through the public API per step:
             one H2D copy of q | k | v from one pinned host buffer, backend.create(cache,
             metadata) (block-table validation + one staged metadata copy),
             forward(), D2H of the output.
  roofline   the decode-attention launch (one split-context kernel whose last
             split per request merges the partials) timed alone with CUDA
             events; peak = measured HBM copy bandwidth; traffic = DRAM bytes
             per launch from the committed ncu summary of this workload.
  cpu_baseline  the CPU oracle (a restatement of the reference's
             TorchPagedAttention) on this host's cores over the same batch.
  awq        (detail) the W4A16 linear through B200AWQScheme on config 1 and
             model-scale shapes: decode sizes (m <= 64) run the packed
             tensor-memory kernel, prefill sizes the dequantising GEMM.

Multi-GPU (torchrun): attention shards over requests with no exchange, so each
rank runs its own copy of the batch ("weak" scaling, replicas); value sums the
ranks' bytes over the slowest rank's time.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tok/s + AWQ GEMM/attn HBM GB/s (% roofline) at 1/2/4/8 B200 vs host CPU"
UNIT = "GB/s"
CFG = dict(num_seqs=64, ctx_lo=512, ctx_hi=4096, hq=28, hkv=4, d=128, block_size=16, num_blocks=40000,
           seed=20261201)
WORKLOAD = ("paged-attention decode (BASELINE config 2): 64 seqs x 1 query, ctx U[512,4096], "
            "28q/4kv heads, head_dim 128, bf16 K/V, block 16, 40k-block pool")


def profiled_traffic(name: str) -> int | None:
    """DRAM bytes per launch (read + write) from a committed ncu summary, if any."""

    path = ROOT / "profiles" / name
    if not path.is_file():
        return None
    for line in path.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_launch:"):
            return int(line.split(":", 1)[1])
    return None


def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.is_file():
        data = json.loads(path.read_text())
        return {"hbm_gbs": float(data["hbm_gbs"]), "bf16_tflops": float(data["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


# ----------------------------------------------------------------------------
# workload
# ----------------------------------------------------------------------------
def cache_types():
    """light-vllm's own PagedKVCache / PagedAttentionMetadata classes (the
    offline install under baseline/_ref, or LIGHT_VLLM_SRC) -- the objects the
    backend receives in a real deployment -- else the oracle's stand-ins with
    the same surface (input construction only; nothing timed runs in them)."""

    from oracle.paged_cache import reference_types

    return reference_types()


def make_workload(torch, device):
    T = cache_types()
    AttentionLayerSpec, ModelKVCacheSpec = T.AttentionLayerSpec, T.ModelKVCacheSpec
    PagedAttentionMetadata, PagedKVCache, PagedKVCacheConfig = T.PagedAttentionMetadata, T.PagedKVCache, T.PagedKVCacheConfig
    linear_query_layout = T.linear_query_layout

    c = CFG
    gen = torch.Generator().manual_seed(c["seed"])
    ctx = torch.randint(c["ctx_lo"], c["ctx_hi"] + 1, (c["num_seqs"],), generator=gen).tolist()
    perm = torch.randperm(c["num_blocks"], generator=gen).tolist()
    tables, off = [], 0
    for n_ctx in ctx:
        n = -(-n_ctx // c["block_size"])
        tables.append(tuple(perm[off:off + n]))
        off += n
    md = PagedAttentionMetadata(block_tables=tuple(tables), num_computed_tokens=tuple(x - 1 for x in ctx),
                                query_layouts=tuple(linear_query_layout(1) for _ in ctx))
    spec = ModelKVCacheSpec((AttentionLayerSpec("layer0", c["hq"], c["hkv"], c["d"]),))
    cache = PagedKVCache(spec, PagedKVCacheConfig(c["num_blocks"], c["block_size"], dtype=torch.bfloat16,
                                                  device=device))
    torch.manual_seed(c["seed"])
    layer = cache.layer("layer0")
    layer.keys.normal_()
    layer.values.normal_()
    q = torch.randn(c["num_seqs"], c["hq"], c["d"], device=device, dtype=torch.bfloat16)
    k = torch.randn(c["num_seqs"], c["hkv"], c["d"], device=device, dtype=torch.bfloat16)
    v = torch.randn(c["num_seqs"], c["hkv"], c["d"], device=device, dtype=torch.bfloat16)
    return cache, md, q, k, v, ctx


def algorithmic_bytes(ctx) -> dict:
    c = CFG
    kv_read = sum(ctx) * c["hkv"] * c["d"] * 2 * 2
    q_bytes = c["num_seqs"] * c["hq"] * c["d"] * 2
    tables = sum(-(-x // c["block_size"]) for x in ctx) * 4
    attention = kv_read + 2 * q_bytes + tables
    kv_write = c["num_seqs"] * c["hkv"] * c["d"] * 2 * 2 * 2  # read new rows + write slots, K and V
    return {"attention": attention, "step": attention + kv_write, "kv_read": kv_read}


# ----------------------------------------------------------------------------
# clocks
# ----------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"lvb_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if self.proc is None or not self.path.is_file():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for _, _, flags in rows for n, f in zip(names, flags) if f.lower().startswith("active")})
        loaded = sorted(r[0] for r in rows)
        upper = loaded[len(loaded) // 2:] or loaded
        return {"sm_mhz": statistics.median(upper), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


# ----------------------------------------------------------------------------
# timing helpers
# ----------------------------------------------------------------------------
def time_graph(torch, graph, steps: int, warmup: int, dist=None) -> float:
    """Average device ms per replay, max over ranks."""

    for _ in range(warmup):
        graph.replay()
    stream = torch.cuda.current_stream()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    start.record(stream)
    for _ in range(steps):
        graph.replay()
    end.record(stream)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / steps
    if dist is not None:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def capture(torch, fn):
    fn()  # eager warm-up: kernel attributes are set outside the capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    torch.cuda.synchronize()
    return graph


# ----------------------------------------------------------------------------
# AWQ detail
# ----------------------------------------------------------------------------
def awq_detail(torch, peaks, steps: int, shapes_arg: str | None = None) -> list[dict]:
    import numpy as np

    from light_vllm_b200.awq import B200AWQScheme
    from oracle import awq as oawq  # input generator only (packing of random codes)

    shapes = [
        ("config1 0.5B up-proj", 16, 896, 4864, 128),
        ("7B gate_up", 1, 3584, 37888, 128),
        ("7B gate_up", 16, 3584, 37888, 128),
        ("7B gate_up", 64, 3584, 37888, 128),
        ("7B down", 16, 18944, 3584, 128),
        ("7B gate_up prefill", 2048, 3584, 37888, 128),
    ]
    if shapes_arg:
        shapes = [("custom",) + tuple(int(v) for v in item.split(",")) + (128,)
                  for item in shapes_arg.split(";") if item]
    out = []
    l2 = 126 * 1024 * 1024
    for name, m, k, n, g in shapes:
        qweight, qzeros, scales = oawq.random_checkpoint(k, n, g, seed=m + k + n)
        weight_bytes = qweight.nbytes + qzeros.nbytes + scales.nbytes
        copies = max(1, math.ceil(2 * l2 / weight_bytes)) if m <= 256 else 1
        dev = torch.device("cuda")
        base = [torch.from_numpy(a).to(dev) for a in (qweight, qzeros, scales)]
        ops = []
        for i in range(copies):
            ts = [t.clone() for t in base] if i else base
            ops.append(B200AWQScheme().prepare(*ts, g, None))
        x = torch.randn(m, k, dtype=torch.float16, device=dev)

        def run():
            for op in ops:
                op(x)

        graph = capture(torch, run)
        ms = time_graph(torch, graph, max(3, steps // 4), 2) / copies
        io_bytes = weight_bytes + m * k * 2 + m * n * 2
        flops = 2.0 * m * k * n
        gbs = io_bytes / (ms * 1e-3) / 1e9
        tflops = flops / (ms * 1e-3) / 1e12
        out.append({"shape": name, "m": m, "k": k, "n": n, "group": g, "us_per_call": round(ms * 1e3, 2),
                    "gbs": round(gbs, 1), "tflops": round(tflops, 2),
                    "hbm_frac": round(gbs / peaks["hbm_gbs"], 3),
                    "tensor_frac": round(tflops / peaks["bf16_tflops"], 3),
                    "rotating_copies": copies})
        del ops, graph, base
        torch.cuda.empty_cache()
    return out


# ----------------------------------------------------------------------------
# The reference's own GPU paths on this B200 (detail, when light-vllm is importable)
# ----------------------------------------------------------------------------
def _time_fn(torch, fn, iters: int) -> float:
    """ms per call of fn: a CUDA graph of one call replayed when capturable,
    else back-to-back eager calls; CUDA events on the current stream."""

    try:
        graph = capture(torch, fn)
        return time_graph(torch, graph, iters, 3)
    except Exception:  # not capturable: eager calls
        torch.cuda.synchronize()
        for _ in range(3):
            fn()
        stream = torch.cuda.current_stream()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(iters):
            fn()
        end.record(stream)
        torch.cuda.synchronize()
        return start.elapsed_time(end) / iters


def reference_gpu_detail(torch, peaks, steps: int, cache, md, q, k, v, ctx, ours: dict) -> dict:
    """light-vllm's own GPU paths on the same B200 -- the CUDA AWQ extension
    (CudaAWQScheme: mma.sync K1 kernel below 256 rows, dequantise + cuBLAS
    above; JIT-built for this GPU by the reference's loader) and the Triton
    paged-attention backend -- on the same shapes and inputs as ours."""

    T = cache_types()
    if T.source != "light_vllm":
        return {"unavailable": "light-vllm is not importable (no baseline/_ref, no LIGHT_VLLM_SRC)"}
    import numpy as np

    from oracle import awq as oawq  # input generator only
    out: dict = {}
    try:
        from light_vllm.modeling.quantization.awq_schemes import CudaAWQScheme

        t0 = time.perf_counter()
        scheme = CudaAWQScheme()
        rows = []
        l2 = 126 * 1024 * 1024
        for name, m, kk, n, g in (("config1 0.5B up-proj", 16, 896, 4864, 128), ("7B gate_up", 1, 3584, 37888, 128),
                                  ("7B gate_up", 16, 3584, 37888, 128), ("7B gate_up", 64, 3584, 37888, 128),
                                  ("7B down", 16, 18944, 3584, 128), ("7B gate_up prefill", 2048, 3584, 37888, 128)):
            qweight, qzeros, scales = oawq.random_checkpoint(kk, n, g, seed=m + kk + n)
            weight_bytes = qweight.nbytes + qzeros.nbytes + scales.nbytes
            copies = max(1, math.ceil(2 * l2 / weight_bytes)) if m <= 256 else 1
            dev = torch.device("cuda")
            base = [torch.from_numpy(a).to(dev) for a in (qweight, qzeros, scales)]
            ops = [scheme.prepare(*([t.clone() for t in base] if i else base), g, None) for i in range(copies)]
            x = torch.randn(m, kk, dtype=torch.float16, device=dev)
            if "build_s" not in out:
                ops[0](x)
                torch.cuda.synchronize()
                out["build_s"] = round(time.perf_counter() - t0, 1)

            def run():
                for op in ops:
                    op(x)

            ms = _time_fn(torch, run, max(3, steps // 4)) / copies
            io_bytes = weight_bytes + m * kk * 2 + m * n * 2
            gbs = io_bytes / (ms * 1e-3) / 1e9
            row = {"shape": name, "m": m, "k": kk, "n": n, "us_per_call": round(ms * 1e3, 2), "gbs": round(gbs, 1),
                   "hbm_frac": round(gbs / peaks["hbm_gbs"], 3),
                   "tflops": round(2.0 * m * kk * n / (ms * 1e-3) / 1e12, 2)}
            mine = [r for r in ours.get("awq", []) if (r["m"], r["k"], r["n"]) == (m, kk, n)]
            if mine:
                row["b200_us_per_call"] = mine[0]["us_per_call"]
                row["b200_speedup"] = round(ms * 1e3 / mine[0]["us_per_call"], 2)
            rows.append(row)
            del ops, base
            torch.cuda.empty_cache()
        out["awq_cuda_extension"] = rows
    except Exception as exc:  # reported, not fatal
        out["awq_cuda_extension"] = {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}
    try:
        from light_vllm.runtime.execution.triton_paged_attention import TritonPagedAttentionBackend

        backend = TritonPagedAttentionBackend()
        scale = 1.0 / math.sqrt(CFG["d"])
        backend.create(cache, md).forward("layer0", q, k, v, scale=scale)  # Triton JIT compile
        torch.cuda.synchronize()
        # Device time of the write + attention kernels: one fresh context's
        # forward captured once and replayed (a context runs each layer once;
        # the Triton kernels were compiled above); and the public API per step
        # (create + forward), as our e2e without the host copies.
        step_ctx = backend.create(cache, md)
        torch.cuda.synchronize()
        try:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                step_ctx.forward("layer0", q, k, v, scale=scale)
            ms_dev = time_graph(torch, graph, steps, 3)
        except Exception:  # not capturable: no device-only figure
            ms_dev = None

        def api_step():
            backend.create(cache, md).forward("layer0", q, k, v, scale=scale)

        stream = torch.cuda.current_stream()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(steps):
            api_step()
        end.record(stream)
        torch.cuda.synchronize()
        ms_api = start.elapsed_time(end) / steps
        nbytes = algorithmic_bytes(ctx)["step"]
        out["attention_triton_config2"] = {
            "ms_per_step_device": None if ms_dev is None else round(ms_dev, 4),
            "gbs_device": None if ms_dev is None else round(nbytes / (ms_dev * 1e-3) / 1e9, 1),
            "ms_per_step_api": round(ms_api, 4), "gbs_api": round(nbytes / (ms_api * 1e-3) / 1e9, 1),
            "b200_ms_per_step_device": ours.get("ms_per_step"),
            "b200_speedup_device": round(ms_dev / ours["ms_per_step"], 2) if ms_dev and ours.get("ms_per_step") else None,
            "b200_e2e_ms_per_step": ours.get("e2e_ms")}
    except Exception as exc:
        out["attention_triton_config2"] = {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}
    return out


# ----------------------------------------------------------------------------
# CPU baseline (the oracle restating the reference's Torch path)
# ----------------------------------------------------------------------------
def cpu_baseline(torch, cache, md, q, k, v, ctx, budget_s: float = 20.0) -> dict:
    from oracle import paged_attention as opa

    layer = cache.layer("layer0")
    kc, vc = layer.keys.cpu(), layer.values.cpu()
    qc, kk, vv = q.cpu(), k.cpu(), v.cpu()
    threads = torch.get_num_threads()
    scale = 1.0 / math.sqrt(CFG["d"])
    n_total = len(ctx)
    # Grow the sample until it takes a few seconds (bounded by the budget).
    n = 1
    elapsed = 0.0
    while True:
        tables = md.block_tables[:n]
        t0 = time.perf_counter()
        opa.attend(qc[:n], kk[:n], vv[:n], kc, vc, tables, md.num_computed_tokens[:n],
                   [(-1,)] * n, scale=scale)
        elapsed = time.perf_counter() - t0
        if n >= n_total or elapsed * (2 * n if 2 * n <= n_total else n_total) / n > budget_s or elapsed > 3.0:
            break
        n = min(n_total, 2 * n)
    sample_ctx = ctx[:n]
    c = CFG
    nbytes = (sum(sample_ctx) * c["hkv"] * c["d"] * 4 + n * c["hq"] * c["d"] * 4
              + sum(-(-x // c["block_size"]) for x in sample_ctx) * 4 + n * c["hkv"] * c["d"] * 8)
    return {"value": round(nbytes / elapsed / 1e9, 4), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"first {n} of {n_total} sequences ({sum(sample_ctx)} context tokens), one step, "
                      f"{elapsed:.2f} s"}


# ----------------------------------------------------------------------------
# ----------------------------------------------------------------------------
# Decode-step detail: the Qwen2 AWQ decoder stack on the B200 kernels
# ----------------------------------------------------------------------------
QWEN2_7B = dict(vocab_size=152064, hidden_size=3584, intermediate_size=18944, num_hidden_layers=28,
                num_attention_heads=28, num_key_value_heads=4, rms_norm_eps=1e-6, rope_theta=1e6)
# Intermediate 29696 = 29568 padded to 232 groups of 128 so that every TP shard is group-aligned.
QWEN2_72B = dict(vocab_size=152064, hidden_size=8192, intermediate_size=29696, num_hidden_layers=80,
                 num_attention_heads=64, num_key_value_heads=8, rms_norm_eps=1e-6, rope_theta=1e6)
# Intermediate 13824 (108 groups); at TP = 8 it is padded to 14336 so every shard is group-aligned.
QWEN2_14B = dict(vocab_size=152064, hidden_size=5120, intermediate_size=13824, num_hidden_layers=48,
                 num_attention_heads=40, num_key_value_heads=8, rms_norm_eps=1e-6, rope_theta=1e6)


def mixed_step_case(torch, shape, rank: int, world: int, device, steps: int, dist) -> dict:
    """one step of a 2048-token prefill chunk (fresh
    prompt) packed with 64 decode requests (contexts U[256, 8192]) through
    the runner's eager forward and ``B200PagedAttentionBackend`` (the
    reference's step-handler path: token-major batch, one create per step);
    the same step repeated, CUDA events, max over ranks.  Prefill GEMMs at
    M = 2112 run on tcgen05; attention runs the tile kernel for the chunk
    and the split decode kernel for the 64 decodes."""

    import gc

    from light_vllm_b200 import B200PagedAttentionBackend
    from light_vllm_b200.qwen2 import Qwen2AWQRunner, random_shard
    from oracle.paged_cache import model_spec

    T = cache_types()
    gc.collect()
    torch.cuda.empty_cache()
    chunk, n_dec = 2048, 64
    gen = torch.Generator().manual_seed(2026)
    ctx = torch.randint(256, 8193, (n_dec,), generator=gen).tolist()
    weights = random_shard(shape, rank, world, device, seed=11)
    runner = Qwen2AWQRunner(shape, weights, device, rank=rank, world=world, max_tokens=chunk + n_dec)
    del weights
    torch.cuda.empty_cache()
    try:
        lengths = [chunk] + [1] * n_dec
        computed = [0] + [c - 1 for c in ctx]
        need = [-(-(c + n) // 16) for c, n in zip(computed, lengths)]
        cache = T.PagedKVCache(model_spec(T, runner.kv_layers()),
                               T.PagedKVCacheConfig(sum(need), 16, dtype=torch.float16, device=device))
        for layer_id, *_ in runner.kv_layers():
            cache.layer(layer_id).keys.zero_()
            cache.layer(layer_id).values.zero_()
        tables, off = [], 0
        for n in need:
            tables.append(tuple(range(off, off + n)))
            off += n
        md = T.PagedAttentionMetadata(block_tables=tuple(tables), num_computed_tokens=tuple(computed),
                                      query_layouts=tuple(T.linear_query_layout(n) for n in lengths))
        ids = torch.randint(0, shape.vocab_size, (chunk + n_dec,), device=device)
        positions = torch.tensor([i for i in range(chunk)] + [c - 1 for c in ctx], dtype=torch.int32, device=device)
        rows = torch.tensor([chunk - 1] + [chunk + i for i in range(n_dec)], device=device)
        backend = B200PagedAttentionBackend()

        def step():
            return runner.forward(ids, positions, backend.create(cache, md), rows)

        for _ in range(2):
            step()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        stream = torch.cuda.current_stream()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for _ in range(steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1) / steps
        if dist is not None:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        lay = runner.layout
        h, d = shape.hidden_size, shape.head_size
        qkv_n = (lay.q_heads + 2 * lay.kv_heads) * d
        inter = lay.inter_part.local_size
        m = chunk + n_dec
        gemm_flops = 2.0 * m * shape.num_hidden_layers * (h * qkv_n + lay.q_heads * d * h + h * 2 * inter + inter * h)
        attn_flops = 4.0 * shape.num_hidden_layers * lay.q_heads * d * (chunk * (chunk + 1) / 2 + sum(ctx))
        return {"tp": world, "prefill_tokens": chunk, "decodes": n_dec, "decode_ctx": "U[256, 8192]",
                "ms_per_step": round(ms, 3), "tok_s": round(m / ms * 1e3, 1),
                "gemm_tflop_per_step_per_rank": round(gemm_flops / 1e12, 3),
                "attention_tflop_per_step_per_rank": round(attn_flops / 1e12, 3),
                "tflops_per_rank": round((gemm_flops + attn_flops) / (ms * 1e-3) / 1e12, 1),
                "intermediate": shape.intermediate_size, "kv": "fp16 pages, zero-filled (timing only)",
                "timing": "eager runner.forward over backend.create(cache, metadata), CUDA events, max over ranks"}
    finally:
        torch.cuda.synchronize()
        runner.close()


def decode_case(torch, shape, rank: int, world: int, device, batches, ctx: int, steps: int, warmup: int,
                dist, random_kv: bool) -> list[dict]:
    """Greedy decode steps of a random-init AWQ model, replayed from a CUDA
    graph (one graph per batch size), timed with CUDA events, max over ranks."""

    import gc

    from oracle.paged_cache import model_spec
    T = cache_types()
    PagedKVCache, PagedKVCacheConfig = T.PagedKVCache, T.PagedKVCacheConfig

    from light_vllm_b200.qwen2 import Qwen2AWQRunner, StaticDecodeAttention, random_shard

    gc.collect()
    torch.cuda.empty_cache()
    weights = random_shard(shape, rank, world, device, seed=7)
    runner = Qwen2AWQRunner(shape, weights, device, rank=rank, world=world, max_tokens=max(batches))
    del weights
    torch.cuda.empty_cache()
    _, _, kv_heads, head_size = runner.kv_layers()[0]
    kv_token_bytes = 2 * kv_heads * head_size * 2 * shape.num_hidden_layers
    def op_bytes(op):  # packed codes + (scale, zero) words, or the checkpoint tensors
        if op.groups is not None:
            return op.qweight.numel() * 4 + op.groups.numel() * op.groups.element_size()
        return op.qweight.numel() * 4 + op.qzeros.numel() * 4 + op.scales.numel() * 2

    awq_bytes = sum(op_bytes(op) for L in runner.layers for op in (L.qkv, L.o, L.gate_up, L.down))
    lm_bytes = runner.lm_head.numel() * 2
    out = []
    try:
        for b in batches:
            per = -(-(ctx + steps + warmup + 2) // 16)
            cache = PagedKVCache(model_spec(T, runner.kv_layers()),
                                 PagedKVCacheConfig(b * per, 16, dtype=torch.float16, device=device))
            for L in runner.layers:
                layer = cache.layer(L.layer_id)
                if random_kv:
                    layer.keys.normal_()
                    layer.values.normal_()
                else:
                    layer.keys.zero_()
                    layer.values.zero_()
            attention = StaticDecodeAttention(cache, [list(range(i * per, (i + 1) * per)) for i in range(b)],
                                              [ctx] * b, device)
            ids = torch.randint(0, shape.vocab_size, (b,), device=device)
            step = runner.capture_decode(attention, ids)
            for _ in range(warmup):
                step.replay()
            torch.cuda.synchronize()
            if dist is not None:
                dist.barrier()
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            stream = torch.cuda.current_stream()
            torch.cuda.nvtx.range_push("decode")  # lets a profiler capture only the timed steps
            ev0.record(stream)
            for _ in range(steps):
                step.replay()
            ev1.record(stream)
            torch.cuda.synchronize()
            torch.cuda.nvtx.range_pop()
            ms = ev0.elapsed_time(ev1) / steps
            if dist is not None:
                t = torch.tensor([ms], device=device)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                ms = float(t.item())
            mean_ctx = ctx + warmup + steps / 2
            step_bytes = awq_bytes + lm_bytes + b * mean_ctx * kv_token_bytes
            out.append({"batch": b, "ctx": ctx, "ms_per_step": round(ms, 3), "tok_s": round(b / ms * 1e3, 1),
                        "bytes_per_step_per_rank": int(step_bytes),
                        "hbm_gbs_per_rank": round(step_bytes / (ms * 1e-3) / 1e9, 1)})
            del step, attention, cache
            torch.cuda.empty_cache()
    finally:
        torch.cuda.synchronize()
        runner.close()
    return out


def decode_cpu_baseline(torch, budget_s: float = 20.0) -> dict:
    """The reference's CPU Torch path for one 7B decoder layer at batch 1
    (the Torch AWQ scheme dequantises every weight per call, then an fp16
    matmul), extrapolated to 28 layers; the lm_head GEMV is timed on an
    eighth of the vocabulary and scaled."""

    import numpy as np

    from oracle import awq as oawq  # CPU baseline leg only

    torch.manual_seed(0)
    h, inter, g = QWEN2_7B["hidden_size"], QWEN2_7B["intermediate_size"], 128
    rng = np.random.default_rng(0)

    def proj(k, n):
        qw = torch.from_numpy(rng.integers(-2**31, 2**31 - 1, (k, n // 8), dtype=np.int32))
        qz = torch.from_numpy(rng.integers(-2**31, 2**31 - 1, (k // g, n // 8), dtype=np.int32))
        sc = torch.rand(k // g, n).mul(0.018).add(0.002).half()
        return qw, qz, sc

    shapes = [(h, 4608), (h, h), (h, 2 * inter), (inter, h)]
    weights = [proj(k, n) for k, n in shapes]
    x = torch.randn(1, h).half()
    threads = torch.get_num_threads()
    t0 = time.perf_counter()
    layers = 0
    while True:
        for (k, n), (qw, qz, sc) in zip(shapes, weights):
            oawq.torch_linear(torch.randn(1, k).half(), qw, qz, sc, g, None)
        layers += 1
        if time.perf_counter() - t0 > budget_s / 2 or layers >= 3:
            break
    layer_s = (time.perf_counter() - t0) / layers
    lm = torch.randn(QWEN2_7B["vocab_size"] // 8, h).half()
    t1 = time.perf_counter()
    torch.mm(x, lm.t())
    lm_s = (time.perf_counter() - t1) * 8
    step_s = 28 * layer_s + lm_s
    return {"value": round(1.0 / step_s, 4), "unit": "decode tok/s (batch 1)", "cores": threads,
            "kind": "port", "sample": f"{layers} layer(s) of 7B AWQ projections through the Torch-scheme "
                                      f"restatement (dequantise per call + fp16 matmul) x 28 layers "
                                      f"extrapolated, plus the lm_head GEMV on 1/8 of the vocabulary x 8"}


def decode_detail(torch, device, rank: int, world: int, dist, steps: int, warmup: int, with_cpu: bool,
                  batches: str | None = None) -> dict:
    from light_vllm_b200.qwen2 import Qwen2Shape

    from light_vllm_b200.qwen2 import RankLayout

    def tp_layout_error(shape) -> str | None:
        try:
            RankLayout.of(shape, 0, world)
        except ValueError as exc:
            return str(exc)
        if (shape.intermediate_size // world) % shape.group_size:
            return "per-rank intermediate size is not a multiple of the AWQ group"
        return None

    steps = max(5, min(steps, 20))
    out = {}
    shape3 = Qwen2Shape(**QWEN2_7B)
    why = tp_layout_error(shape3)
    if why is None:
        sizes = tuple(int(b) for b in batches.split(",")) if batches else (1, 16, 64, 256)
        cfg3 = decode_case(torch, shape3, rank, world, device, sizes, 1024, 128, warmup, dist, random_kv=True)
        out["config3_qwen2.5_7b_awq"] = {"tp": world, "steps": cfg3, "prompt_tokens": 1024, "decode_steps": 128,
                                         "kv": "fp16 pages N(0,1) standing in for the 1024-token prompt's K/V",
                                         "allocated_gb_after": round(torch.cuda.memory_allocated(device) / 1e9, 2)}
    else:
        out["config3_qwen2.5_7b_awq"] = {"tp": world, "skipped": f"no TP={world} layout: {why}"}
    if not batches:  # BASELINE config 4 (TP = 2 / 4 / 8); TP = 1 fits one B200 (~128 GB) and anchors the scaling curve
        shape4 = Qwen2Shape(**QWEN2_72B)
        why = tp_layout_error(shape4)
        if why is None:
            cfg4 = decode_case(torch, shape4, rank, world, device, (128,), 2048, max(5, steps // 4), warmup, dist,
                               random_kv=False)
            out["config4_qwen2.5_72b_awq"] = {"tp": world, "steps": cfg4, "prompt_tokens": 2048,
                                              "intermediate": 29696, "kv": "fp16 pages, zero-filled (timing only)"}
        else:
            out["config4_qwen2.5_72b_awq"] = {"tp": world, "skipped": f"no TP={world} layout: {why}"}
    shape5 = Qwen2Shape(**dict(QWEN2_14B, intermediate_size=14336 if world == 8 else 13824))
    why = tp_layout_error(shape5)
    if not batches:
        out["config5_qwen2.5_14b_awq_mixed"] = (mixed_step_case(torch, shape5, rank, world, device, 5, dist)
                                                if why is None else {"tp": world, "skipped": f"no TP={world} layout: {why}"})
    out.update({
           "timing": "one CUDA graph per batch size: embedding, 4 AWQ projections, RoPE, K/V write, paged "
                     "attention, SiLU-mul, 2 fused all-reduce+add+RMSNorm per layer, lm_head, greedy pick; "
                     "CUDA events over K replays, max over ranks"})
    if with_cpu and rank == 0 and world == 1:
        out["cpu_baseline"] = decode_cpu_baseline(torch)
    return out


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--no-awq", action="store_true", help="skip the AWQ detail measurements")
    ap.add_argument("--only", choices=("all", "attention", "awq", "decode", "mixed"), default="all",
                    help="run one part (profiling); 'awq' prints only the AWQ detail")
    ap.add_argument("--awq-shapes", default=None,
                    help="AWQ detail shapes as 'm,k,n[;m,k,n...]' (group 128)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline (profiling)")
    ap.add_argument("--no-decode", action="store_true", help="skip the Qwen2 decode-step detail")
    ap.add_argument("--decode-batches", default=None,
                    help="config-3 batch sizes only, e.g. '1,16' (profiling; skips configs 4 and 5)")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing light-vllm's own GPU paths (CUDA AWQ extension, Triton attention)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return reference_arm(torch, args, rank, world)

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as tdist

        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
        dist = tdist

    from light_vllm_b200 import _native
    from light_vllm_b200.paged_attention import B200PagedAttentionBackend

    peaks = measured_peaks()
    if args.only == "decode":
        detail = decode_detail(torch, device, rank, world, dist, args.steps, args.warmup, with_cpu=not args.no_cpu,
                               batches=args.decode_batches)
        if rank == 0:
            print(json.dumps({"decode": detail}), flush=True)
        if dist is not None:
            dist.destroy_process_group()
        return 0
    if args.only == "mixed":  # BASELINE config 5 step alone (profiling the tile kernel)
        from light_vllm_b200.qwen2 import Qwen2Shape

        shape5 = Qwen2Shape(**dict(QWEN2_14B, intermediate_size=14336 if world == 8 else 13824))
        detail = mixed_step_case(torch, shape5, rank, world, device, max(1, min(args.steps, 5)), dist)
        if rank == 0:
            print(json.dumps({"config5_qwen2.5_14b_awq_mixed": detail}), flush=True)
        if dist is not None:
            dist.destroy_process_group()
        return 0
    if args.only == "awq":
        detail = awq_detail(torch, peaks, args.steps, args.awq_shapes)
        if rank == 0:
            print(json.dumps({"awq": detail}), flush=True)
        if dist is not None:
            dist.destroy_process_group()
        return 0
    cache, md, q, k, v, ctx = make_workload(torch, device)
    nbytes = algorithmic_bytes(ctx)
    scale = 1.0 / math.sqrt(CFG["d"])
    backend = B200PagedAttentionBackend()
    step_ctx = backend.create(cache, md)
    out = torch.empty_like(q)

    step_graph = capture(torch, lambda: step_ctx.launch("layer0", q, k, v, scale=scale, out=out))
    attn_graph = capture(torch, lambda: step_ctx.launch("layer0", q, k, v, scale=scale, out=out,
                                                        write_kv=False))

    gpu_index = int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local_rank)).split(",")[local_rank]) \
        if os.environ.get("CUDA_VISIBLE_DEVICES") else local_rank
    with ClockSampler(gpu_index) as clocks:
        step_ms = time_graph(torch, step_graph, args.steps, args.warmup, dist)
        attn_ms = time_graph(torch, attn_graph, args.steps, args.warmup, dist)
    clock_summary = clocks.summary()

    # End to end through the public API with host buffers, as a serving loop
    # runs it: the step's q | k | v sit in one pinned buffer (as the rows of a
    # merged QKV projection would) and reach the device in one copy; the API
    # gets views of the device copy; the output goes back to pinned memory.
    # The uploads and read-backs run on two copy streams (lvb_copy_async,
    # ordered by events), so step i + 1's upload and step i - 1's read-back
    # overlap step i's kernels; two device input buffers alternate, each
    # reused only after the attention that read it.  No host synchronisation
    # between steps.
    lib = _native.library()
    sizes = [t.numel() for t in (q, k, v)]
    pinned = torch.cat([t.reshape(-1) for t in (q, k, v)]).cpu().pin_memory()
    in_bytes = pinned.numel() * pinned.element_size()
    out_bytes = q.numel() * q.element_size()
    host_outs = [torch.empty(q.shape, dtype=q.dtype, pin_memory=True) for _ in range(2)]
    staged_flat = [torch.empty_like(pinned, device=device) for _ in range(2)]
    staged = [[part.view(t.shape) for part, t in zip(buf.split(sizes), (q, k, v))] for buf in staged_flat]
    stream = torch.cuda.current_stream()
    copy_in, copy_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    s_main, s_in, s_out = stream.cuda_stream, copy_in.cuda_stream, copy_out.cuda_stream
    pin_ptr = pinned.data_ptr()
    staged_ptr = [t.data_ptr() for t in staged_flat]
    hout_ptr = [t.data_ptr() for t in host_outs]

    def new_event():
        h = ctypes.c_void_p()
        _native.check(lib.lvb_event_create(ctypes.byref(h)), "lvb_event_create")
        return h.value

    ev_in = [new_event() for _ in range(2)]
    ev_done = [new_event() for _ in range(2)]
    ev_out = new_event()
    for ev in ev_done:
        lib.lvb_event_record(ev, s_main)

    def e2e_step(i):
        b = i & 1
        lib.lvb_stream_wait_event(s_in, ev_done[b])  # the attention that last read buffer b has finished
        lib.lvb_copy_async(staged_ptr[b], pin_ptr, in_bytes, s_in)
        lib.lvb_event_record(ev_in[b], s_in)
        lib.lvb_stream_wait_event(s_main, ev_in[b])
        o = backend.create(cache, md).forward("layer0", *staged[b], scale=scale)
        lib.lvb_event_record(ev_done[b], s_main)
        lib.lvb_stream_wait_event(s_out, ev_done[b])
        lib.lvb_copy_async(hout_ptr[b], o.data_ptr(), out_bytes, s_out)
        o.record_stream(copy_out)

    for i in range(args.warmup):
        e2e_step(i)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    e2e_steps = max(20, args.steps)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    host_t0 = time.perf_counter()
    for i in range(e2e_steps):
        e2e_step(i)
    host_ms = (time.perf_counter() - host_t0) * 1e3 / e2e_steps
    lib.lvb_event_record(ev_out, s_out)
    lib.lvb_stream_wait_event(s_main, ev_out)
    ev1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = ev0.elapsed_time(ev1) / e2e_steps
    if dist is not None:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    for ev in ev_in + ev_done + [ev_out]:
        lib.lvb_event_destroy(ev)
    dev_err = _native.device_error()
    if dev_err:
        raise RuntimeError(f"device error word {dev_err:#x}")

    meta_bytes = 4 * (sum(len(t) for t in md.block_tables) + 3 * len(ctx) + 1)
    h2d = sum(t.numel() * t.element_size() for t in (q, k, v)) + meta_bytes
    d2h = q.numel() * q.element_size()
    value = world * nbytes["step"] / (step_ms * 1e-3) / 1e9
    attn_gbs = nbytes["attention"] / (attn_ms * 1e-3) / 1e9
    e2e_value = world * nbytes["step"] / (e2e_ms * 1e-3) / 1e9

    result = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(step_ms, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) K/V pages, random-permutation block tables)",
        "config": {
            "workload": WORKLOAD,
            "global_batch": CFG["num_seqs"] * world,
            "parallelism": f"replicas x{world} (attention shards over requests, no collective)",
            "l2": "no flush: 302 MB of K/V pages per step exceed the 126 MB L2",
            "timing": "CUDA graph replays, CUDA events on the launching stream, max over ranks",
            "algorithmic_bytes_per_step": nbytes["step"],
            "decode_tokens_per_step": CFG["num_seqs"] * world,
            "decode_attention_tok_s": round(world * CFG["num_seqs"] / (step_ms * 1e-3), 1),
        },
        "roofline": {
            "bound": "hbm",
            "achieved": round(attn_gbs, 1),
            "peak": peaks["hbm_gbs"],
            "unit": "GB/s",
            "frac": round(attn_gbs / peaks["hbm_gbs"], 4),
            "traffic": profiled_traffic("paged_decode_cfg2.txt"),
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch "
                              "of this workload (profiles/paged_decode_cfg2.txt)",
            "kernel": "paged_decode_kernel (split-context decode) + decode_merge_kernel (split merge); "
                      "one lvb_paged_attention call",
            "peak_source": peaks["source"],
            "algorithmic_bytes_per_launch": nbytes["attention"],
            "launch_us": round(attn_ms * 1e3, 2),
        },
        "e2e": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4),
                "host_ms_per_step": round(host_ms, 4),
                "path": "backend.create(cache, metadata).forward(...) with pinned host q/k/v and output; "
                        "uploads and read-backs on two copy streams overlapping the neighbouring steps' kernels, "
                        "no host synchronisation between steps"},
        # per timed step: the split decode kernel (which also stores the
        # step's K/V rows) and the split merge
        "gpu_launches": 2 * args.steps,
        "clocks": clock_summary,
    }
    if rank == 0 and world == 1:
        if not args.no_cpu:
            result["cpu_baseline"] = cpu_baseline(torch, cache, md, q, k, v, ctx)
        if not args.no_awq and args.only == "all":
            result["awq"] = awq_detail(torch, peaks, args.steps, args.awq_shapes)
        if not args.no_reference_gpu and args.only == "all":
            result["reference_gpu"] = reference_gpu_detail(torch, peaks, args.steps, cache, md, q, k, v, ctx,
                                                           {"awq": result.get("awq", []), "ms_per_step": step_ms,
                                                            "e2e_ms": e2e_ms})
    if args.only == "all" and not args.no_decode:
        cache = step_ctx = step_graph = attn_graph = None
        torch.cuda.empty_cache()
        result["decode"] = decode_detail(torch, device, rank, world, dist, args.steps, args.warmup,
                                         with_cpu=not args.no_cpu)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result), flush=True)
    return 0


def reference_arm(torch, args, rank: int, world: int) -> int:
    """The reference's CPU implementation of the path (the oracle port of
    TorchPagedAttention) on this host's cores, same workload and metric."""

    if rank != 0:
        return 0
    torch.set_num_threads(os.cpu_count() or 1)
    cache, md, q, k, v, ctx = make_workload(torch, torch.device("cuda", 0) if torch.cuda.is_available()
                                            else torch.device("cpu"))
    from oracle import paged_attention as opa

    layer = cache.layer("layer0")
    kc, vc = layer.keys.cpu(), layer.values.cpu()
    qc, kk, vv = q.cpu(), k.cpu(), v.cpu()
    n = len(ctx)
    scale = 1.0 / math.sqrt(CFG["d"])
    # Each step is the whole 64-sequence batch (about 1.2 s on 16 host
    # threads), the same workload as the GPU arm's step.
    times = []
    total_bytes = 0
    steps = args.warmup + args.steps
    for i in range(steps):
        sl = slice(0, n)
        sample_ctx = ctx[sl]
        t0 = time.perf_counter()
        opa.attend(qc[sl], kk[sl], vv[sl], kc, vc, md.block_tables[sl], md.num_computed_tokens[sl],
                   [(-1,)] * len(sample_ctx), scale=scale)
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            times.append(dt)
            c = CFG
            total_bytes += (sum(sample_ctx) * c["hkv"] * c["d"] * 4 + len(sample_ctx) * c["hq"] * c["d"] * 4
                            + sum(-(-x // c["block_size"]) for x in sample_ctx) * 4
                            + len(sample_ctx) * c["hkv"] * c["d"] * 8)
    secs = sum(times)
    value = total_bytes / secs / 1e9
    result = {
        "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(secs / len(times) * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "impl": "reference",
        "config": {"workload": WORKLOAD, "global_batch": CFG["num_seqs"], "parallelism": "host CPU",
                   "step": f"the whole batch of {n} sequences per step"},
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": f"all {n} sequences per step, {args.steps} timed steps"},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(result), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
