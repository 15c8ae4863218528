"""Fused row-parallel epilogue on B200: all-reduce + residual add + RMSNorm.

``all_reduce_add_rms_norm`` (one launch over peer memory) against the CPU
oracle (oracle/tensor_parallel.py) and the reference's own outputs
(tests/golden/fused_norm.npz, written by ``fused_add_rms_norm``,
_qwen2_kernels.py:145-180, after a rank sum).

Tolerances: the residual is bit-exact (an fp16 rounding of an exact sum);
the normalised output is within 2 fp16 ulps of the oracle (fp32 sums in a
different order and ``rsqrtf``).
"""

from __future__ import annotations

import ctypes
import datetime
import os
import socket
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import tensor_parallel as otp

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def _close_fp16(got: torch.Tensor, want: torch.Tensor) -> None:
    got = got.float().cpu()
    want = want.float().cpu()
    ulp = torch.clamp(want.abs(), min=2.0**-14) * 2.0**-10
    err = (got - want).abs() / ulp
    assert float(err.max()) <= 2.0, f"max error {float(err.max()):.2f} ulp"


@pytest.fixture(scope="module")
def workspace():
    from light_vllm_b200.collectives import PeerWorkspace

    ws = PeerWorkspace(256, 3584, torch.device("cuda:0"), distributed=False)
    yield ws
    ws.close()


@pytest.mark.parametrize("mode", [1, 2, 3])
@pytest.mark.parametrize("tokens", [1, 16, 200, 256])
def test_single_rank_matches_oracle(workspace, tokens, mode):
    from light_vllm_b200 import _native
    from light_vllm_b200.collectives import all_reduce_add_rms_norm

    g = torch.Generator().manual_seed(tokens)
    partial = (torch.randn(tokens, 3584, generator=g) * 4).half()
    residual = (torch.randn(tokens, 3584, generator=g) * 8).half()
    weight = (torch.rand(3584, generator=g) * 2).half()
    want_norm, want_res = otp.all_reduce_add_rms_norm([partial], residual, weight, 1e-6)
    res_dev = residual.cuda()
    out, res_after = all_reduce_add_rms_norm(workspace, partial.cuda(), res_dev, weight.cuda(), 1e-6, mode=mode)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    assert res_after.data_ptr() == res_dev.data_ptr()
    assert torch.equal(res_after.cpu(), want_res)
    _close_fp16(out, want_norm)


def test_golden_reduced_tensors(workspace):
    """One rank handed the reference's reduced tensor reproduces its outputs."""

    from light_vllm_b200.collectives import all_reduce_add_rms_norm

    fx = np.load(GOLDEN / "fused_norm.npz")
    name = "w4_t3_h3584"
    partials = torch.from_numpy(fx[f"{name}_partials"])
    reduced = partials.float().sum(0).half()
    residual = torch.from_numpy(fx[f"{name}_residual"]).cuda()
    weight = torch.from_numpy(fx[f"{name}_weight"]).cuda()
    out, res = all_reduce_add_rms_norm(workspace, reduced.cuda(), residual, weight, float(fx[f"{name}_eps"]))
    assert torch.equal(res.cpu(), torch.from_numpy(fx[f"{name}_new_residual"]).half())
    _close_fp16(out, torch.from_numpy(fx[f"{name}_normed"]))


def test_rejects_shapes_outside_the_workspace(workspace):
    from light_vllm_b200.collectives import all_reduce_add_rms_norm

    x = torch.zeros(257, 3584, dtype=torch.float16, device="cuda")
    w = torch.ones(3584, dtype=torch.float16, device="cuda")
    with pytest.raises(ValueError):
        all_reduce_add_rms_norm(workspace, x, x.clone(), w, 1e-6)
    y = torch.zeros(4, 1024, dtype=torch.float16, device="cuda")
    with pytest.raises(ValueError):
        all_reduce_add_rms_norm(workspace, y, y.clone(), w[:1024], 1e-6)


@pytest.mark.parametrize("mode", [1, 3])
def test_wait_times_out_when_a_peer_never_arrives(mode):
    """World 2 with only rank 0 launching: its bounded wait on rank 1's flag
    (mode 1) or data (mode 3) runs out, the device error word says TIMEOUT
    and no output row is written.  Both workspaces are local allocations;
    nothing plays rank 1."""

    from light_vllm_b200 import _native

    lib = _native.library()
    nbytes = lib.lvb_allreduce_workspace_bytes(2, 8, 256)
    ptrs = []
    for _ in range(2):
        p = ctypes.c_void_p()
        _native.check(lib.lvb_ipc_alloc(nbytes, ctypes.byref(p), ctypes.create_string_buffer(64)), "alloc")
        ptrs.append(p.value)
        _native.check(lib.lvb_allreduce_workspace_init(p.value, 2, 8, 256), "init")
    try:
        arr = (ctypes.c_void_p * 2)(*ptrs)
        partial = torch.ones(8, 256, dtype=torch.float16, device="cuda")
        residual = torch.full((8, 256), 3.0, dtype=torch.float16, device="cuda")
        weight = torch.ones(256, dtype=torch.float16, device="cuda")
        out = torch.full((8, 256), -7.0, dtype=torch.float16, device="cuda")
        _native.check(lib.lvb_allreduce_add_rmsnorm(
            arr, 0, 2, partial.data_ptr(), residual.data_ptr(), weight.data_ptr(), out.data_ptr(),
            8, 256, 8, 1e-6, mode, torch.cuda.current_stream().cuda_stream), "launch")
        torch.cuda.synchronize()
        assert _native.device_error() == 1  # LVB_DEVERR_TIMEOUT
        assert bool((out == -7.0).all()) and bool((residual == 3.0).all())
    finally:
        torch.cuda.synchronize()
        for p in ptrs:
            _native.check(lib.lvb_ipc_free(p), "free")


def test_workspace_geometry_mismatch_is_refused_on_the_device():
    """A call whose world / rows / hidden differ from the workspace's
    initialisation records LVB_DEVERR_INDEX and touches nothing (two local
    workspaces play the ranks; the check runs before any peer access)."""

    from light_vllm_b200 import _native

    lib = _native.library()
    nbytes = lib.lvb_allreduce_workspace_bytes(2, 8, 256)
    ptrs = []
    for _ in range(2):
        p = ctypes.c_void_p()
        _native.check(lib.lvb_ipc_alloc(nbytes, ctypes.byref(p), ctypes.create_string_buffer(64)), "alloc")
        ptrs.append(p.value)
        _native.check(lib.lvb_allreduce_workspace_init(p.value, 2, 8, 256), "init")
    try:
        arr = (ctypes.c_void_p * 2)(*ptrs)
        partial = torch.ones(8, 256, dtype=torch.float16, device="cuda")
        out = torch.full((8, 256), -7.0, dtype=torch.float16, device="cuda")
        # max_tokens 4 describes a smaller workspace than the one initialised
        _native.check(lib.lvb_allreduce_add_rmsnorm(arr, 0, 2, partial.data_ptr(), None, None, out.data_ptr(),
                                                    4, 256, 4, 0.0, 3, torch.cuda.current_stream().cuda_stream),
                      "launch")
        torch.cuda.synchronize()
        assert _native.device_error() == 2  # LVB_DEVERR_INDEX
        assert bool((out == -7.0).all())
    finally:
        torch.cuda.synchronize()
        for p in ptrs:
            _native.check(lib.lvb_ipc_free(p), "free")


def test_single_rank_plain_sum_is_a_copy(workspace):
    from light_vllm_b200.collectives import all_reduce_sum_peer

    t = torch.randn(5, 3584, device="cuda").half()
    want = t.clone()
    all_reduce_sum_peer(workspace, t)
    torch.cuda.synchronize()
    assert torch.equal(t, want)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_worker(rank: int, world: int, port: int, results) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=60))
    from light_vllm_b200 import _native
    from light_vllm_b200.collectives import PeerWorkspace, all_reduce_add_rms_norm, all_reduce_sum_peer

    def inputs(seed, tokens):
        g = torch.Generator().manual_seed(seed)
        partials = (torch.randn(world, tokens, 3584, generator=g) * 4).half()
        residual = (torch.randn(tokens, 3584, generator=g) * 8).half()
        weight = (torch.rand(3584, generator=g) * 2).half()
        return partials, residual, weight

    def ulps(got, want):
        ulp = torch.clamp(want.float().abs(), min=2.0**-14) * 2.0**-10
        return float(((got.float().cpu() - want.float()).abs() / ulp).max())

    try:
        dev = torch.device("cuda", rank)
        ws = PeerWorkspace(512, 3584, dev)
        worst = 0.0
        cases = ((5, 1), (1, 2), (16, 0), (512, 2), (77, 3), (512, 3), (9, 3), (77, 1), (512, 1), (300, 2), (3, 3),
                 (1, 4), (77, 4), (512, 4), (9, 3), (300, 4), (13, 1), (100, 4))
        for it, (tokens, mode) in enumerate(cases):
            partials, residual, weight = inputs(100 * it, tokens)
            want_norm, want_res = otp.all_reduce_add_rms_norm(list(partials), residual, weight, 1e-6)
            out, res = all_reduce_add_rms_norm(ws, partials[rank].to(dev), residual.to(dev), weight.to(dev), 1e-6,
                                               mode=mode)
            torch.cuda.synchronize(dev)
            if not torch.equal(res.cpu(), want_res):
                raise AssertionError(f"residual mismatch at iteration {it}")
            worst = max(worst, ulps(out, want_norm))
            # plain in-place sum: bit-exact fp16 rounding of the fp32 rank sum
            t = partials[rank].to(dev)
            all_reduce_sum_peer(ws, t, mode=mode)
            if not torch.equal(t.cpu(), partials.float().sum(0).half()):
                raise AssertionError(f"sum mismatch at iteration {it}")
        # CUDA graph: the call counter lives on the device, so replays stay in step
        partials, residual, weight = inputs(7, 64)
        p_dev, r_dev, w_dev = partials[rank].to(dev), residual.to(dev), weight.to(dev)
        r_ref = residual.clone()
        stream = torch.cuda.Stream(dev)
        stream.wait_stream(torch.cuda.current_stream(dev))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            all_reduce_add_rms_norm(ws, p_dev, r_dev.clone(), w_dev, 1e-6)  # warm-up outside capture
            torch.cuda.synchronize(dev)
            with torch.cuda.graph(graph, stream=stream):
                g_out, _ = all_reduce_add_rms_norm(ws, p_dev, r_dev, w_dev, 1e-6, mode=1)
                g_out2, _ = all_reduce_add_rms_norm(ws, g_out, r_dev, w_dev, 1e-6, mode=2)
                g_out3, _ = all_reduce_add_rms_norm(ws, g_out2, r_dev, w_dev, 1e-6, mode=3)
                g_out4, _ = all_reduce_add_rms_norm(ws, g_out3, r_dev, w_dev, 1e-6, mode=4)
        for _ in range(3):
            graph.replay()
            torch.cuda.synchronize(dev)
            n1, r_ref = otp.all_reduce_add_rms_norm(list(partials), r_ref, weight, 1e-6)
            worst = max(worst, ulps(g_out, n1))
            # the second partial is the first output, identical on every rank
            n2, r_ref = otp.all_reduce_add_rms_norm([g_out.cpu()] * world, r_ref, weight, 1e-6)
            worst = max(worst, ulps(g_out2, n2))
            n3, r_ref = otp.all_reduce_add_rms_norm([g_out2.cpu()] * world, r_ref, weight, 1e-6)
            worst = max(worst, ulps(g_out3, n3))
            n4, r_ref = otp.all_reduce_add_rms_norm([g_out3.cpu()] * world, r_ref, weight, 1e-6)
            worst = max(worst, ulps(g_out4, n4))
            if not torch.equal(r_dev.cpu(), r_ref):
                raise AssertionError("graph replay residual mismatch")
        del graph
        err = _native.device_error()
        ws.close()
        results[rank] = ("ok", worst, err)
    except Exception as exc:  # reported to the parent
        results[rank] = ("error", repr(exc), -1)
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ranks_over_peer_memory(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank_worker, args=(r, world, port, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(180)
        for p in procs:
            if p.is_alive():
                p.kill()
        got = dict(results)
    for r in range(world):
        status, worst, err = got.get(r, ("missing", None, None))
        assert status == "ok", f"rank {r}: {worst}"
        assert err == 0
        assert worst <= 2.0, f"rank {r}: {worst:.2f} ulp"
