"""The allocation-free AWQ entry point agrees with the workspace entry point.

``lvb_awq_linear_static`` exists for callers that cannot allocate device
memory for a workspace (their device memory belongs to another allocator, or
cudaMalloc's device-wide synchronisation is off limits on their path); it uses
a fixed scratch array inside the library instead.  This test calls both entry
points through the C ABI on the same inputs: three shapes in a row (two
split-K plans, whose semaphores live in the shared array, and one plan without
split-K), each shape called twice back to back on the static entry point, so
later calls reuse scratch that earlier ones left behind.  Every static result
must equal the workspace result within the tolerance the AWQ tests use
(max-abs 2e-2, relative L2 1e-3), and both must meet that tolerance against
the fp32-accumulated CPU oracle.  This file is named to be collected last.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from light_vllm_b200 import _native
from oracle import awq as oawq

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _inputs(m, k, n, g, seed):
    qweight, qzeros, scales = oawq.random_checkpoint(k, n, g, seed=seed)
    rng = np.random.default_rng(seed + 1)
    x = rng.standard_normal((m, k)).astype(np.float16)
    bias = rng.standard_normal(n).astype(np.float16)
    return [torch.from_numpy(a).to(DEV) for a in (x, qweight, qzeros, scales, bias)]


def _with_workspace(lib, x, qw, qz, sc, bias, g):
    m, k = x.shape
    n = sc.shape[1]
    need = int(lib.lvb_awq_workspace_bytes(m, k, n, g))
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=DEV)
    y = torch.empty(m, n, dtype=torch.float16, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    _native.check(lib.lvb_awq_linear(x.data_ptr(), qw.data_ptr(), qz.data_ptr(), sc.data_ptr(),
                                     bias.data_ptr(), y.data_ptr(), m, k, n, g, ws.data_ptr(),
                                     ws.numel(), stream), "lvb_awq_linear")
    return y


def _static(lib, x, qw, qz, sc, bias, g):
    m, k = x.shape
    n = sc.shape[1]
    y = torch.empty(m, n, dtype=torch.float16, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    _native.check(lib.lvb_awq_linear_static(x.data_ptr(), qw.data_ptr(), qz.data_ptr(), sc.data_ptr(),
                                            bias.data_ptr(), y.data_ptr(), m, k, n, g, stream),
                  "lvb_awq_linear_static")
    return y


def test_static_scratch_entry_point_matches_workspace_entry_point():
    lib = _native.library()
    # Config-1 shape (split-K, BN=16), a BN=64 split-K shape, then m = 128
    # with enough output tiles that the plan has no split-K.
    shapes = ((16, 896, 4864, 128, 101), (40, 1024, 2048, 64, 202), (128, 1024, 4096, 128, 303))
    for m, k, n, g, seed in shapes:
        x, qw, qz, sc, bias = _inputs(m, k, n, g, seed)
        first = _static(lib, x, qw, qz, sc, bias, g)
        second = _static(lib, x, qw, qz, sc, bias, g)
        reference_y = _with_workspace(lib, x, qw, qz, sc, bias, g)
        torch.cuda.synchronize()
        assert _native.device_error() == 0
        want = reference_y.float().cpu().numpy()
        oracle_y = oawq.linear_fp32(x.cpu().numpy(), qw.cpu().numpy(), qz.cpu().numpy(), sc.cpu().numpy(), g,
                                    bias.cpu().numpy())
        for got in (first, second):
            max_abs, rel = oawq.error_metrics(got.float().cpu().numpy(), want)
            assert max_abs <= 2e-2 and rel <= 1e-3, (m, k, n, max_abs, rel)
            max_abs, rel = oawq.error_metrics(got.float().cpu().numpy(), oracle_y)
            assert max_abs <= 2e-2 and rel <= 1e-3, ("oracle", m, k, n, max_abs, rel)
        max_abs, rel = oawq.error_metrics(want, oracle_y)
        assert max_abs <= 2e-2 and rel <= 1e-3, ("workspace vs oracle", m, k, n, max_abs, rel)
