"""The allocation-free AWQ entry point agrees with the workspace entry point.

``lvb_awq_linear_static`` exists for callers that cannot allocate device
memory for a workspace (their device memory belongs to another allocator, or
cudaMalloc's device-wide synchronisation is off limits on their path); it uses
a fixed scratch array inside the library instead.  This test calls both entry
points through the C ABI on the same inputs, twice in a row with different
shapes (so the second call reuses scratch the first one left behind), and
checks each static result against the workspace result with the tolerance the
AWQ tests use (max-abs 2e-2, relative L2 1e-3).  This file is named to be
collected last.
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
    # Config-1 shape (split-K, BN=16), then a BN=64 split-K shape.
    for m, k, n, g, seed in ((16, 896, 4864, 128, 101), (40, 1024, 2048, 64, 202)):
        x, qw, qz, sc, bias = _inputs(m, k, n, g, seed)
        static_y = _static(lib, x, qw, qz, sc, bias, g)
        reference_y = _with_workspace(lib, x, qw, qz, sc, bias, g)
        torch.cuda.synchronize()
        assert _native.device_error() == 0
        max_abs, rel = oawq.error_metrics(static_y.float().cpu().numpy(),
                                          reference_y.float().cpu().numpy())
        assert max_abs <= 2e-2 and rel <= 1e-3, (m, k, n, max_abs, rel)
