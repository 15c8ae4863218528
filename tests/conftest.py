from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

# light-vllm itself (baseline/_ref or LIGHT_VLLM_SRC) goes on sys.path before
# the package is imported, so that the backend's KVCacheError derives from the
# reference's and the tests drive the reference's own cache and metadata.
from oracle.paged_cache import reference_types  # noqa: E402

REF = reference_types()


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def pytest_collection_modifyitems(config: pytest.Config, items: list[pytest.Item]) -> None:
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
