"""The C-ABI library loads and exports exactly what include/lvb200.h declares.

CPU-only: no entry point that launches work is called here.
"""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from light_vllm_b200 import _native, build

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "lvb200.h"


def _declared_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^LVB_API [^;]*?\b(lvb_\w+)\(", text, flags=re.M))


def test_header_declares_every_bound_prototype():
    declared = _declared_symbols()
    assert declared, "no LVB_API declarations found"
    assert declared == set(_native.PROTOTYPES)


def test_library_is_built_and_current():
    assert _native.LIB_PATH.is_file(), "run python -m light_vllm_b200.build"
    assert not build.is_stale(), "library is older than its sources; rebuild it"


def test_library_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", str(_native.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = _declared_symbols() - exported
    assert not missing, f"not exported: {sorted(missing)}"
    # Internal helpers stay hidden.
    assert all(name.startswith("lvb_") for name in exported if "lvb" in name)


def test_library_loads_and_reports_abi():
    lib = _native.library()
    assert lib.lvb_abi_version() == _native.ABI_VERSION
    assert isinstance(lib.lvb_last_error(), bytes)
    for name in _native.PROTOTYPES:
        assert isinstance(getattr(lib, name), ctypes._CFuncPtr)


def test_invalid_arguments_are_rejected_before_any_launch():
    lib = _native.library()
    # m < 0 is rejected by argument validation alone (no device call).
    status = lib.lvb_awq_linear(None, None, None, None, None, None, -1, 128, 128, 32, None, 0, None)
    assert status == _native.LVB_ERR_INVALID
    assert b"invalid AWQ shape" in lib.lvb_last_error()
    with pytest.raises(ValueError, match="invalid AWQ shape"):
        _native.check(status, "lvb_awq_linear")
    status = lib.lvb_paged_attention(None, 0, None, None, None, 0, None, 0, None, None, None, None, None,
                                     None, 1, 1, 1, 1, 1, 4, 4, 8, 16, 1, 1.0, 7, None, 0, None)
    assert status == _native.LVB_ERR_INVALID
    assert b"unknown dtype" in lib.lvb_last_error()


def test_allreduce_workspace_bytes_cover_every_slot():
    """Header + 2*world staging + 2 gather + 3*world sentinel + 3 sentinel gather slots."""

    lib = _native.library()
    for world, tokens, hidden in ((1, 8, 256), (2, 512, 3584), (8, 128, 8192)):
        slot = tokens * hidden * 2
        assert lib.lvb_allreduce_workspace_bytes(world, tokens, hidden) == 65536 + (5 * world + 5) * slot
    assert lib.lvb_allreduce_workspace_bytes(9, 8, 256) == 0
    assert lib.lvb_allreduce_workspace_bytes(2, 0, 256) == 0
