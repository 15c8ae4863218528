"""Build the sm_100a library in-tree: ``python -m light_vllm_b200.build``.

One nvcc invocation compiles ``csrc/lvb200.cu`` (which includes every kernel)
into ``_lib/liblvb200.so`` for ``compute_100a``/``sm_100a`` only, with the CUDA
runtime linked statically so the library does not depend on which libcudart
the host process loaded first.  The small CPython module ``csrc/hostpack.c``
(step metadata read out of Python objects) is compiled by the C compiler into
``_lib/_hostpack<suffix>``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
SOURCE = PACKAGE / "csrc" / "lvb200.cu"
OUTPUT = PACKAGE / "_lib" / "liblvb200.so"
HOSTPACK_SOURCE = PACKAGE / "csrc" / "hostpack.c"
HOSTPACK_OUTPUT = PACKAGE / "_lib" / ("_hostpack" + sysconfig.get_config_var("EXT_SUFFIX"))

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-shared",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "-cudart", "static",
]


def _nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found; the sm_100a library needs the CUDA toolkit (12.8+)")


def sources() -> list[Path]:
    return sorted((PACKAGE / "csrc").glob("*.cu*")) + [PACKAGE.parent / "include" / "lvb200.h"]


def build_hostpack(force: bool = False) -> Path:
    """Compile the CPython step-metadata module if missing or stale."""

    if (not force and HOSTPACK_OUTPUT.is_file()
            and HOSTPACK_OUTPUT.stat().st_mtime >= HOSTPACK_SOURCE.stat().st_mtime):
        return HOSTPACK_OUTPUT
    HOSTPACK_OUTPUT.parent.mkdir(parents=True, exist_ok=True)
    cc = os.environ.get("CC") or shutil.which("gcc") or shutil.which("cc")
    if not cc:
        raise RuntimeError("no C compiler found for csrc/hostpack.c")
    tmp = HOSTPACK_OUTPUT.with_name(HOSTPACK_OUTPUT.name + ".tmp")
    cmd = [cc, "-O2", "-shared", "-fPIC", "-fvisibility=hidden", "-Wall",
           "-I", sysconfig.get_paths()["include"], "-o", str(tmp), str(HOSTPACK_SOURCE)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"{cc} failed ({result.returncode}):\n{result.stderr}")
    os.replace(tmp, HOSTPACK_OUTPUT)
    return HOSTPACK_OUTPUT


def is_stale() -> bool:
    if not OUTPUT.is_file():
        return True
    built = OUTPUT.stat().st_mtime
    return any(src.stat().st_mtime > built for src in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if it is missing or older than its sources."""

    build_hostpack(force)
    if not force and not is_stale():
        return OUTPUT
    OUTPUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUTPUT.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, "-o", str(tmp), str(SOURCE)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    result = subprocess.run(cmd, capture_output=not verbose, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed ({result.returncode}):\n{result.stderr}")
    os.replace(tmp, OUTPUT)
    return OUTPUT


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(path)
