"""Build the sm_100a library in-tree: ``python -m light_vllm_b200.build``.

One nvcc invocation compiles ``csrc/lvb200.cu`` (which includes every kernel)
into ``_lib/liblvb200.so`` for ``compute_100a``/``sm_100a`` only, with the CUDA
runtime linked statically so the library does not depend on which libcudart
the host process loaded first.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
SOURCE = PACKAGE / "csrc" / "lvb200.cu"
OUTPUT = PACKAGE / "_lib" / "liblvb200.so"

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


def is_stale() -> bool:
    if not OUTPUT.is_file():
        return True
    built = OUTPUT.stat().st_mtime
    return any(src.stat().st_mtime > built for src in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if it is missing or older than its sources."""

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
