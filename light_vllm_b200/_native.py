"""ctypes binding of the sm_100a library ``_lib/liblvb200.so`` (C ABI in
``include/lvb200.h``).

There is no fallback: if the library is missing or cannot be loaded, every
entry point raises ``RuntimeError`` naming the build command.  Status codes map
to the exception types the reference uses at the same boundary
(``modeling/quantization/cuda_awq.py:53-80`` raises ``ValueError`` for bad
shapes, ``RuntimeError`` for toolchain/runtime failures).
"""

from __future__ import annotations

import ctypes
import functools
import importlib.machinery
import importlib.util
import sysconfig
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "liblvb200.so"
HOSTPACK_PATH = Path(__file__).resolve().parent / "_lib" / ("_hostpack" + sysconfig.get_config_var("EXT_SUFFIX"))
ABI_VERSION = 8

LVB_OK = 0
LVB_ERR_INVALID = 1
LVB_ERR_UNSUPPORTED = 2
LVB_ERR_CUDA = 3
LVB_ERR_WORKSPACE = 4
LVB_ERR_METADATA = 5

DTYPE_F16 = 0
DTYPE_BF16 = 1

_c_ptr = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_size = ctypes.c_size_t
_f32 = ctypes.c_float

# name -> (restype, argtypes); every symbol declared in include/lvb200.h.
PROTOTYPES: dict[str, tuple[object, tuple[object, ...]]] = {
    "lvb_abi_version": (_int, ()),
    "lvb_last_error": (ctypes.c_char_p, ()),
    "lvb_device_error": (_int, (ctypes.POINTER(ctypes.c_uint32),)),
    "lvb_awq_workspace_bytes": (_size, (_i64, _i64, _i64, _i64)),
    "lvb_awq_linear": (
        _int,
        (_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _i64, _i64, _i64, _i64, _c_ptr, _size, _c_ptr),
    ),
    "lvb_awq_linear_static": (
        _int, (_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _i64, _i64, _i64, _i64, _c_ptr),
    ),
    "lvb_awq_dequantize": (_int, (_c_ptr, _c_ptr, _c_ptr, _c_ptr, _i64, _i64, _i64, _c_ptr)),
    "lvb_awq_pack_bytes": (_int, (_i64, _i64, _i64, ctypes.POINTER(_size), ctypes.POINTER(_size))),
    "lvb_awq_pack": (_int, (_c_ptr, _c_ptr, _c_ptr, _i64, _i64, _i64, _c_ptr, _c_ptr, _c_ptr)),
    "lvb_awq_linear_packed": (
        _int, (_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _i64, _i64, _i64, _i64, _c_ptr, _size, _c_ptr),
    ),
    "lvb_awq_qkv_rope_packed": (
        _int,
        (_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _i64, _i64, _i64, _i64, _c_ptr, _size, _c_ptr, _c_ptr, _c_ptr,
         _i64, _c_ptr, _c_ptr, _c_ptr, _i64, _c_ptr, _c_ptr, _c_ptr, _i64, _i64, _i64, _i64, _c_ptr),
    ),
    "lvb_awq_silu_linear_packed": (
        _int,
        (_c_ptr, _i64, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _i64, _i64, _i64, _i64, _c_ptr, _size, _c_ptr),
    ),
    "lvb_paged_kv_write": (
        _int,
        (_c_ptr, _i64, _c_ptr, _i64, _c_ptr, _c_ptr, _c_ptr, _i64, _c_ptr, _c_ptr, _c_ptr, _i64, _i64,
         _i64, _i64, _int, _c_ptr),
    ),
    "lvb_kv_scatter": (
        _int,
        (_c_ptr, _i64, _c_ptr, _i64, _c_ptr, _c_ptr, _c_ptr, _i64, _i64, _i64, _i64, _int, _c_ptr),
    ),
    "lvb_kv_compact_plan": (
        _int, (_c_ptr, _i64, _c_ptr, _c_ptr, _i64, _i64, _i64, _c_ptr, _c_ptr, ctypes.POINTER(_i64)),
    ),
    "lvb_kv_move_rows": (_int, (_c_ptr, _c_ptr, _c_ptr, _c_ptr, _i64, _i64, _i64, _i64, _int, _c_ptr)),
    "lvb_paged_attention_workspace_bytes": (_size, (_i64, _i64, _i64, _i64, _i64)),
    "lvb_pack_step_metadata": (
        _int,
        (_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _i64, _i64, _i64, _c_ptr, _i64,
         ctypes.POINTER(_i64), ctypes.POINTER(_i64)),
    ),
    "lvb_stage_step_metadata": (
        _int,
        (_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _i64, _i64, _i64, _c_ptr, _i64, _c_ptr, _i64,
         _c_ptr, _c_ptr, ctypes.POINTER(_i64), ctypes.POINTER(_i64)),
    ),
    "lvb_event_create": (_int, (ctypes.POINTER(_c_ptr),)),
    "lvb_event_destroy": (_int, (_c_ptr,)),
    "lvb_event_record": (_int, (_c_ptr, _c_ptr)),
    "lvb_event_wait_host": (_int, (_c_ptr,)),
    "lvb_stream_wait_event": (_int, (_c_ptr, _c_ptr)),
    "lvb_copy_async": (_int, (_c_ptr, _c_ptr, _size, _c_ptr)),
    "lvb_ipc_alloc": (_int, (_size, ctypes.POINTER(_c_ptr), _c_ptr)),
    "lvb_ipc_open": (_int, (_c_ptr, ctypes.POINTER(_c_ptr))),
    "lvb_ipc_close": (_int, (_c_ptr,)),
    "lvb_ipc_free": (_int, (_c_ptr,)),
    "lvb_allreduce_workspace_bytes": (_size, (_int, _i64, _i64)),
    "lvb_allreduce_workspace_init": (_int, (_c_ptr, _int, _i64, _i64)),
    "lvb_allreduce_peer_max_bytes": (_size, (_int,)),
    "lvb_allreduce_add_rmsnorm": (
        _int,
        (_c_ptr, _int, _int, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _i64, _i64, _i64, _f32, _int, _c_ptr),
    ),
    "lvb_rope_qk": (
        _int,
        (_c_ptr, _i64, _i64, _i64, _i64, _i64, _c_ptr, _c_ptr, _c_ptr, _i64, _c_ptr),
    ),
    "lvb_silu_mul": (_int, (_c_ptr, _i64, _i64, _i64, _c_ptr, _i64, _c_ptr)),
    "lvb_lm_head_workspace_bytes": (_size, ()),
    "lvb_lm_head_argmax": (
        _int, (_c_ptr, _i64, _i64, _c_ptr, _i64, _i64, _i64, _c_ptr, _c_ptr, _c_ptr, _c_ptr),
    ),
    "lvb_embedding": (_int, (_c_ptr, _i64, _c_ptr, _i64, _i64, _i64, _c_ptr, _i64, _c_ptr)),
    "lvb_rope_kv_write": (
        _int,
        (_c_ptr, _i64, _i64, _i64, _i64, _i64, _c_ptr, _c_ptr, _c_ptr, _i64, _c_ptr, _c_ptr, _c_ptr, _i64, _c_ptr,
         _c_ptr, _c_ptr, _i64, _c_ptr),
    ),
    "lvb_paged_attention": (
        _int,
        (_c_ptr, _i64, _c_ptr, _c_ptr, _c_ptr, _i64, _c_ptr, _i64, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr,
         _c_ptr, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _int, _c_ptr, _size,
         _c_ptr),
    ),
    "lvb_paged_attention_kv": (
        _int,
        (_c_ptr, _i64, _c_ptr, _i64, _c_ptr, _i64, _c_ptr, _c_ptr, _c_ptr, _i64, _c_ptr, _i64, _c_ptr, _c_ptr,
         _c_ptr, _c_ptr, _c_ptr, _c_ptr, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _int,
         _c_ptr, _size, _c_ptr),
    ),
}


class NativeLibraryError(RuntimeError):
    """The sm_100a library is missing, stale or failed to load."""


@functools.lru_cache(maxsize=1)
def library() -> ctypes.CDLL:
    """Load the library once and declare every prototype; raise if absent."""

    if not LIB_PATH.is_file():
        raise NativeLibraryError(
            f"{LIB_PATH} is not built; run `python -m light_vllm_b200.build` (needs nvcc 12.8+)"
        )
    try:
        lib = ctypes.CDLL(str(LIB_PATH))
    except OSError as exc:
        raise NativeLibraryError(f"cannot load {LIB_PATH}: {exc}") from exc
    for name, (restype, argtypes) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = list(argtypes)
    version = lib.lvb_abi_version()
    if version != ABI_VERSION:
        raise NativeLibraryError(f"{LIB_PATH} has ABI {version}, expected {ABI_VERSION}; rebuild it")
    return lib


def stream_handle(device) -> int:
    """The raw ``cudaStream_t`` of the current stream on ``device`` (what
    ``torch.cuda.current_stream(device).cuda_stream`` returns, without
    building a Stream object: ~0.1 instead of ~2 us per call)."""

    index = device.index
    if index is None:
        import torch

        index = torch.cuda.current_device()
    return _raw_stream(index)


def _raw_stream(index: int) -> int:
    import torch

    return torch._C._cuda_getCurrentRawStream(index)


@functools.lru_cache(maxsize=1)
def hostpack():
    """The CPython module that reads step metadata out of Python objects."""

    if not HOSTPACK_PATH.is_file():
        raise NativeLibraryError(f"{HOSTPACK_PATH} is not built; run `python -m light_vllm_b200.build`")
    loader = importlib.machinery.ExtensionFileLoader("light_vllm_b200._hostpack", str(HOSTPACK_PATH))
    spec = importlib.util.spec_from_file_location("light_vllm_b200._hostpack", str(HOSTPACK_PATH), loader=loader)
    module = importlib.util.module_from_spec(spec)
    loader.exec_module(module)
    # The call trampolines reach the library's entry points directly.
    lib = library()
    module.bind(*(ctypes.cast(getattr(lib, name), ctypes.c_void_p).value
                  for name in ("lvb_paged_kv_write", "lvb_paged_attention", "lvb_stage_step_metadata",
                               "lvb_paged_attention_kv")))
    return module


def check(status: int, what: str) -> None:
    """Raise the exception type matching a non-zero C status."""

    if status == LVB_OK:
        return
    message = library().lvb_last_error().decode(errors="replace")
    text = f"{what}: {message}"
    if status == LVB_ERR_METADATA:
        from light_vllm_b200.kv_cache import KVCacheError

        raise KVCacheError(message)
    if status in (LVB_ERR_INVALID, LVB_ERR_UNSUPPORTED, LVB_ERR_WORKSPACE):
        raise ValueError(text)
    raise RuntimeError(text)


def device_error() -> int:
    """Read and clear the device-side error word (synchronises the device)."""

    value = ctypes.c_uint32(0)
    check(library().lvb_device_error(ctypes.byref(value)), "lvb_device_error")
    return int(value.value)
