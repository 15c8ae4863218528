"""B200 AWQ W4A16 scheme (drop-in ``AWQScheme``).

``B200AWQScheme().prepare(qweight, qzeros, scales, group_size, bias)`` returns
a ``LinearOperation`` -- the contract of ``AWQScheme.prepare``
(modeling/quantization/awq.py:468-486) and ``LinearOperation.__call__``
(modeling/quantization/interfaces.py:23-26).  It replaces ``CudaAWQScheme`` /
``CudaAWQOperation`` (modeling/quantization/awq_schemes.py:56-73,
cuda_awq.py:96-146) and consumes the same AutoAWQ GEMM tensors.

Ownership: ``prepare`` repacks the int4 codes once, in place, into the
layout the tensor-memory kernel streams (``lvb_awq_pack``; the ``AWQScheme``
protocol leaves one-time conversion to the backend, and a repack replaces the
checkpoint layout rather than adding a second resident copy of the codes,
awq.py:506-535, cuda_awq.py:101-102).  After ``prepare`` the layer's
``qweight`` buffer holds the packed codes; ``qzeros`` and ``scales`` are left
as they are and one (scale, zero) word per group and column is added (1/32 of
the code bytes).  Preparing the same storage again reuses the packing.  Shapes
that do not tile (n % 128 or k % 64 non-zero) keep the checkpoint layout and
run the checkpoint-layout GEMM (``lvb_awq_linear``).

Every call runs one sm_100a kernel on tcgen05 tensor cores with the bias
fused into the epilogue and split-K for small grids, whose workspace is
allocated once here.

Inject it without touching Engine, Scheduler or Worker, e.g.
``AWQLinearMethod(AWQConfig.from_mapping(cfg), B200AWQScheme())`` passed as a
prebuilt ``ModelSpec.linear_method`` (modeling/loaders/safetensors.py:101-102).
"""

from __future__ import annotations

import ctypes
import weakref
from dataclasses import dataclass

import torch
from torch import Tensor

from light_vllm_b200 import _native

_PACK_FACTOR = 8
# Row counts whose fastest plans the prepared split-K workspace covers (one
# per token-tile class); other sizes run the best plan that fits in it.
_SPLIT_K_ROWS = (1, 2, 4, 16, 32, 64, 128, 256)
# Storages already repacked in place: (device index, data_ptr, bytes) -> weak
# reference to a checkpoint tensor over that storage (the model's buffer keeps
# it alive; the entry dies with it).
_PACKED_STORAGES: dict[tuple[int, int, int], weakref.ref] = {}


def _validate_static_weights(qweight: Tensor, qzeros: Tensor, scales: Tensor,
                             group_size: int) -> tuple[int, int]:
    """Same rules and messages as the reference CUDA scheme (cuda_awq.py:53-80),
    except that output widths need only be multiples of 32."""

    if qweight.device.type != "cuda":
        raise ValueError("CUDA AWQ weights must be on CUDA")
    if torch.cuda.get_device_capability(qweight.device) < (10, 0):
        raise ValueError("B200 AWQ requires compute capability 10.0 (sm_100a)")
    if qweight.dtype != torch.int32 or qzeros.dtype != torch.int32:
        raise ValueError("CUDA AWQ packed weights and zeros must use int32")
    if scales.dtype != torch.float16:
        raise ValueError("CUDA AWQ first-stage scales must use float16")
    if any(t.device != qweight.device for t in (qzeros, scales)):
        raise ValueError("CUDA AWQ tensors must share one CUDA device")
    if not all(t.is_contiguous() for t in (qweight, qzeros, scales)):
        raise ValueError("CUDA AWQ checkpoint tensors must be contiguous")
    inner = qweight.shape[0]
    output = qweight.shape[1] * _PACK_FACTOR
    if group_size <= 0 or inner % group_size or group_size % 32:
        raise ValueError("CUDA AWQ group_size must divide K and be a multiple of 32")
    if output % 32:
        raise ValueError("CUDA AWQ output width must be divisible by 32")
    expected = (inner // group_size, output // _PACK_FACTOR)
    if tuple(qzeros.shape) != expected or tuple(scales.shape) != (expected[0], output):
        raise ValueError("CUDA AWQ qzeros/scales do not match qweight and group_size")
    return inner, output


@dataclass(frozen=True, slots=True)
class B200AWQOperation:
    """A prepared W4A16 linear over the model-owned AutoAWQ tensors."""

    qweight: Tensor
    qzeros: Tensor
    scales: Tensor
    group_size: int
    bias: Tensor | None
    inner: int
    output_width: int
    workspace: Tensor
    codes: Tensor | None   # packed codes (a view of qweight's storage), or None
    groups: Tensor | None  # packed (scale, zero) words, or None

    def __call__(self, inputs: Tensor) -> Tensor:
        flat = inputs.reshape(-1, self.inner)
        if flat.dtype != torch.float16:
            raise ValueError("B200 AWQ activations must be float16")
        if not flat.is_contiguous() or flat.data_ptr() % 16:
            flat = flat.contiguous()
        rows = flat.shape[0]
        out = torch.empty((rows, self.output_width), dtype=torch.float16, device=flat.device)
        if self.codes is not None:
            _native.check(
                _native.library().lvb_awq_linear_packed(
                    flat.data_ptr(), self.codes.data_ptr(), self.groups.data_ptr(),
                    None if self.bias is None else self.bias.data_ptr(), out.data_ptr(), rows,
                    self.inner, self.output_width, self.group_size, self.workspace.data_ptr(),
                    self.workspace.numel(), _native.stream_handle(flat.device),
                ),
                "lvb_awq_linear_packed",
            )
            return out.reshape(*inputs.shape[:-1], self.output_width)
        _native.check(
            _native.library().lvb_awq_linear(
                flat.data_ptr(), self.qweight.data_ptr(), self.qzeros.data_ptr(),
                self.scales.data_ptr(), None if self.bias is None else self.bias.data_ptr(),
                out.data_ptr(), rows, self.inner, self.output_width, self.group_size,
                self.workspace.data_ptr(), self.workspace.numel(),
                _native.stream_handle(flat.device),
            ),
            "lvb_awq_linear",
        )
        return out.reshape(*inputs.shape[:-1], self.output_width)

    def qkv_rope(self, inputs: Tensor, positions: Tensor, cos: Tensor, sin: Tensor, kv_args: tuple,
                 q_heads: int, kv_heads: int, head_size: int) -> Tensor | None:
        """The merged QKV projection with its decode epilogue in one launch
        (``lvb_awq_qkv_rope_packed``): RoPE on the query heads of the output,
        rotated keys and the values written to the tokens' paged cache slots.
        ``kv_args`` = (key_cache, value_cache, block_tables, table_stride,
        num_computed, query_start_loc, request_indices, block_size) as device
        addresses.  Returns None when the shape is not covered (the caller
        then runs the projection and ``lvb_rope_kv_write``)."""

        if self.codes is None:
            return None
        flat = inputs.reshape(-1, self.inner)
        if flat.dtype != torch.float16:
            raise ValueError("B200 AWQ activations must be float16")
        if not flat.is_contiguous() or flat.data_ptr() % 16:
            flat = flat.contiguous()
        rows = flat.shape[0]
        out = torch.empty((rows, self.output_width), dtype=torch.float16, device=flat.device)
        kc, vc, tables, stride, computed, qsl, req, block_size = kv_args
        status = _native.library().lvb_awq_qkv_rope_packed(
            flat.data_ptr(), self.codes.data_ptr(), self.groups.data_ptr(),
            None if self.bias is None else self.bias.data_ptr(), out.data_ptr(), rows, self.inner,
            self.output_width, self.group_size, self.workspace.data_ptr(), self.workspace.numel(),
            positions.data_ptr(), cos.data_ptr(), sin.data_ptr(), cos.shape[0], kc, vc, tables, stride, computed,
            qsl, req, q_heads, kv_heads, head_size, block_size, _native.stream_handle(flat.device))
        if status == _native.LVB_ERR_UNSUPPORTED:
            return None
        _native.check(status, "lvb_awq_qkv_rope_packed")
        return out

    def silu_mul_linear(self, gate_up: Tensor) -> Tensor:
        """``self(silu(gate) * up)`` for merged [gate | up] rows of 2 x inner
        values (the Qwen2 MLP's down projection after ``silu_and_mul``,
        qwen2.py:237-247).  Decode batches run the SiLU-mul inside the
        projection's activation prologue (``lvb_awq_silu_linear_packed``);
        other shapes run ``lvb_silu_mul`` and then the projection."""

        flat = gate_up.reshape(-1, 2 * self.inner)
        if flat.dtype != torch.float16:
            raise ValueError("B200 AWQ activations must be float16")
        if not flat.is_contiguous() or flat.data_ptr() % 16:
            flat = flat.contiguous()
        rows = flat.shape[0]
        lib = _native.library()
        stream = _native.stream_handle(flat.device)
        if self.codes is not None:
            out = torch.empty((rows, self.output_width), dtype=torch.float16, device=flat.device)
            status = lib.lvb_awq_silu_linear_packed(
                flat.data_ptr(), flat.stride(0), self.codes.data_ptr(), self.groups.data_ptr(),
                None if self.bias is None else self.bias.data_ptr(), out.data_ptr(), rows, self.inner,
                self.output_width, self.group_size, self.workspace.data_ptr(), self.workspace.numel(), stream)
            if status == _native.LVB_OK:
                return out.reshape(*gate_up.shape[:-1], self.output_width)
            if status != _native.LVB_ERR_UNSUPPORTED:
                _native.check(status, "lvb_awq_silu_linear_packed")
        act = torch.empty((rows, self.inner), dtype=torch.float16, device=flat.device)
        _native.check(lib.lvb_silu_mul(flat.data_ptr(), flat.stride(0), rows, self.inner, act.data_ptr(),
                                       act.stride(0), stream), "lvb_silu_mul")
        return self(act).reshape(*gate_up.shape[:-1], self.output_width)


def prepare_b200_awq_operation(qweight: Tensor, qzeros: Tensor, scales: Tensor, group_size: int,
                               bias: Tensor | None) -> B200AWQOperation:
    inner, output = _validate_static_weights(qweight, qzeros, scales, group_size)
    if bias is not None and (bias.device != qweight.device or bias.dtype != scales.dtype
                             or tuple(bias.shape) != (output,)):
        raise ValueError("CUDA AWQ bias must match output width, dtype, and device")
    if bias is not None and not bias.is_contiguous():
        bias = bias.contiguous()
    lib = _native.library()
    with torch.cuda.device(qweight.device):
        need = max(int(lib.lvb_awq_workspace_bytes(m, inner, output, group_size)) for m in _SPLIT_K_ROWS)
        # Split-K semaphores must start at zero; every call leaves them zero.
        workspace = torch.zeros(max(need, 256), dtype=torch.uint8, device=qweight.device)
        codes = groups = None
        if output % 128 == 0 and inner % 64 == 0:
            codes, groups = _pack_in_place(qweight, qzeros, scales, group_size)
    return B200AWQOperation(qweight, qzeros, scales, group_size, bias, inner, output, workspace, codes,
                            groups)


def _pack_in_place(qweight: Tensor, qzeros: Tensor, scales: Tensor,
                   group_size: int) -> tuple[Tensor, Tensor]:
    """Replace ``qweight``'s contents by the packed codes (same byte size when
    n % 128 == 0 and k % 64 == 0) and return (codes view, group words)."""

    key = (qweight.device.index or 0, qweight.data_ptr(), qweight.numel() * qweight.element_size())
    ref = _PACKED_STORAGES.get(key)
    already = ref is not None and ref() is not None
    codes, groups = pack_awq_decode_layout(qweight, qzeros, scales, group_size)
    target = qweight.view(torch.uint8).reshape(-1)
    if already:
        return target, groups  # repacked earlier: the fresh codes read packed bytes
    if target.numel() != codes.numel():
        raise ValueError("packed AWQ codes must have the checkpoint's byte size")
    target.copy_(codes)
    _PACKED_STORAGES[key] = weakref.ref(qweight, lambda _r, k=key: _PACKED_STORAGES.pop(k, None))
    return target, groups


def pack_awq_decode_layout(qweight: Tensor, qzeros: Tensor, scales: Tensor,
                           group_size: int) -> tuple[Tensor, Tensor]:
    """Packed codes and (scale, zero) words (``lvb_awq_pack``) in new buffers;
    the checkpoint tensors are left untouched."""

    inner, output = _validate_static_weights(qweight, qzeros, scales, group_size)
    lib = _native.library()
    codes_bytes = ctypes.c_size_t()
    groups_bytes = ctypes.c_size_t()
    _native.check(lib.lvb_awq_pack_bytes(inner, output, group_size, ctypes.byref(codes_bytes),
                                         ctypes.byref(groups_bytes)), "lvb_awq_pack_bytes")
    codes = torch.empty(codes_bytes.value, dtype=torch.uint8, device=qweight.device)
    groups = torch.empty(groups_bytes.value // 4, dtype=torch.int32, device=qweight.device)
    _native.check(
        lib.lvb_awq_pack(qweight.data_ptr(), qzeros.data_ptr(), scales.data_ptr(), inner, output,
                         group_size, codes.data_ptr(), groups.data_ptr(),
                         _native.stream_handle(qweight.device)),
        "lvb_awq_pack",
    )
    return codes, groups


class B200AWQScheme:
    """AWQ Scheme whose operations run the sm_100a W4A16 kernel."""

    name = "b200"

    def __init__(self) -> None:
        _native.library()  # fail loudly when the library is missing

    def prepare(self, qweight: Tensor, qzeros: Tensor, scales: Tensor, group_size: int,
                bias: Tensor | None) -> B200AWQOperation:
        return prepare_b200_awq_operation(qweight, qzeros, scales, group_size, bias)


def b200_awq_linear(inputs: Tensor, qweight: Tensor, qzeros: Tensor, scales: Tensor,
                    group_size: int, bias: Tensor | None) -> Tensor:
    """One-shot entry for tests and microbenchmarks (mirrors cuda_awq.py:245-255)."""

    return prepare_b200_awq_operation(qweight, qzeros, scales, group_size, bias)(inputs)


def b200_awq_dequantize(qweight: Tensor, qzeros: Tensor, scales: Tensor, group_size: int) -> Tensor:
    """Full fp16 weight [K, N] (the reference's ``awq_dequantize``)."""

    inner, output = _validate_static_weights(qweight, qzeros, scales, group_size)
    w = torch.empty((inner, output), dtype=torch.float16, device=qweight.device)
    _native.check(
        _native.library().lvb_awq_dequantize(
            qweight.data_ptr(), qzeros.data_ptr(), scales.data_ptr(), w.data_ptr(), inner, output,
            group_size, _native.stream_handle(qweight.device),
        ),
        "lvb_awq_dequantize",
    )
    return w
