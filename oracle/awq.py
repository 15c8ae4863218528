"""CPU restatement of the reference's AutoAWQ W4A16 arithmetic (test oracle).

TEST INFRASTRUCTURE ONLY -- see ``oracle/__init__.py``.  Each function names
the reference source it restates (paths relative to the light-vllm source
tree).  Integer packing is done with numpy; the floating-point parts use torch
on the CPU so that fp16 rounding is identical to the reference's Torch scheme.

AutoAWQ GEMM layout (``modeling/quantization/awq.py:26-32``):
  qweight int32 [K, N/8]; qzeros int32 [K/G, N/8]; scales fp16 [K/G, N].
  Nibble p (bits 4p..4p+3) of a packed word holds natural column
  8*j + PACK_ORDER[p] with PACK_ORDER = (0, 2, 4, 6, 1, 3, 5, 7).
"""

from __future__ import annotations

import numpy as np
import torch

BITS = 4
PACK_FACTOR = 32 // BITS
# modeling/quantization/awq.py:31 -- the order in which natural columns of an
# 8-column group occupy nibbles 0..7 of one int32 word.
PACK_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)
# Inverse permutation: nibble index that holds natural column c.
NIBBLE_OF_COLUMN = tuple(PACK_ORDER.index(c) for c in range(PACK_FACTOR))


def pack(values: np.ndarray) -> np.ndarray:
    """Pack uint4 values [R, C] into AutoAWQ int32 words [R, C/8].

    Restates ``pack_awq`` (modeling/quantization/awq.py:329-341).
    """

    values = np.asarray(values)
    if values.ndim != 2 or values.shape[1] % PACK_FACTOR:
        raise ValueError("AWQ values must be a 2D array with a multiple-of-8 width")
    if values.size and (values.min() < 0 or values.max() > 15):
        raise ValueError("AWQ packed values must stay within uint4 range")
    groups = values.astype(np.uint32).reshape(values.shape[0], -1, PACK_FACTOR)
    words = np.zeros(groups.shape[:2], dtype=np.uint32)
    for nibble, column in enumerate(PACK_ORDER):
        words |= groups[..., column] << np.uint32(BITS * nibble)
    return words.view(np.int32)


def unpack(packed: np.ndarray) -> np.ndarray:
    """Unpack AutoAWQ int32 words [R, C/8] into natural-order uint4 [R, C].

    Restates ``unpack_awq`` (modeling/quantization/awq.py:318-326).
    """

    packed = np.asarray(packed)
    if packed.dtype != np.int32 or packed.ndim != 2:
        raise ValueError("packed AWQ tensors must be two-dimensional int32")
    words = packed.view(np.uint32)
    out = np.empty((packed.shape[0], packed.shape[1], PACK_FACTOR), dtype=np.int32)
    for column in range(PACK_FACTOR):
        shift = np.uint32(BITS * NIBBLE_OF_COLUMN[column])
        out[..., column] = ((words >> shift) & np.uint32(0xF)).astype(np.int32)
    return out.reshape(packed.shape[0], packed.shape[1] * PACK_FACTOR)


def dequantize(
    qweight: np.ndarray,
    qzeros: np.ndarray,
    scales: np.ndarray,
    group_size: int,
) -> np.ndarray:
    """Return fp16 W[K, N] = fp16(q - z) * s with one fp16 rounding.

    Restates ``dequantize_awq`` (modeling/quantization/awq.py:433-450): the
    integer difference converts to fp16 exactly and the product with the fp16
    scale is rounded once (numpy float16 multiply rounds to nearest even, as
    torch's CPU and CUDA half multiplies do).
    """

    qweight = np.asarray(qweight)
    if group_size <= 0 or qweight.shape[0] % group_size:
        raise ValueError("AWQ group_size must divide the packed input dimension")
    weights = unpack(qweight)
    zeros = unpack(np.asarray(qzeros))
    scales = np.asarray(scales, dtype=np.float16)
    groups = qweight.shape[0] // group_size
    if zeros.shape != (groups, weights.shape[1]) or scales.shape != zeros.shape:
        raise ValueError("AWQ qzeros/scales do not match qweight and group_size")
    group_ids = np.arange(qweight.shape[0]) // group_size
    diff = (weights - zeros[group_ids]).astype(np.float16)
    return (diff * scales[group_ids]).astype(np.float16)


def linear_fp32(
    inputs: np.ndarray,
    qweight: np.ndarray,
    qzeros: np.ndarray,
    scales: np.ndarray,
    group_size: int,
    bias: np.ndarray | None,
) -> np.ndarray:
    """fp32-accumulated reference y = x @ W (+ bias), returned as float64.

    The reference's Torch scheme (``_torch_awq_linear``,
    modeling/quantization/awq.py:453-465) multiplies the fp16 activations by
    the fp16 dequantised weight; this is the same product accumulated exactly
    (float64) so kernels can be judged against it with max-abs / rel-L2.
    """

    w = dequantize(qweight, qzeros, scales, group_size).astype(np.float64)
    x = np.asarray(inputs, dtype=np.float16).astype(np.float64)
    y = x.reshape(-1, w.shape[0]) @ w
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float16).astype(np.float64)
    return y.reshape(*np.asarray(inputs).shape[:-1], w.shape[1])


def linear_exact_weight(
    inputs: np.ndarray,
    qweight: np.ndarray,
    qzeros: np.ndarray,
    scales: np.ndarray,
    group_size: int,
    bias: np.ndarray | None,
) -> tuple[np.ndarray, np.ndarray]:
    """Not a reference function: the same product with the unrounded weight
    (q - z) * s (float64), and sum_k |x_k W_k| with the reference's fp16 W.

    The reference rounds W to fp16 before the product
    (modeling/quantization/awq.py:433-450); a kernel that applies the zero
    point and scale exactly (the integer-limb decode paths) differs from it
    by at most 2^-11 * sum_k |x_k W_k| (half an fp16 ulp per weight).  Tests
    use the first array to check such a kernel's own arithmetic and the second
    to bound its distance from the reference.  Returns (y_exact, abs_sum).
    """

    codes = unpack(np.asarray(qweight)).astype(np.float64)
    zeros = unpack(np.asarray(qzeros)).astype(np.float64)
    group_ids = np.arange(codes.shape[0]) // group_size
    w = (codes - zeros[group_ids]) * np.asarray(scales, dtype=np.float16).astype(np.float64)[group_ids]
    x = np.asarray(inputs, dtype=np.float16).astype(np.float64).reshape(-1, w.shape[0])
    y = x @ w
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float16).astype(np.float64)
    w16 = dequantize(qweight, qzeros, scales, group_size).astype(np.float64)
    return y, np.abs(x) @ np.abs(w16)


def torch_linear(
    inputs: torch.Tensor,
    qweight: torch.Tensor,
    qzeros: torch.Tensor,
    scales: torch.Tensor,
    group_size: int,
    bias: torch.Tensor | None,
) -> torch.Tensor:
    """The reference Torch scheme's call, restated with torch CPU ops.

    ``_torch_awq_linear`` (modeling/quantization/awq.py:453-465): dequantise the
    full W, ``torch.matmul`` in the activation dtype, then add the bias.  Used as
    the timed CPU baseline.
    """

    words = qweight.view(torch.int32)
    shifts = torch.tensor([BITS * n for n in NIBBLE_OF_COLUMN], dtype=torch.int32)
    q = (words.unsqueeze(-1) >> shifts) & 0xF
    q = q.reshape(words.shape[0], -1)
    z = (qzeros.unsqueeze(-1) >> shifts) & 0xF
    z = z.reshape(qzeros.shape[0], -1)
    group_ids = torch.arange(words.shape[0]) // group_size
    w = (q - z[group_ids]).to(scales.dtype) * scales[group_ids]
    out = torch.matmul(inputs, w.to(inputs.dtype))
    if bias is not None:
        out = out + bias
    return out


def quantize_groups(weight: torch.Tensor, group_size: int):
    """Asymmetric int4 quantisation of a [out, in] weight along ``in``.

    Restates ``_quantize_awq_groups`` (modeling/quantization/awq.py:363-384):
    per group the fp16-rounded scale is (max - min).clamp_min(1e-5) / 15, the
    zero point round(-min / scale) and the code round(w / scale + zero), both
    clamped to [0, 15].
    """

    width = weight.shape[-1]
    size = width if group_size == -1 else group_size
    if size <= 0 or width % size:
        raise ValueError("AWQ group_size must divide the weight input dimension")
    grouped = weight.float().reshape(*weight.shape[:-1], -1, size)
    lo = grouped.amin(dim=-1, keepdim=True)
    hi = grouped.amax(dim=-1, keepdim=True)
    scale = ((hi - lo).clamp_min(1e-5) / 15).to(weight.dtype)
    fscale = scale.float()
    zero = torch.round(-lo / fscale).clamp_(0, 15).to(torch.int32)
    code = torch.round(grouped / fscale + zero).clamp_(0, 15).to(torch.int32)
    return code, zero, scale


def quantize_weight(weight: torch.Tensor, group_size: int):
    """Quantise an ``nn.Linear``-style [out, in] weight into the AutoAWQ layout.

    Restates ``pack_awq_checkpoint_weight`` + ``quantize_awq_weight``
    (modeling/quantization/awq.py:387-430).  Returns numpy arrays
    ``(qweight [in, out/8], qzeros [in/G, out/8], scales fp16 [in/G, out],
    dequantized fp16 [out, in])``.
    """

    out_features, in_features = weight.shape
    size = in_features if group_size == -1 else group_size
    if out_features % PACK_FACTOR:
        raise ValueError("AWQ weight output dimension must be divisible by 8")
    code, zero, scale = quantize_groups(weight, size)
    natural_q = code.reshape(weight.shape).t().contiguous().numpy()
    natural_z = zero.squeeze(-1).t().contiguous().numpy()
    scales = scale.squeeze(-1).t().contiguous().to(torch.float16).numpy()
    qweight = pack(natural_q)
    qzeros = pack(natural_z)
    deq = dequantize(qweight, qzeros, scales, size).T.copy()
    return qweight, qzeros, scales, deq


def random_checkpoint(k: int, n: int, group_size: int, *, seed: int,
                      scale_lo: float = 0.002, scale_hi: float = 0.02):
    """Seeded synthetic AWQ tensors with BASELINE config-1 distributions.

    int4 codes and zero points uniform in 0..15, packed with ``pack``; fp16
    scales uniform in [scale_lo, scale_hi].  Returns numpy
    ``(qweight, qzeros, scales)``.
    """

    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 16, size=(k, n), dtype=np.int64)
    zeros = rng.integers(0, 16, size=(k // group_size, n), dtype=np.int64)
    scales = rng.uniform(scale_lo, scale_hi, size=(k // group_size, n)).astype(np.float16)
    return pack(codes), pack(zeros), scales


def error_metrics(actual: np.ndarray, expected: np.ndarray) -> tuple[float, float]:
    """(max-abs error, relative L2 error) of ``actual`` against ``expected``."""

    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    diff = a - e
    max_abs = float(np.max(np.abs(diff))) if diff.size else 0.0
    denom = float(np.linalg.norm(e))
    rel_l2 = float(np.linalg.norm(diff) / denom) if denom > 0 else float(np.linalg.norm(diff))
    return max_abs, rel_l2


# Nibble slot of k offset e (0..3) within a 4-k quad of the packed decode
# layout's lower half; the upper half (k + 16) uses the next nibble.
_DECODE_SLOT = (0, 4, 2, 6)


def pack_decode_layout(qweight: np.ndarray, qzeros: np.ndarray, scales: np.ndarray,
                       group_size: int) -> tuple[np.ndarray, np.ndarray]:
    """The B200 decode layout (``lvb_awq_pack``), restated with numpy.

    Not a reference function: this is the layout the B200 scheme converts the
    AutoAWQ checkpoint into once at ``AWQScheme.prepare`` time
    (``modeling/quantization/awq.py:468-486``).  Used only to check the pack
    kernel bit for bit.  Returns ``(codes uint8 [tiles, runs, 128, 16],
    groups uint32 [tiles, K/G, 128])``.
    """

    codes = unpack(qweight)  # [K, N] natural order
    zeros = unpack(qzeros)   # [K/G, N]
    k, n = codes.shape
    tiles = -(-n // 128)
    runs = 2 * (-(-k // 64))
    padded = np.zeros((runs * 32, tiles * 128), dtype=np.uint32)
    padded[:k, :n] = codes
    # [tiles, 128 cols, runs, 32 k]
    per_col = padded.reshape(runs, 32, tiles, 128).transpose(2, 3, 0, 1)
    words = np.zeros((tiles, 128, runs, 4), dtype=np.uint32)
    for w in range(4):
        for e in range(4):
            words[..., w] |= per_col[..., 4 * w + e] << (4 * _DECODE_SLOT[e])
            words[..., w] |= per_col[..., 16 + 4 * w + e] << (4 * (_DECODE_SLOT[e] + 1))
    packed_codes = words.transpose(0, 2, 1, 3).astype("<u4").view(np.uint8).reshape(tiles, runs, 128, 16)

    groups = k // group_size
    scale_bits = np.zeros((groups, tiles * 128), dtype=np.uint32)
    scale_bits[:, :n] = np.asarray(scales, dtype=np.float16).view(np.uint16)
    zero_vals = np.zeros((groups, tiles * 128), dtype=np.uint32)
    zero_vals[:, :n] = zeros
    words_g = scale_bits | (zero_vals << 16)
    packed_groups = words_g.reshape(groups, tiles, 128).transpose(1, 0, 2).copy()
    return packed_codes, packed_groups
