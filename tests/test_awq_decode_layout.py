"""The packed decode layout of the B200 AWQ scheme, restated by the oracle.

CPU: the oracle's ``pack_decode_layout`` agrees with the layout documented in
``include/lvb200.h`` (decoded here independently, nibble by nibble), pads
partial column tiles and k runs with zeros, and keeps every scale and zero
point.  GPU: ``lvb_awq_pack`` writes the same bytes.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import awq as oawq

# Documented nibble of k offset j (0..31) inside a 16-byte run: (word, nibble).
_NIBBLE = {}
for _w in range(4):
    for _e, _slot in enumerate((0, 4, 2, 6)):
        _NIBBLE[4 * _w + _e] = (_w, _slot)
        _NIBBLE[16 + 4 * _w + _e] = (_w, _slot + 1)


def _decode(codes: np.ndarray, k: int, n: int) -> np.ndarray:
    tiles, runs = codes.shape[:2]
    words = codes.reshape(tiles, runs, 128, 16).view("<u4").reshape(tiles, runs, 128, 4)
    out = np.zeros((runs * 32, tiles * 128), dtype=np.int64)
    for j, (w, nib) in _NIBBLE.items():
        vals = (words[..., w] >> np.uint32(4 * nib)) & np.uint32(0xF)  # [tiles, runs, 128]
        out[j::32, :] = vals.transpose(1, 0, 2).reshape(runs, tiles * 128)
    return out


@pytest.mark.parametrize("k,n,g", [(96, 256, 32), (896, 4864, 128), (512, 2112, 64), (640, 160, 640)])
def test_decode_layout_round_trip(k, n, g):
    qweight, qzeros, scales = oawq.random_checkpoint(k, n, g, seed=k + n)
    codes, groups = oawq.pack_decode_layout(qweight, qzeros, scales, g)
    tiles, runs = -(-n // 128), 2 * (-(-k // 64))
    assert codes.shape == (tiles, runs, 128, 16) and codes.dtype == np.uint8
    assert groups.shape == (tiles, k // g, 128) and groups.dtype == np.uint32
    decoded = _decode(codes, k, n)
    np.testing.assert_array_equal(decoded[:k, :n], oawq.unpack(qweight))
    assert not decoded[k:, :].any() and not decoded[:, n:].any()
    flat = groups.transpose(1, 0, 2).reshape(k // g, tiles * 128)
    np.testing.assert_array_equal((flat[:, :n] & 0xFFFF).astype(np.uint16), scales.view(np.uint16))
    np.testing.assert_array_equal(flat[:, :n] >> 16, oawq.unpack(qzeros))
    assert not flat[:, n:].any()


@pytest.mark.gpu
@pytest.mark.parametrize("k,n,g", [(96, 256, 32), (896, 4864, 128), (512, 2112, 64), (640, 160, 640)])
def test_pack_kernel_matches_oracle(k, n, g):
    import torch

    from light_vllm_b200.awq import pack_awq_decode_layout

    qweight, qzeros, scales = oawq.random_checkpoint(k, n, g, seed=k * 3 + n)
    expected_codes, expected_groups = oawq.pack_decode_layout(qweight, qzeros, scales, g)
    dev = torch.device("cuda:0")
    qw, qz, sc = (torch.from_numpy(a).to(dev) for a in (qweight, qzeros, scales))
    codes, groups = pack_awq_decode_layout(qw, qz, sc, g)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(codes.cpu().numpy(), expected_codes.reshape(-1))
    np.testing.assert_array_equal(groups.cpu().numpy().view(np.uint32), expected_groups.reshape(-1))
