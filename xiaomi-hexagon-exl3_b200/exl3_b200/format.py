"""Host-side EXL3 storage formats (numpy only).

Two layouts describe one k x n EXL3 matrix:

* upstream tensors (ExLlamaV3 / safetensors, src/exl3_model.cpp:79-157):
  ``trellis`` uint16 [k/16][n/16][16*bits], ``suh`` fp16 [k], ``svh`` fp16 [n];
* runtime group records (include/exl3-block.h:14,34-39,
  tools/export_native_gguf.py:27-36): n/128 * k/128 records of
  2048*bits + 512 bytes, record (nb, kb) at index nb*(k/128)+kb holding its 64
  trellis tiles in order r*8+c, then suh[kb*128:+128], then svh[nb*128:+128].
  This is what a ggml EXL3_4/6/8 tensor's data holds.

Both go to the GPU through the C ABI, which converts them to the device
layout; these helpers only move bytes between the two host forms.
"""
from __future__ import annotations

import numpy as np

GROUP = 128
GGML_TYPE_BITS = {43: 4, 44: 6, 45: 8}
BITS_GGML_TYPE = {v: k for k, v in GGML_TYPE_BITS.items()}


def group_bytes(bits: int) -> int:
    return 2048 * bits + 512


def records_nbytes(k: int, n: int, bits: int) -> int:
    return (k // GROUP) * (n // GROUP) * group_bytes(bits)


def _check(k: int, n: int, bits: int) -> None:
    if not (1 <= bits <= 8):
        raise ValueError("EXL3 integer bitrate must be in [1,8]")
    if k <= 0 or n <= 0 or k % GROUP or n % GROUP:
        raise ValueError("k and n must be positive multiples of 128")


def pack_records(trellis: np.ndarray, suh: np.ndarray, svh: np.ndarray, bits: int) -> np.ndarray:
    """Upstream tensors -> runtime records (flat uint8)."""
    trellis = np.ascontiguousarray(trellis, dtype=np.uint16)
    kt, nt, tw = trellis.shape
    k, n = kt * 16, nt * 16
    _check(k, n, bits)
    if tw != 16 * bits:
        raise ValueError("trellis last dimension must be 16*bits")
    kb, nb = k // GROUP, n // GROUP
    tile_words = 16 * bits
    rec_words = group_bytes(bits) // 2
    out = np.empty((nb, kb, rec_words), np.uint16)
    # [kb, r, nb, c, w] -> [nb, kb, r, c, w]
    tiles = trellis.reshape(kb, 8, nb, 8, tile_words).transpose(2, 0, 1, 3, 4)
    out[:, :, :64 * tile_words] = tiles.reshape(nb, kb, 64 * tile_words)
    out[:, :, 64 * tile_words:64 * tile_words + 128] = np.asarray(suh, np.uint16).reshape(1, kb, 128)
    out[:, :, 64 * tile_words + 128:] = np.asarray(svh, np.uint16).reshape(nb, 1, 128)
    return out.reshape(-1).view(np.uint8)


def unpack_records(records: np.ndarray, k: int, n: int, bits: int):
    """Runtime records -> (trellis, suh, svh); scales come from records (0,kb) and (nb,0)."""
    _check(k, n, bits)
    kb, nb = k // GROUP, n // GROUP
    tile_words = 16 * bits
    rec = np.ascontiguousarray(records, np.uint8).view(np.uint16).reshape(nb, kb, group_bytes(bits) // 2)
    tiles = rec[:, :, :64 * tile_words].reshape(nb, kb, 8, 8, tile_words).transpose(1, 2, 0, 3, 4)
    trellis = np.ascontiguousarray(tiles.reshape(k // 16, n // 16, tile_words))
    suh = np.ascontiguousarray(rec[0, :, 64 * tile_words:64 * tile_words + 128].reshape(k))
    svh = np.ascontiguousarray(rec[:, 0, 64 * tile_words + 128:].reshape(n))
    return trellis, suh, svh
