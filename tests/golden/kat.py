"""Deterministic known-answer inputs shared by the golden generator and the tests.

The patterns follow the reference's own device probe and graph test:

* packed trellis words: a xorshift32 stream (x ^= x<<13; x ^= x>>17; x ^= x<<5)
  seeded with 0x78ef12ab, k=256, n=384 -- tools/exl3_npu_probe.cpp:20-21, 86-91.
  Here the stream restarts at the seed for each bitrate so every case is
  independently reproducible.
* channel scales suh[i] = fp16((i%7-3)/7), svh[i] = fp16((i%9-4)/9)
  -- tools/exl3_npu_probe.cpp:118-120.
* activations x[i] = ((i*13)%17 - 8)/17 -- tests/test-exl3-graph.cpp:71.
* H128 probe blocks: zero, impulse, ones, alternating signs, then scaled
  xorshift noise -- tools/exl3_npu_probe.cpp:24-31.
"""
from __future__ import annotations

import numpy as np

KAT_SEED = 0x78EF12AB
KAT_K, KAT_N = 256, 384


def xorshift32_stream(count: int, seed: int = KAT_SEED) -> tuple[np.ndarray, int]:
    out = np.empty(count, np.uint32)
    x = seed & 0xFFFFFFFF
    for i in range(count):
        x ^= (x << 13) & 0xFFFFFFFF
        x ^= x >> 17
        x ^= (x << 5) & 0xFFFFFFFF
        out[i] = x
    return out, x


def kat_packed(bits: int, k: int = KAT_K, n: int = KAT_N) -> np.ndarray:
    """Upstream trellis layout [k/16][n/16][16*bits] of uint16 (low half of each draw)."""
    words, _ = xorshift32_stream(k * n * bits // 16)
    return (words & 0xFFFF).astype(np.uint16).reshape(k // 16, n // 16, 16 * bits)


def kat_scales(k: int = KAT_K, n: int = KAT_N) -> tuple[np.ndarray, np.ndarray]:
    suh = ((np.arange(k) % 7 - 3) / 7).astype(np.float32).astype(np.float16).view(np.uint16)
    svh = ((np.arange(n) % 9 - 4) / 9).astype(np.float32).astype(np.float16).view(np.uint16)
    return suh, svh


def kat_input(rows: int, k: int = KAT_K) -> np.ndarray:
    i = np.arange(rows * k, dtype=np.int64)
    return (((i * 13) % 17 - 8) / 17).astype(np.float32).reshape(rows, k)


def kat_h128_blocks() -> np.ndarray:
    """128 blocks of 128 float32 values; the probe's first normalize pass."""
    words, _ = xorshift32_stream(128 * 128)
    vals = np.empty(128 * 128, np.float32)
    for i in range(vals.size):
        block, j = divmod(i, 128)
        r = int(words[i])
        if block == 0:
            v = 0.0
        elif block == 1:
            v = float(j == 0)
        elif block == 2:
            v = 1.0
        elif block == 3:
            v = -1.0 if (j & 1) else 1.0
        else:
            v = float(int(r % 8192) - 4096) / (997.0 if (block & 1) else 8192.0)
        vals[i] = np.float32(v)
    return vals.reshape(128, 128)


def rows_ids(count: int, n: int) -> np.ndarray:
    """Token ids of the reference's get_rows cases -- tests/test-exl3-graph.cpp:112."""
    if count == 1:
        return np.array([n - 1], np.int32)
    return np.array([0 if r % 3 == 0 else (n // 2 if r % 3 == 1 else n - 1) for r in range(count)], np.int32)
