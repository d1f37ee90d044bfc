"""Seeded synthetic EXL3 workloads with the shapes and distributions of the
benchmark configurations (no public dataset or checkpoint is involved):

* trellis: uniform random uint16 words (every bitstream is a valid EXL3 tile);
* suh: +-1 input signs; svh: +-1 x U(0.01, 0.03) per-output scale, fp16;
* activations: N(0, 1) rounded to fp16.

Generators are numpy PCG64 with explicit seeds so every run is reproducible.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .format import pack_records

# Per-layer linear shapes (k, n) of the 2B-class hybrid decoder (hidden 2048, FFN 6144).
LAYER_SHAPES = {
    "q": (2048, 2048),
    "k": (2048, 512),
    "v": (2048, 512),
    "o": (2048, 2048),
    "gate": (2048, 6144),
    "up": (2048, 6144),
    "down": (6144, 2048),
}


@dataclass
class SyntheticMatrix:
    k: int
    n: int
    bits: int
    trellis: np.ndarray  # uint16 [k/16, n/16, 16*bits]
    suh: np.ndarray      # fp16 bits [k]
    svh: np.ndarray      # fp16 bits [n]

    def records(self) -> np.ndarray:
        return pack_records(self.trellis, self.suh, self.svh, self.bits)

    @property
    def trellis_bytes(self) -> int:
        return self.k * self.n * self.bits // 8


def matrix(k: int, n: int, bits: int, seed: int) -> SyntheticMatrix:
    rng = np.random.Generator(np.random.PCG64(seed))
    trellis = rng.integers(0, 65536, size=(k // 16, n // 16, 16 * bits), dtype=np.uint16)
    suh = rng.choice(np.array([-1.0, 1.0], np.float32), size=k).astype(np.float16).view(np.uint16)
    sign = rng.choice(np.array([-1.0, 1.0], np.float32), size=n)
    svh = (sign * rng.uniform(0.01, 0.03, size=n)).astype(np.float16).view(np.uint16)
    return SyntheticMatrix(k, n, bits, trellis, suh, svh)


def activations(rows: int, k: int, seed: int) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(seed))
    return rng.standard_normal((rows, k), dtype=np.float32).astype(np.float16)


def algorithmic_bytes(k: int, n: int, bits: int, rows: int = 1) -> int:
    """Useful bytes one mul_mat must move: packed trellis + one copy of su and sv
    + fp16 activations + fp32 outputs."""
    return k * n * bits // 8 + 2 * (k + n) + 2 * k * rows + 4 * n * rows
