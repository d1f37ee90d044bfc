"""Writes deployment directories (model.safetensors + hexagon-exl3.json) for
the loader tests: the reference reader test's fixture
(tests/test_model_reader.cpp:22-41 of the reference) and seeded mixed-bit
models, with hooks to corrupt one field at a time."""
from __future__ import annotations

import copy
import json
import struct
from pathlib import Path

import numpy as np

MUL1_MARKER = 0x83DCD12D
MCG_MARKER = 0xCBAC1FED


class Deployment:
    """An ordered tensor list plus a manifest; write() lays them out as the
    reference's fixture writer does (header JSON padded with spaces to a
    multiple of 8, tensors back to back in list order)."""

    def __init__(self):
        self.entries = []  # (name, dtype, shape, bytes)
        self.manifest = {}
        self.header_patch = {}  # name -> dict merged into that header entry after layout
        self.truncate = 0
        self.extra_payload = b""
        self.metadata = None

    def add(self, name, dtype, shape, data: bytes):
        self.entries.append((name, dtype, list(shape), bytes(data)))
        return self

    def payload(self) -> int:
        return sum(len(e[3]) for e in self.entries) + len(self.extra_payload)

    def header(self) -> dict:
        h = {}
        if self.metadata is not None:
            h["__metadata__"] = self.metadata
        off = 0
        for name, dtype, shape, data in self.entries:
            h[name] = {"dtype": dtype, "shape": shape, "data_offsets": [off, off + len(data)]}
            off += len(data)
        for name, patch in self.header_patch.items():
            h.setdefault(name, {}).update(copy.deepcopy(patch))
        return h

    def write(self, directory, header_text: str | None = None):
        d = Path(directory)
        d.mkdir(parents=True, exist_ok=True)
        text = header_text if header_text is not None else json.dumps(self.header())
        text += " " * ((8 - len(text.encode()) % 8) % 8)
        blob = struct.pack("<Q", len(text.encode())) + text.encode()
        blob += b"".join(e[3] for e in self.entries) + self.extra_payload
        if self.truncate:
            blob = blob[:-self.truncate]
        (d / "model.safetensors").write_bytes(blob)
        (d / "hexagon-exl3.json").write_text(json.dumps(self.manifest))
        return d


def manifest(source, hidden, vocab, parameters, payload, **over):
    m = {"format": "hexagon-exl3", "version": 1, "kv_cache": "f16", "reference_parameter_count": parameters,
         "weight_payload_bytes": payload,
         "input_embedding": {"type": "tied_linear", "source": source, "basis": "original", "token_axis": 1,
                             "hidden_size": hidden, "vocab_size": vocab}}
    m.update(over)
    return m


def reference_fixture() -> Deployment:
    """tests/test_model_reader.cpp:22-36: a 128x128 4-bit mul1 head with an all-zero
    trellis and unit scales; 8708 payload bytes, 16384 reference parameters."""
    d = Deployment()
    d.add("lm_head.trellis", "I16", [8, 8, 64], bytes(8192))
    ones = np.full(128, 1.0, np.float16).tobytes()
    d.add("lm_head.suh", "F16", [128], ones)
    d.add("lm_head.svh", "F16", [128], ones)
    d.add("lm_head.mul1", "I32", [], struct.pack("<I", MUL1_MARKER))
    d.manifest = manifest("lm_head", 128, 128, 16384, 8708)
    return d


def add_matrix(d: Deployment, prefix, k, n, bits, codebook, rng, scale_lo=0.01, scale_hi=0.03):
    """An EXL3 matrix: seeded trellis words, +-1 input signs, signed output scales, marker."""
    trellis = rng.integers(0, 65536, size=(k // 16, n // 16, 16 * bits), dtype=np.uint16)
    suh = rng.choice(np.array([-1.0, 1.0], np.float32), size=k).astype(np.float16)
    svh = (rng.choice(np.array([-1.0, 1.0], np.float32), size=n) * rng.uniform(scale_lo, scale_hi, n)).astype(
        np.float16)
    d.add(prefix + ".trellis", "I16", list(trellis.shape), trellis.tobytes())
    d.add(prefix + ".suh", "F16", [k], suh.tobytes())
    d.add(prefix + ".svh", "F16", [n], svh.tobytes())
    if codebook == "mul1":
        d.add(prefix + ".mul1", "I32", [], struct.pack("<I", MUL1_MARKER))
    elif codebook == "mcg":
        d.add(prefix + ".mcg", "I32", [], struct.pack("<I", MCG_MARKER))
    return k * n


# (prefix, k, n, bits, codebook) of the seeded mixed-bit model
MIXED_MATRICES = (
    ("lm_head", 256, 512, 4, "mul1"),
    ("model.layers.0.mlp.up_proj", 256, 384, 6, "mul1"),
    ("model.layers.0.self_attn.q_proj", 256, 256, 4, "mul1"),
    ("model.layers.0.self_attn.k_proj", 256, 128, 2, "mcg"),
    ("model.layers.0.mlp.down_proj", 384, 256, 3, "3inst"),
)


def mixed_model(seed: int = 7) -> Deployment:
    """4/6/2/3-bit matrices with all three codebooks, plus plain F32/BF16/F16/I32 tensors."""
    rng = np.random.Generator(np.random.PCG64(seed))
    d = Deployment()
    params = 0
    for prefix, k, n, bits, cb in MIXED_MATRICES:
        params += add_matrix(d, prefix, k, n, bits, cb, rng)
    norm = (1.0 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    d.add("model.norm.weight", "F32", [256], norm.tobytes())
    d.add("model.layers.0.linear_attn.A_log", "F32", [16], rng.standard_normal(16).astype(np.float32).tobytes())
    conv = rng.standard_normal((4, 256)).astype(np.float32)
    d.add("model.layers.0.linear_attn.conv1d.weight", "BF16", [4, 256],
          (conv.view(np.uint32) >> 16).astype(np.uint16).tobytes())
    d.add("model.layers.0.input_layernorm.weight", "F16", [256], rng.standard_normal(256).astype(np.float16).tobytes())
    d.add("model.layers.0.layer_types", "I32", [3], np.array([1, 0, 2], np.int32).tobytes())
    params += 256 + 16 + 1024 + 256 + 3
    d.metadata = {"format": "pt", "note": "seeded synthetic é"}
    d.manifest = manifest("lm_head", 256, 512, params, d.payload())
    return d
