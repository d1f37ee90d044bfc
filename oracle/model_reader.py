"""CPU restatement of the reference's deployment reader -- TEST INFRASTRUCTURE.

Only tests/ may use this module: it is the checker for the B200 loader
(exl3cu_model_open), never part of the product path.

It restates the constructor of exl3::Model (src/exl3_model.cpp:79-157) with
Python's json and struct modules, raising ModelError with the reference's
messages, and the matrix inventory rules of tools/inspect_model.py:68-99 that
the B200 loader applies to every EXL3 matrix (plus the device operator's
requirements: in/out features multiples of 128, F16 X.suh [k] and X.svh [n]).

Pinning: the reference's own reader test (tests/test_model_reader.cpp:22-79)
is rebuilt in tests/test_model_loader.py and must give the reference's
answers here (accept with tensor_count 4 and payload 8708; reject the budget,
overlapping-span, negative-dimension and truncation cases).  The reference
reader itself cannot be compiled in this container (it needs nlohmann/json,
which is absent), so no live run backs this restatement.
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass, field
from pathlib import Path

WIDTHS = {"F16": 2, "BF16": 2, "I16": 2, "F32": 4, "I32": 4}  # src/exl3_model.cpp:87
MUL1_MARKER = 0x83DCD12D  # src/exl3_model.cpp:146
MCG_MARKER = 0xCBAC1FED   # src/exl3_model.cpp:153
CB_3INST, CB_MCG, CB_MUL1 = 0, 1, 2


class ModelError(ValueError):
    pass


def _is_int(v) -> bool:
    return isinstance(v, int) and not isinstance(v, bool)


def positive_integer(v, zero_allowed: bool = False) -> int:
    """src/exl3_model.cpp:45-50."""
    if not _is_int(v):
        raise ModelError("Expected an integer dimension or offset")
    if v < 0 or (v == 0 and not zero_allowed):
        raise ModelError("Invalid dimension or offset")
    return v


@dataclass
class Tensor:
    dtype: str
    shape: tuple
    begin: int
    end: int


@dataclass
class Matrix:
    name: str
    k: int
    n: int
    bits: int
    codebook: int


@dataclass
class ModelInfo:
    tensors: dict
    payload: int
    data_begin: int
    hidden: int
    vocab: int
    parameters: int
    head: str
    head_bits: int
    head_codebook: int
    matrices: list = field(default_factory=list)
    raw: bytes = b""

    @property
    def bits_per_weight(self) -> float:
        return self.payload * 8 / self.parameters

    def array(self, name: str):
        """The tensor's bytes as a numpy array of its dtype and shape (I16/BF16 as uint16)."""
        import numpy as np

        t = self.tensors[name]
        dt = {"F16": np.float16, "BF16": np.uint16, "I16": np.uint16, "F32": np.float32, "I32": np.int32}[t.dtype]
        buf = self.raw[self.data_begin + t.begin:self.data_begin + t.end]
        return np.frombuffer(buf, dtype=dt).reshape(t.shape)


def at(obj, key):
    """nlohmann's json::at: the member, or an error naming the key (also for a non-object)."""
    if not isinstance(obj, dict) or key not in obj:
        raise ModelError(f'missing key "{key}"')
    return obj[key]


def _codebook(info_tensors, raw, data_begin, prefix, what) -> int:
    """src/exl3_model.cpp:140-156."""
    mul1 = info_tensors.get(prefix + ".mul1")
    mcg = info_tensors.get(prefix + ".mcg")
    if mul1 is not None and mcg is not None:
        raise ModelError(f"Ambiguous {what} codebook")
    marker = mul1 if mul1 is not None else mcg
    if marker is None:
        return CB_3INST
    if marker.dtype != "I32" or marker.end - marker.begin != 4:
        raise ModelError("Invalid codebook marker")
    value, = struct.unpack_from("<I", raw, data_begin + marker.begin)
    if mul1 is not None:
        if value != MUL1_MARKER:
            raise ModelError("Unsupported mul1 codebook multiplier")
        return CB_MUL1
    if value != MCG_MARKER:
        raise ModelError("Unsupported mcg codebook multiplier")
    return CB_MCG


def read_model(directory) -> ModelInfo:
    directory = Path(directory)
    try:
        raw = (directory / "model.safetensors").read_bytes()
    except OSError:
        raise ModelError("Cannot open model weights") from None
    if len(raw) < 8:
        raise ModelError("Invalid weight file size")
    header_size, = struct.unpack_from("<Q", raw, 0)                       # :81-82
    if header_size > 64 * 1024 * 1024 or header_size > len(raw) - 8:     # :83
        raise ModelError("Invalid safetensors header length")
    try:
        header = json.loads(raw[8:8 + header_size])
    except (ValueError, UnicodeDecodeError) as e:
        raise ModelError(f"JSON: {e}") from None
    if not isinstance(header, dict):
        raise ModelError("Invalid safetensors header")
    data_begin = 8 + header_size
    payload_size = len(raw) - data_begin
    tensors = {}
    spans = []
    for name, info in header.items():                                      # :88-108
        if name == "__metadata__":
            continue
        dtype = at(info, "dtype")
        if not isinstance(dtype, str) or dtype not in WIDTHS:
            raise ModelError("Unsupported model dtype")
        width = WIDTHS[dtype]
        shape = at(info, "shape")
        if not isinstance(shape, list):
            raise ModelError("Expected an integer dimension or offset")
        elements = 1
        dims = []
        for d in shape:
            dim = positive_integer(d)
            if elements > (2**64 - 1) // dim:
                raise ModelError("Tensor shape overflow")
            elements *= dim
            dims.append(dim)
        offsets = at(info, "data_offsets")
        if not isinstance(offsets, list) or len(offsets) != 2:
            raise ModelError("Invalid tensor offset pair")
        begin = positive_integer(offsets[0], True)
        end = positive_integer(offsets[1], True)
        if end < begin or end > payload_size or elements > (2**64 - 1) // width or end - begin != elements * width:
            raise ModelError("Invalid tensor data span")
        tensors[name] = Tensor(dtype, tuple(dims), begin, end)
        spans.append((begin, end))
    payload = 0
    for begin, end in sorted(spans):                                       # :109-113
        if begin != payload:
            raise ModelError("Overlapping or missing tensor data")
        payload = end
    if payload != payload_size:                                            # :114
        raise ModelError("Unaccounted model payload")

    try:
        manifest = json.loads((directory / "hexagon-exl3.json").read_bytes())
    except OSError:
        raise ModelError("Cannot open deployment manifest") from None
    except (ValueError, UnicodeDecodeError) as e:
        raise ModelError(f"JSON: {e}") from None
    if not isinstance(manifest, dict):
        raise ModelError("Unsupported deployment manifest")

    def is_str(v, text):
        return isinstance(v, str) and v == text

    def is_num(v, value):
        return isinstance(v, (int, float)) and not isinstance(v, bool) and v == value

    if not (is_str(at(manifest, "format"), "hexagon-exl3") and is_num(at(manifest, "version"), 1)
            and is_str(at(manifest, "kv_cache"), "f16")):                # :116-118
        raise ModelError("Unsupported deployment manifest")
    emb = at(manifest, "input_embedding")
    if not (is_str(at(emb, "type"), "tied_linear") and is_str(at(emb, "basis"), "original")
            and is_num(at(emb, "token_axis"), 1)):                        # :120-123
        raise ModelError("Unsupported embedding alias")
    k = positive_integer(at(emb, "hidden_size"))                           # :124-126
    n = positive_integer(at(emb, "vocab_size"))
    if k % 128 or n % 128 or k > 16384 or n > 1048576:
        raise ModelError("Invalid embedding geometry")
    parameters = positive_integer(at(manifest, "reference_parameter_count"))   # :127-130
    if positive_integer(at(manifest, "weight_payload_bytes")) != payload or payload * 8 / parameters > 5.0:
        raise ModelError("Model payload or budget mismatch")
    head = at(emb, "source")
    if not isinstance(head, str):
        raise ModelError("Unsupported embedding alias")

    def tensor(key):
        if key not in tensors:
            raise ModelError("Missing model tensor: " + key)
        return tensors[key]

    packed = tensor(head + ".trellis")                                     # :132-135
    s = packed.shape
    if (packed.dtype != "I16" or len(s) != 3 or s[0] != k // 16 or s[1] != n // 16 or s[2] % 16 or s[2] < 16
            or s[2] > 128):
        raise ModelError("Invalid head trellis")
    for suffix, size in (("suh", k), ("svh", n)):                          # :137-140
        sc = tensor(head + "." + suffix)
        if sc.dtype != "F16" or sc.shape != (size,):
            raise ModelError("Invalid head scale")
    head_cb = _codebook(tensors, raw, data_begin, head, "head")

    matrices = []
    for name in sorted(tensors):                                           # tools/inspect_model.py:68-99
        if not name.endswith(".trellis") or len(name) <= len(".trellis"):
            continue
        prefix = name[:-len(".trellis")]
        if prefix + ".signs" in tensors:
            continue
        t = tensors[name]
        if t.dtype != "I16" or len(t.shape) != 3 or t.shape[2] % 16:
            raise ModelError("Unsupported EXL3 trellis: " + name)
        bits = t.shape[2] // 16
        if not 1 <= bits <= 8:
            raise ModelError("Invalid EXL3 bitrate: " + name)
        mk, mn = t.shape[0] * 16, t.shape[1] * 16
        if mk % 128 or mn % 128:
            raise ModelError(f"EXL3 matrix {prefix}: in and out features must be multiples of 128")
        su, sv = tensors.get(prefix + ".suh"), tensors.get(prefix + ".svh")
        if (su is None or sv is None or su.dtype != "F16" or sv.dtype != "F16" or su.shape != (mk,)
                or sv.shape != (mn,)):
            raise ModelError("Invalid EXL3 scales: " + prefix)
        matrices.append(Matrix(prefix, mk, mn, bits, _codebook(tensors, raw, data_begin, prefix, "matrix")))
    return ModelInfo(tensors, payload, data_begin, k, n, parameters, head, s[2] // 16, head_cb, matrices, raw)
