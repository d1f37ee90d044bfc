"""Exl3Model: a deployment directory loaded onto one GPU (exl3cu_model_* C ABI).

Mirrors exl3::Model (src/exl3_model.cpp, include/exl3_model.h): the
constructor validates model.safetensors and hexagon-exl3.json with the same
rules and messages (failures raise Exl3InvalidArgument), and tensor_count(),
payload_bytes(), hidden_size(), vocab_size(), bits_per_weight() and
embedding(token) keep their meaning.  Beyond the reference, every EXL3 matrix
of the file is a persistent device weight (at its own bit width) and every
other tensor a device buffer:

    m = Exl3Model("deploy/", device=0)
    w = m.weight("model.layers.0.mlp.down_proj")    # Exl3Weight owned by m
    y = w.mul_mat(x)
    e = m.embed(torch.tensor([1, 2, 3], dtype=torch.int32, device="cuda"))
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from ._lib import MODEL_VALIDATE_ONLY, ST_BF16, ST_F16, ST_F32, ST_I16, ST_I32, check, lib

_TYPESTR = {ST_F16: "<f2", ST_BF16: "<i2", ST_I16: "<i2", ST_F32: "<f4", ST_I32: "<i4"}
DTYPE_NAMES = {ST_F16: "F16", ST_BF16: "BF16", ST_I16: "I16", ST_F32: "F32", ST_I32: "I32"}


@dataclass(frozen=True)
class MatrixInfo:
    name: str
    k: int
    n: int
    bits: int
    codebook: int


@dataclass(frozen=True)
class TensorInfo:
    name: str
    dtype: str
    shape: tuple
    nbytes: int
    device_ptr: int  # 0 for parts of an EXL3 matrix and for validate-only models


class _DeviceArray:
    """__cuda_array_interface__ view of a model tensor; keeps the model alive."""

    def __init__(self, owner, ptr: int, shape: tuple, typestr: str):
        self._owner = owner
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 3,
                                         "strides": None}


class Exl3Model:
    def __init__(self, directory, device: int = 0, validate_only: bool = False):
        self._h = ctypes.c_void_p()
        self.device = device
        self.directory = str(directory)
        flags = MODEL_VALIDATE_ONLY if validate_only else 0
        check(lib().exl3cu_model_open(self.directory.encode(), int(device), flags, ctypes.byref(self._h)))
        L = lib()
        tc, pb, hs, vs, pc = (ctypes.c_size_t() for _ in range(5))
        bpw = ctypes.c_double()
        check(L.exl3cu_model_info(self._h, ctypes.byref(tc), ctypes.byref(pb), ctypes.byref(hs), ctypes.byref(vs),
                                  ctypes.byref(pc), ctypes.byref(bpw)))
        self._info = (tc.value, pb.value, hs.value, vs.value, pc.value, bpw.value)
        head = ctypes.c_size_t()
        check(L.exl3cu_model_head(self._h, ctypes.byref(head)))
        self._matrices = [self._matrix(i) for i in range(L.exl3cu_model_matrix_count(self._h))]
        self._head = self._matrices[head.value].name
        self._weights = {}

    # -- exl3::Model accessors (src/exl3_model.cpp:162-166) -------------------------------------
    def tensor_count(self) -> int:
        return self._info[0]

    def payload_bytes(self) -> int:
        return self._info[1]

    def hidden_size(self) -> int:
        return self._info[2]

    def vocab_size(self) -> int:
        return self._info[3]

    def parameter_count(self) -> int:
        return self._info[4]

    def bits_per_weight(self) -> float:
        return self._info[5]

    def embedding(self, token: int) -> np.ndarray:
        """exl3::Model::embedding: the tied head's original-basis column `token` as fp16 bits [hidden]."""
        out = np.empty(self.hidden_size(), np.uint16)
        if not 0 <= int(token) < 2**32:
            raise ValueError("Token ID outside vocabulary")
        check(lib().exl3cu_model_embedding(self._h, int(token), out.ctypes.data_as(ctypes.c_void_p)))
        return out

    # -- device-side extensions ------------------------------------------------------------------
    @property
    def head_name(self) -> str:
        return self._head

    def matrices(self) -> list[MatrixInfo]:
        return list(self._matrices)

    def _matrix(self, i: int) -> MatrixInfo:
        name = ctypes.c_char_p()
        k, n = ctypes.c_size_t(), ctypes.c_size_t()
        bits, cb = ctypes.c_uint(), ctypes.c_uint()
        check(lib().exl3cu_model_matrix(self._h, i, ctypes.byref(name), ctypes.byref(k), ctypes.byref(n),
                                        ctypes.byref(bits), ctypes.byref(cb), None))
        return MatrixInfo(name.value.decode(), k.value, n.value, bits.value, cb.value)

    def weight(self, name: str):
        """The device weight of EXL3 matrix `name` (an Exl3Weight that keeps this model alive)."""
        if name in self._weights:
            return self._weights[name]
        from .ops import Exl3Weight

        idx = ctypes.c_size_t()
        check(lib().exl3cu_model_find_matrix(self._h, name.encode(), ctypes.byref(idx)))
        h = ctypes.c_void_p()
        check(lib().exl3cu_model_matrix(self._h, idx.value, None, None, None, None, None, ctypes.byref(h)))
        if not h.value:
            raise RuntimeError("model was opened for validation only")
        w = Exl3Weight(h, self.device, owner=self)
        self._weights[name] = w
        return w

    def tensors(self) -> list[TensorInfo]:
        return [self._tensor(i) for i in range(self.tensor_count())]

    def _tensor(self, i: int) -> TensorInfo:
        name = ctypes.c_char_p()
        dtype = ctypes.c_int()
        ndim, nbytes = ctypes.c_size_t(), ctypes.c_size_t()
        shape = ctypes.POINTER(ctypes.c_size_t)()
        ptr = ctypes.c_void_p()
        check(lib().exl3cu_model_tensor(self._h, i, ctypes.byref(name), ctypes.byref(dtype), ctypes.byref(ndim),
                                        ctypes.byref(shape), ctypes.byref(nbytes), ctypes.byref(ptr)))
        dims = tuple(int(shape[j]) for j in range(ndim.value))
        return TensorInfo(name.value.decode(), DTYPE_NAMES[dtype.value], dims, nbytes.value, ptr.value or 0)

    def tensor_info(self, name: str) -> TensorInfo:
        idx = ctypes.c_size_t()
        check(lib().exl3cu_model_find_tensor(self._h, name.encode(), ctypes.byref(idx)))
        return self._tensor(idx.value)

    def tensor(self, name: str):
        """A plain (non-EXL3) tensor as a torch tensor viewing the model's device arena."""
        import torch

        info = self.tensor_info(name)
        if not info.device_ptr:
            raise ValueError(f"{name} has no device copy (an EXL3 matrix part, or a validate-only model)")
        code = {v: k for k, v in DTYPE_NAMES.items()}[info.dtype]
        t = torch.as_tensor(_DeviceArray(self, info.device_ptr, info.shape, _TYPESTR[code]),
                            device=f"cuda:{self.device}")
        return t.view(torch.bfloat16) if code == ST_BF16 else t

    def embed(self, ids, out=None, stream=None):
        """Batched tied-head embedding on the device: f32 [count, hidden] (exl3cu_model_embed)."""
        import torch

        from .ops import _ptr, _stream_handle

        if ids.dtype != torch.int32:
            raise TypeError("ids must be int32")
        ids2 = ids.reshape(-1).contiguous()
        k = self.hidden_size()
        if out is None:
            out = torch.empty((ids2.numel(), k), dtype=torch.float32, device=ids.device)
        check(lib().exl3cu_model_embed(self._h, _ptr(ids2), ids2.numel(), _ptr(out), out.stride(0),
                                       _stream_handle(stream)))
        return out

    def close(self) -> None:
        if getattr(self, "_h", None) and self._h.value:
            for w in self._weights.values():
                w._h = None
            self._weights.clear()
            lib().exl3cu_model_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
