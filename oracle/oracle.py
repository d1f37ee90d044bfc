"""EXL3 CPU oracle loader -- TEST INFRASTRUCTURE ONLY.

ctypes bindings for the two CPU checkers built by ``oracle/Makefile``:

* ``liboracle.so``        -- our plain-C restatement of the reference algorithm
                             (``oracle/exl3_oracle.c``);
* ``_ref/libexl3ref.so``  -- the reference's own ``src/exl3_codec.cpp`` and
                             ``src/exl3-ggml.cpp`` compiled unmodified, with
                             ``oracle/ref_shim.cpp`` as the C entry layer.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU leg import
this module, as the checker; the shipped library never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libexl3ref.so"

MUL1, MCG, THREE_INST = 2, 1, 0

_c = ctypes
_u16p = _c.POINTER(_c.c_uint16)
_f32p = _c.POINTER(_c.c_float)
_u8p = _c.POINTER(_c.c_uint8)
_i32p = _c.POINTER(_c.c_int32)
_sz = _c.c_size_t


def build() -> None:
    """Compile liboracle.so (and _ref when the reference sources are present)."""
    subprocess.run(["make", "-s", "-C", str(HERE), "all"], check=True)


def _ptr(a: np.ndarray, t):
    return a.ctypes.data_as(t)


class _Lib:
    def __init__(self, path: Path, prefix: str):
        if not path.exists():
            raise FileNotFoundError(f"{path} not built (run make -C oracle)")
        self.lib = _c.CDLL(str(path))
        self.prefix = prefix
        L = self.lib
        p = prefix
        getattr(L, p + "half_to_float").restype = _c.c_float
        getattr(L, p + "half_to_float").argtypes = [_c.c_uint16]
        getattr(L, p + "float_to_half").restype = _c.c_uint16
        getattr(L, p + "float_to_half").argtypes = [_c.c_float]
        getattr(L, p + "decode_tile").argtypes = [_u16p, _c.c_uint, _c.c_uint, _u16p]
        getattr(L, p + "decode_inner").argtypes = [_u16p, _sz, _sz, _sz, _sz, _c.c_uint, _c.c_uint, _u16p]
        getattr(L, p + "hadamard128").argtypes = [_f32p, _sz]
        getattr(L, p + "reconstruct").argtypes = [_u16p, _u16p, _u16p, _sz, _sz, _sz, _sz, _c.c_uint, _c.c_uint,
                                                  _u16p]

    def _fn(self, name):
        return getattr(self.lib, self.prefix + name)

    def half_to_float(self, h: int) -> float:
        return self._fn("half_to_float")(h)

    def float_to_half(self, f: float) -> int:
        return self._fn("float_to_half")(f)

    def decode_tile(self, packed: np.ndarray, bits: int, codebook: int = MUL1) -> np.ndarray:
        packed = np.ascontiguousarray(packed, dtype=np.uint16)
        out = np.zeros(256, np.uint16)
        if self._fn("decode_tile")(_ptr(packed, _u16p), bits, codebook, _ptr(out, _u16p)):
            raise ValueError("invalid EXL3 tile arguments")
        return out.reshape(16, 16)

    def decode_inner(self, packed: np.ndarray, k: int, n: int, bits: int, codebook: int = MUL1,
                     first_column: int = 0, column_count: int | None = None) -> np.ndarray:
        packed = np.ascontiguousarray(packed, dtype=np.uint16)
        cc = n - first_column if column_count is None else column_count
        out = np.zeros((k, max(cc, 0)), np.uint16)
        if self._fn("decode_inner")(_ptr(packed, _u16p), k, n, first_column, cc, bits, codebook, _ptr(out, _u16p)):
            raise ValueError("invalid EXL3 decode arguments")
        return out

    def hadamard128(self, values: np.ndarray) -> np.ndarray:
        v = np.array(values, dtype=np.float32, copy=True).reshape(-1)
        if self._fn("hadamard128")(_ptr(v, _f32p), v.size):
            raise ValueError("H128 length must be a multiple of 128")
        return v.reshape(np.shape(values))

    def reconstruct(self, packed, suh, svh, k, n, bits, codebook=MUL1, first_column=0, column_count=None):
        packed = np.ascontiguousarray(packed, dtype=np.uint16)
        suh = np.ascontiguousarray(suh, dtype=np.uint16)
        svh = np.ascontiguousarray(svh, dtype=np.uint16)
        cc = n - first_column if column_count is None else column_count
        out = np.zeros((k, cc), np.uint16)
        if self._fn("reconstruct")(_ptr(packed, _u16p), _ptr(suh, _u16p), _ptr(svh, _u16p), k, n, first_column, cc,
                                   bits, codebook, _ptr(out, _u16p)):
            raise ValueError("invalid EXL3 reconstruct arguments")
        return out


class Oracle(_Lib):
    """Our C restatement (liboracle.so)."""

    def __init__(self, path: Path = ORACLE_SO):
        super().__init__(path, "orc_")
        L = self.lib
        L.orc_decode_codebook.restype = _c.c_uint16
        L.orc_decode_codebook.argtypes = [_c.c_uint16, _c.c_uint]
        L.orc_group_bytes.restype = _sz
        L.orc_group_bytes.argtypes = [_c.c_uint]
        L.orc_pack_records.argtypes = [_u16p, _u16p, _u16p, _sz, _sz, _c.c_uint, _u8p]
        L.orc_mul_mat.argtypes = [_u8p, _c.c_uint, _c.c_uint, _sz, _sz, _c.c_void_p, _c.c_int, _sz, _sz, _f32p, _sz,
                                  _c.c_int]
        L.orc_get_rows.argtypes = [_u8p, _c.c_uint, _c.c_uint, _sz, _sz, _i32p, _sz, _f32p]

    def decode_codebook(self, states: np.ndarray, codebook: int = MUL1) -> np.ndarray:
        states = np.asarray(states, dtype=np.uint16).reshape(-1)
        f = self.lib.orc_decode_codebook
        return np.fromiter((f(int(s), codebook) for s in states), dtype=np.uint16, count=states.size)

    def codebook_table(self, codebook: int = MUL1) -> np.ndarray:
        return self.decode_codebook(np.arange(65536, dtype=np.uint16), codebook)

    def pack_records(self, packed, suh, svh, k, n, bits) -> np.ndarray:
        packed = np.ascontiguousarray(packed, dtype=np.uint16)
        suh = np.ascontiguousarray(suh, dtype=np.uint16)
        svh = np.ascontiguousarray(svh, dtype=np.uint16)
        out = np.zeros((n // 128) * (k // 128) * self.lib.orc_group_bytes(bits), np.uint8)
        if self.lib.orc_pack_records(_ptr(packed, _u16p), _ptr(suh, _u16p), _ptr(svh, _u16p), k, n, bits,
                                     _ptr(out, _u8p)):
            raise ValueError("invalid EXL3 record geometry")
        return out

    def mul_mat(self, records, bits, k, n, x, codebook=MUL1, nth: int = 1) -> np.ndarray:
        records = np.ascontiguousarray(records, dtype=np.uint8)
        x = np.ascontiguousarray(x)
        if x.dtype not in (np.float16, np.float32):
            raise TypeError("x must be float16 or float32")
        x2 = x.reshape(-1, k)
        rows = x2.shape[0]
        y = np.zeros((rows, n), np.float32)
        if self.lib.orc_mul_mat(_ptr(records, _u8p), bits, codebook, k, n, x2.ctypes.data_as(_c.c_void_p),
                                int(x.dtype == np.float16), rows, k, _ptr(y, _f32p), n, nth):
            raise ValueError("invalid EXL3 mul_mat arguments")
        return y

    def get_rows(self, records, bits, k, n, ids, codebook=MUL1) -> np.ndarray:
        records = np.ascontiguousarray(records, dtype=np.uint8)
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.zeros((ids.size, k), np.float32)
        if self.lib.orc_get_rows(_ptr(records, _u8p), bits, codebook, k, n, _ptr(ids, _i32p), ids.size,
                                 _ptr(out, _f32p)):
            raise ValueError("invalid EXL3 get_rows arguments")
        return out


class Reference(_Lib):
    """The reference's own sources, compiled unmodified (oracle/_ref/libexl3ref.so)."""

    def __init__(self, path: Path = REF_SO):
        super().__init__(path, "ref_")
        L = self.lib
        L.ref_decode_codebook.argtypes = [_u16p, _sz, _c.c_uint, _u16p]
        L.ref_ggml_mul_mat.argtypes = [_c.c_void_p, _c.c_uint, _sz, _sz, _c.c_void_p, _c.c_int, _sz, _f32p, _c.c_int]
        L.ref_ggml_get_rows.argtypes = [_c.c_void_p, _c.c_uint, _sz, _sz, _i32p, _sz, _f32p, _c.c_int]
        L.ref_loop_mul_mat.argtypes = [_c.c_void_p, _c.c_uint, _c.c_uint, _sz, _sz, _c.c_void_p, _c.c_int, _sz,
                                       _f32p, _c.c_int]

    def codebook_table(self, codebook: int = MUL1) -> np.ndarray:
        states = np.arange(65536, dtype=np.uint16)
        out = np.zeros(65536, np.uint16)
        if self.lib.ref_decode_codebook(_ptr(states, _u16p), 65536, codebook, _ptr(out, _u16p)):
            raise ValueError("invalid codebook")
        return out

    def mul_mat(self, records, bits, k, n, x, codebook=MUL1, nth: int = 1) -> np.ndarray:
        """ggml_exl3_mul_mat itself for 4/6/8-bit mul1; the reference-codec loop otherwise."""
        records = np.ascontiguousarray(records, dtype=np.uint8)
        x = np.ascontiguousarray(x)
        rows = x.size // k
        y = np.zeros((rows, n), np.float32)
        is16 = int(x.dtype == np.float16)
        if bits in (4, 6, 8) and codebook == MUL1:
            rc = self.lib.ref_ggml_mul_mat(records.ctypes.data_as(_c.c_void_p), bits, k, n,
                                           x.ctypes.data_as(_c.c_void_p), is16, rows, _ptr(y, _f32p), nth)
        else:
            rc = self.lib.ref_loop_mul_mat(records.ctypes.data_as(_c.c_void_p), bits, codebook, k, n,
                                           x.ctypes.data_as(_c.c_void_p), is16, rows, _ptr(y, _f32p), nth)
        if rc:
            raise ValueError("invalid EXL3 mul_mat arguments")
        return y

    def get_rows(self, records, bits, k, n, ids, nth: int = 1) -> np.ndarray:
        records = np.ascontiguousarray(records, dtype=np.uint8)
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.zeros((ids.size, k), np.float32)
        if self.lib.ref_ggml_get_rows(records.ctypes.data_as(_c.c_void_p), bits, k, n, _ptr(ids, _i32p), ids.size,
                                      _ptr(out, _f32p), nth):
            raise ValueError("invalid EXL3 get_rows arguments")
        return out


def have_reference() -> bool:
    return REF_SO.exists()


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1
