"""ctypes binding of libexl3cu.so, the C ABI declared in include/exl3cu.h.

The library is built in-tree (``xiaomi-hexagon-exl3_b200/build.py``); there is
no fallback: if it is missing or fails to load, :func:`lib` raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parents[1]
LIB_PATH = PKG_DIR / "libexl3cu.so"
GGML_LIB_PATH = PKG_DIR / "libexl3cu_ggml.so"

OK, INVALID_ARGUMENT, NO_SUPPORT, OUT_OF_MEMORY, CUDA_ERROR = range(5)
F32, F16 = 0, 1
X_GLU, X_RMSNORM = 2, 3
CB_3INST, CB_MCG, CB_MUL1 = 0, 1, 2
ST_F16, ST_BF16, ST_I16, ST_F32, ST_I32 = range(5)
MODEL_VALIDATE_ONLY = 1

# every symbol include/exl3cu.h declares
EXPORTS = (
    "exl3cu_abi_version", "exl3cu_status_string", "exl3cu_last_error",
    "exl3cu_decode_codebook", "exl3cu_decode_inner", "exl3cu_hadamard128", "exl3cu_reconstruct",
    "exl3cu_weight_from_records", "exl3cu_weight_from_trellis", "exl3cu_weight_free", "exl3cu_weight_info",
    "exl3cu_weight_decode_inner", "exl3cu_mul_mat", "exl3cu_mul_mat_workspace_bytes", "exl3cu_mul_mat_ws",
    "exl3cu_mul_mat_host", "exl3cu_mul_mat_noalloc", "exl3cu_mul_mat_batch",
    "exl3cu_device_status", "exl3cu_gemm_config", "exl3cu_pack_ragged", "exl3cu_mul_mat_ragged",
    "exl3cu_get_rows", "exl3cu_get_rows_host",
    "exl3cu_mul_mat_batch_ex",
    "exl3cu_ipc_alloc", "exl3cu_ipc_free", "exl3cu_ipc_open", "exl3cu_ipc_close", "exl3cu_store_peers",
    "exl3cu_wait_peers", "exl3cu_mul_mat_peers",
    "exl3cu_model_open", "exl3cu_model_free", "exl3cu_model_info", "exl3cu_model_matrix_count",
    "exl3cu_model_matrix", "exl3cu_model_find_matrix", "exl3cu_model_head", "exl3cu_model_tensor",
    "exl3cu_model_find_tensor", "exl3cu_model_embedding", "exl3cu_model_embed",
)


class Exl3Error(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"exl3cu status {status}: {message}")
        self.status = status
        self.message = message


class Exl3InvalidArgument(Exl3Error, ValueError):
    pass


_LIB = None

_c = ctypes
_vp = _c.c_void_p
_sz = _c.c_size_t


def _declare(L):
    L.exl3cu_abi_version.restype = _c.c_int
    L.exl3cu_status_string.restype = _c.c_char_p
    L.exl3cu_status_string.argtypes = [_c.c_int]
    L.exl3cu_last_error.restype = _c.c_char_p
    L.exl3cu_decode_codebook.argtypes = [_vp, _sz, _c.c_uint, _vp, _vp]
    L.exl3cu_decode_inner.argtypes = [_vp, _sz, _sz, _sz, _sz, _c.c_uint, _c.c_uint, _vp, _vp]
    L.exl3cu_hadamard128.argtypes = [_vp, _sz, _vp]
    L.exl3cu_reconstruct.argtypes = [_vp, _vp, _vp, _sz, _sz, _sz, _sz, _c.c_uint, _c.c_uint, _vp, _vp]
    L.exl3cu_weight_from_records.argtypes = [_vp, _sz, _sz, _sz, _c.c_uint, _c.c_uint, _sz, _sz, _c.c_int,
                                             _c.POINTER(_vp)]
    L.exl3cu_weight_from_trellis.argtypes = [_vp, _vp, _vp, _sz, _sz, _c.c_uint, _c.c_uint, _sz, _sz, _c.c_int,
                                             _c.POINTER(_vp)]
    L.exl3cu_weight_free.argtypes = [_vp]
    L.exl3cu_weight_info.argtypes = [_vp, _c.POINTER(_sz), _c.POINTER(_sz), _c.POINTER(_c.c_uint),
                                     _c.POINTER(_c.c_uint), _c.POINTER(_sz)]
    L.exl3cu_weight_decode_inner.argtypes = [_vp, _vp, _vp]
    L.exl3cu_mul_mat.argtypes = [_vp, _vp, _c.c_int, _sz, _sz, _vp, _sz, _vp]
    L.exl3cu_mul_mat_workspace_bytes.restype = _sz
    L.exl3cu_mul_mat_workspace_bytes.argtypes = [_vp]
    L.exl3cu_mul_mat_ws.argtypes = [_vp, _vp, _c.c_int, _sz, _sz, _vp, _sz, _vp, _sz, _vp]
    L.exl3cu_mul_mat_host.argtypes = [_vp, _vp, _c.c_int, _sz, _sz, _vp, _sz, _c.c_int, _vp]
    L.exl3cu_get_rows.argtypes = [_vp, _vp, _sz, _vp, _sz, _vp]
    L.exl3cu_get_rows_host.argtypes = [_vp, _vp, _sz, _vp, _sz, _c.c_int, _vp]
    L.exl3cu_mul_mat_noalloc.argtypes = [_vp, _vp, _c.c_int, _sz, _sz, _vp, _sz, _vp]
    L.exl3cu_device_status.argtypes = [_c.c_int, _c.POINTER(_c.c_uint), _c.c_int]
    L.exl3cu_gemm_config.argtypes = [_sz, _c.c_int, _c.c_int]
    L.exl3cu_pack_ragged.argtypes = [_sz, _vp, _vp, _c.c_int32, _vp, _vp, _vp, _vp]
    L.exl3cu_mul_mat_ragged.argtypes = [_vp, _vp, _c.c_int, _sz, _vp, _sz, _sz, _vp, _sz, _vp]
    L.exl3cu_mul_mat_batch.argtypes = [_sz, _c.POINTER(_vp), _c.POINTER(_vp), _c.POINTER(_c.c_int),
                                       _c.POINTER(_sz), _c.POINTER(_sz), _c.POINTER(_vp), _c.POINTER(_sz), _vp]
    L.exl3cu_mul_mat_batch_ex.argtypes = [_sz, _c.POINTER(_vp), _c.POINTER(_vp), _c.POINTER(_c.c_int),
                                          _c.POINTER(_sz), _c.POINTER(_sz), _c.POINTER(_vp), _c.c_float,
                                          _c.POINTER(_vp), _c.POINTER(_sz), _c.POINTER(_c.c_int), _c.POINTER(_vp),
                                          _c.POINTER(_vp), _vp]
    _P = _c.POINTER
    L.exl3cu_ipc_alloc.argtypes = [_c.c_int, _sz, _P(_vp), _vp]
    L.exl3cu_ipc_free.argtypes = [_c.c_int, _vp]
    L.exl3cu_ipc_open.argtypes = [_c.c_int, _vp, _P(_vp)]
    L.exl3cu_ipc_close.argtypes = [_c.c_int, _vp]
    L.exl3cu_store_peers.argtypes = [_vp, _sz, _sz, _sz, _c.c_int, _vp, _sz, _sz, _sz, _vp, _vp]
    L.exl3cu_wait_peers.argtypes = [_vp, _vp, _sz, _sz, _vp, _sz, _sz, _sz, _vp]
    L.exl3cu_mul_mat_peers.argtypes = [_vp, _vp, _c.c_int, _sz, _sz, _vp, _sz, _c.c_int, _vp, _sz, _sz, _sz, _vp, _vp]
    L.exl3cu_model_open.argtypes = [_c.c_char_p, _c.c_int, _c.c_uint, _P(_vp)]
    L.exl3cu_model_free.argtypes = [_vp]
    L.exl3cu_model_info.argtypes = [_vp, _P(_sz), _P(_sz), _P(_sz), _P(_sz), _P(_sz), _P(_c.c_double)]
    L.exl3cu_model_matrix_count.restype = _sz
    L.exl3cu_model_matrix_count.argtypes = [_vp]
    L.exl3cu_model_matrix.argtypes = [_vp, _sz, _P(_c.c_char_p), _P(_sz), _P(_sz), _P(_c.c_uint), _P(_c.c_uint),
                                      _P(_vp)]
    L.exl3cu_model_find_matrix.argtypes = [_vp, _c.c_char_p, _P(_sz)]
    L.exl3cu_model_head.argtypes = [_vp, _P(_sz)]
    L.exl3cu_model_tensor.argtypes = [_vp, _sz, _P(_c.c_char_p), _P(_c.c_int), _P(_sz), _P(_P(_sz)), _P(_sz),
                                      _P(_vp)]
    L.exl3cu_model_find_tensor.argtypes = [_vp, _c.c_char_p, _P(_sz)]
    L.exl3cu_model_embedding.argtypes = [_vp, _c.c_uint32, _vp]
    L.exl3cu_model_embed.argtypes = [_vp, _vp, _sz, _vp, _sz, _vp]
    non_status = ("exl3cu_status_string", "exl3cu_last_error", "exl3cu_mul_mat_workspace_bytes",
                  "exl3cu_model_matrix_count")
    for name in EXPORTS:
        if name not in non_status:
            getattr(L, name).restype = _c.c_int


def lib():
    """Load (once) and return the C-ABI library; raises if it is not built."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is not built; run xiaomi-hexagon-exl3_b200/build.py")
        L = _c.CDLL(str(LIB_PATH))
        _declare(L)
        _LIB = L
    return _LIB


def check(status: int) -> None:
    if status == OK:
        return
    msg = lib().exl3cu_last_error().decode(errors="replace")
    if status == INVALID_ARGUMENT:
        raise Exl3InvalidArgument(status, msg)
    raise Exl3Error(status, msg)
