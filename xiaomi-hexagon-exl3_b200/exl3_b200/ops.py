"""Python face of the exl3cu C ABI: persistent EXL3 weights and the operator.

Everything here calls into libexl3cu.so through ctypes; torch is used only for
device memory and the current CUDA stream.  Mirrors the reference interface
for this path: ``mul_mat`` is ``ggml_exl3_mul_mat`` (src/exl3-ggml.cpp:51-92,
y = x . W with W = diag(su) H W_inner H diag(sv) per 128 block, f32 out), and
the codec functions are those of include/exl3_codec.h:10-29.  Invalid
arguments raise :class:`Exl3InvalidArgument` (a ValueError), as the reference
raises std::invalid_argument.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from ._lib import CB_MUL1, F16, F32, check, lib

_vp = ctypes.c_void_p


def _stream_handle(stream) -> _vp:
    if stream is None:
        stream = torch.cuda.current_stream()
    return _vp(stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream))


def _ptr(t) -> _vp:
    if isinstance(t, torch.Tensor):
        return _vp(t.data_ptr())
    if isinstance(t, np.ndarray):
        return _vp(t.ctypes.data)
    raise TypeError(f"unsupported buffer type {type(t)!r}")


def _as_u16_tensor(a, device) -> torch.Tensor:
    if isinstance(a, torch.Tensor):
        t = a
    else:
        t = torch.from_numpy(np.ascontiguousarray(a).view(np.int16))
    if t.dtype != torch.int16:
        t = t.view(torch.int16) if t.element_size() == 2 else t
    return t.to(device).contiguous()


class Exl3Weight:
    """An EXL3 matrix resident in device memory (column blocks [first_block, +block_count))."""

    def __init__(self, handle: _vp, device: int, owner=None):
        self._h = handle
        self.device = device
        self._owner = owner  # an Exl3Model that owns the handle (kept alive by this reference)
        k, n_local, dev_bytes = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
        bits, cb = ctypes.c_uint(), ctypes.c_uint()
        check(lib().exl3cu_weight_info(self._h, ctypes.byref(k), ctypes.byref(n_local), ctypes.byref(bits),
                                       ctypes.byref(cb), ctypes.byref(dev_bytes)))
        self.k, self.n, self.bits, self.codebook = k.value, n_local.value, bits.value, cb.value
        self.device_bytes = dev_bytes.value

    # -- construction ------------------------------------------------------------------------
    @classmethod
    def from_records(cls, records, k: int, n: int, bits: int, codebook: int = CB_MUL1, device: int = 0,
                     first_block: int = 0, block_count: int = 0) -> "Exl3Weight":
        if isinstance(records, (bytes, bytearray)):
            records = np.frombuffer(records, np.uint8)
        if isinstance(records, np.ndarray):
            records = np.ascontiguousarray(records)
            nbytes = records.nbytes
        else:
            records = records.contiguous()
            nbytes = records.numel() * records.element_size()
        h = _vp()
        check(lib().exl3cu_weight_from_records(_ptr(records), nbytes, k, n, bits, codebook, first_block,
                                               block_count, device, ctypes.byref(h)))
        return cls(h, device)

    @classmethod
    def from_trellis(cls, trellis, suh, svh, codebook: int = CB_MUL1, device: int = 0, first_block: int = 0,
                     block_count: int = 0) -> "Exl3Weight":
        if isinstance(trellis, torch.Tensor):  # host or device tensors; the ABI copies either
            trellis, suh, svh = (t.contiguous() for t in (trellis, suh, svh))
            if trellis.element_size() != 2 or suh.element_size() != 2 or svh.element_size() != 2:
                raise TypeError("trellis, suh and svh must be 16-bit tensors")
        else:
            trellis = np.ascontiguousarray(np.asarray(trellis).view(np.uint16))
            suh = np.ascontiguousarray(np.asarray(suh).view(np.uint16))
            svh = np.ascontiguousarray(np.asarray(svh).view(np.uint16))
        kt, nt, tw = trellis.shape
        h = _vp()
        check(lib().exl3cu_weight_from_trellis(_ptr(trellis), _ptr(suh), _ptr(svh), kt * 16, nt * 16, tw // 16,
                                               codebook, first_block, block_count, device, ctypes.byref(h)))
        return cls(h, device)

    def free(self) -> None:
        if getattr(self, "_h", None):
            if getattr(self, "_owner", None) is None:
                lib().exl3cu_weight_free(self._h)
            self._h = None

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.free()
        except Exception:
            pass

    @property
    def handle(self) -> _vp:
        return self._h

    @property
    def workspace_bytes(self) -> int:
        return lib().exl3cu_mul_mat_workspace_bytes(self._h)

    # -- operator ------------------------------------------------------------------------------
    def mul_mat(self, x: torch.Tensor, out: torch.Tensor | None = None, stream=None,
                workspace: torch.Tensor | None = None) -> torch.Tensor:
        """y = x . W for device tensors x [rows, k] (f32 or f16) -> y [rows, n] f32."""
        if x.dtype not in (torch.float32, torch.float16):
            raise TypeError("x must be float32 or float16")
        x2 = x.reshape(-1, x.shape[-1])
        if x2.stride(-1) != 1:
            x2 = x2.contiguous()
        rows = x2.shape[0]
        if out is None:
            out = torch.empty((rows, self.n), dtype=torch.float32, device=x.device)
        dt = F32 if x.dtype == torch.float32 else F16
        st = _stream_handle(stream)
        if workspace is None:
            check(lib().exl3cu_mul_mat(self._h, _ptr(x2), dt, rows, x2.stride(0), _ptr(out), out.stride(0), st))
        else:
            check(lib().exl3cu_mul_mat_ws(self._h, _ptr(x2), dt, rows, x2.stride(0), _ptr(out), out.stride(0),
                                          _ptr(workspace), workspace.numel() * workspace.element_size(), st))
        return out

    def mul_mat_ragged(self, x: torch.Tensor, row_offsets: torch.Tensor, out: torch.Tensor | None = None,
                       stream=None) -> torch.Tensor:
        """y = x . W over the row_offsets[-1] packed rows of x [max_rows, k] (a count read on the
        device; exl3cu_mul_mat_ragged).  Rows of `out` at or past the count are not written."""
        if x.dtype not in (torch.float32, torch.float16):
            raise TypeError("x must be float32 or float16")
        if row_offsets.dtype != torch.int32 or row_offsets.dim() != 1 or row_offsets.numel() < 2:
            raise ValueError("row_offsets must be a 1-D int32 device tensor of n_seq + 1 entries")
        x2 = x if x.stride(-1) == 1 else x.contiguous()
        max_rows = x2.shape[0]
        if out is None:
            out = torch.empty((max_rows, self.n), dtype=torch.float32, device=x.device)
        dt = F32 if x.dtype == torch.float32 else F16
        check(lib().exl3cu_mul_mat_ragged(self._h, _ptr(x2), dt, x2.stride(0), _ptr(row_offsets),
                                          row_offsets.numel() - 1, max_rows, _ptr(out), out.stride(0),
                                          _stream_handle(stream)))
        return out

    def mul_mat_host(self, x: np.ndarray, out: np.ndarray | None = None, synchronize: bool = True,
                     stream=None) -> np.ndarray:
        """Host-buffer form (copies inside the call), the ggml CPU-backend contract."""
        x = np.ascontiguousarray(x)
        if x.dtype not in (np.float32, np.float16):
            raise TypeError("x must be float32 or float16")
        x2 = x.reshape(-1, x.shape[-1])
        rows = x2.shape[0]
        if out is None:
            out = np.empty((rows, self.n), np.float32)
        dt = F32 if x.dtype == np.float32 else F16
        check(lib().exl3cu_mul_mat_host(self._h, _ptr(x2), dt, rows, x2.shape[1], _ptr(out), out.shape[1],
                                        int(synchronize), _stream_handle(stream)))
        return out

    def get_rows(self, ids: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """Original-basis columns W[:, id] for each id as float32 rows [count, k]
        (exl3cu_get_rows; the reference's ggml_exl3_get_rows).  ids: int32 device tensor,
        local to this handle's columns; an id out of range gives a NaN row and sets bit 1
        of device_status()."""
        if ids.dtype != torch.int32:
            raise TypeError("ids must be int32")
        ids2 = ids.reshape(-1).contiguous()
        if out is None:
            out = torch.empty((ids2.numel(), self.k), dtype=torch.float32, device=ids.device)
        if out.dim() != 2 or out.stride(1) != 1 or out.shape[0] < ids2.numel() or out.shape[1] < self.k:
            raise ValueError("out must be a row-major float32 [count, >=k] tensor")
        check(lib().exl3cu_get_rows(self._h, _ptr(ids2), ids2.numel(), _ptr(out), out.stride(0),
                                    _stream_handle(stream)))
        return out

    def get_rows_host(self, ids: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
        """Host-buffer form of get_rows (ids checked on the host; synchronous)."""
        ids = np.ascontiguousarray(ids, dtype=np.int32).reshape(-1)
        if out is None:
            out = np.empty((ids.size, self.k), np.float32)
        check(lib().exl3cu_get_rows_host(self._h, _ptr(ids), ids.size, _ptr(out), out.shape[1], 1, None))
        return out

    def decode_inner(self, stream=None) -> np.ndarray:
        """The handle's device-layout weights decoded back to row-major inner fp16 bits [k, n]."""
        out = torch.empty((self.k, self.n), dtype=torch.int16, device=f"cuda:{self.device}")
        check(lib().exl3cu_weight_decode_inner(self._h, _ptr(out), _stream_handle(stream)))
        torch.cuda.synchronize(self.device)
        return out.cpu().numpy().view(np.uint16)


def mul_mat_batch(weights, xs, outs=None, stream=None):
    """Independent y_i = x_i . W_i in grouped launches (exl3cu_mul_mat_batch)."""
    n = len(weights)
    if len(xs) != n:
        raise ValueError("one activation tensor per weight")
    xs2 = []
    for x in xs:
        if x.dtype not in (torch.float32, torch.float16):
            raise TypeError("x must be float32 or float16")
        x2 = x.reshape(-1, x.shape[-1])
        xs2.append(x2 if x2.stride(-1) == 1 else x2.contiguous())
    if outs is None:
        outs = [torch.empty((x.shape[0], w.n), dtype=torch.float32, device=x.device) for w, x in zip(weights, xs2)]
    VP = ctypes.c_void_p * n
    SZ = ctypes.c_size_t * n
    IN = ctypes.c_int * n
    check(lib().exl3cu_mul_mat_batch(
        n, VP(*[w.handle.value for w in weights]), VP(*[x.data_ptr() for x in xs2]),
        IN(*[F32 if x.dtype == torch.float32 else F16 for x in xs2]), SZ(*[x.shape[0] for x in xs2]),
        SZ(*[x.stride(0) for x in xs2]), VP(*[o.data_ptr() for o in outs]), SZ(*[o.stride(0) for o in outs]),
        _stream_handle(stream)))
    return outs


# -- codec on device tensors (include/exl3_codec.h:10-29) ------------------------------------------

def decode_codebook(states, codebook: int = CB_MUL1, device: int = 0) -> np.ndarray:
    dev = f"cuda:{device}"
    s = _as_u16_tensor(states, dev).reshape(-1)
    out = torch.empty_like(s)
    check(lib().exl3cu_decode_codebook(_ptr(s), s.numel(), codebook, _ptr(out), _stream_handle(None)))
    return out.cpu().numpy().view(np.uint16)


def decode_inner(packed, k: int, n: int, bits: int, codebook: int = CB_MUL1, first_column: int = 0,
                 column_count: int | None = None, device: int = 0) -> np.ndarray:
    dev = f"cuda:{device}"
    p = _as_u16_tensor(packed, dev)
    cc = n - first_column if column_count is None else column_count
    out = torch.empty((k, max(cc, 0)), dtype=torch.int16, device=dev)
    check(lib().exl3cu_decode_inner(_ptr(p), k, n, first_column, cc, bits, codebook, _ptr(out), _stream_handle(None)))
    return out.cpu().numpy().view(np.uint16)


def hadamard128(values, device: int = 0) -> np.ndarray:
    t = torch.as_tensor(np.ascontiguousarray(values, np.float32)).to(f"cuda:{device}")
    check(lib().exl3cu_hadamard128(_ptr(t), t.numel(), _stream_handle(None)))
    return t.cpu().numpy()


def reconstruct(packed, suh, svh, k: int, n: int, bits: int, codebook: int = CB_MUL1, first_column: int = 0,
                column_count: int | None = None, device: int = 0) -> np.ndarray:
    dev = f"cuda:{device}"
    p, su, sv = (_as_u16_tensor(a, dev) for a in (packed, suh, svh))
    cc = n - first_column if column_count is None else column_count
    out = torch.empty((k, max(cc, 0)), dtype=torch.int16, device=dev)
    check(lib().exl3cu_reconstruct(_ptr(p), _ptr(su), _ptr(sv), k, n, first_column, cc, bits, codebook, _ptr(out),
                                   _stream_handle(None)))
    return out.cpu().numpy().view(np.uint16)


__all__ = ["Exl3Weight", "mul_mat_batch", "decode_codebook", "decode_inner", "hadamard128", "reconstruct", "_lib"]


def pack_ragged(want: torch.Tensor, pos: torch.Tensor, max_rows: int, stream=None,
                out: tuple | None = None):
    """GPU-side packer (exl3cu_pack_ragged): sequence i is granted min(want[i], rows left of
    max_rows) rows in order.  Returns (row_offsets [n_seq+1], row_seq [max_rows], row_pos [max_rows]),
    device int32; row_offsets[-1] is the packed row count, -1 marks rows past it."""
    if want.dtype != torch.int32 or pos.dtype != torch.int32 or want.shape != pos.shape or want.dim() != 1:
        raise ValueError("want and pos must be 1-D int32 device tensors of one length")
    n_seq = want.numel()
    if out is None:
        dev = want.device
        out = (torch.empty(n_seq + 1, dtype=torch.int32, device=dev),
               torch.empty(max_rows, dtype=torch.int32, device=dev),
               torch.empty(max_rows, dtype=torch.int32, device=dev))
    offs, rseq, rpos = out
    if not (want.is_contiguous() and pos.is_contiguous()):
        raise ValueError("want and pos must be contiguous")
    check(lib().exl3cu_pack_ragged(n_seq, _ptr(want), _ptr(pos), int(max_rows),
                                   _ptr(offs), _ptr(rseq), _ptr(rpos), _stream_handle(stream)))
    return offs, rseq, rpos


# -- plan and status ---------------------------------------------------------------------------

def gemm_config(min_rows: int = 0, tokens_per_cta: int = 0, splits: int = 0) -> None:
    """Process-wide overrides of the batched path (exl3cu_gemm_config): operands of at least
    `min_rows` rows use the tensor-core GEMM; tokens_per_cta (multiple of 32, <= 256) / splits
    replace its automatic plan (0 = automatic; min_rows 0 = unchanged)."""
    check(lib().exl3cu_gemm_config(int(min_rows), int(tokens_per_cta), int(splits)))


def device_status(device: int = 0, clear: bool = True) -> int:
    """Sticky kernel error bits of `device` (bit 0: a bounded wait ran out); synchronises it."""
    st = ctypes.c_uint(0)
    check(lib().exl3cu_device_status(int(device), ctypes.byref(st), int(bool(clear))))
    return st.value
