"""CPU-only tests of the host side: the C ABI library loads and exports every
symbol include/exl3cu.h declares, argument validation that needs no GPU, the
ggml adapter library, and the host record-format helpers against the oracle."""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

import kat

ROOT = Path(__file__).resolve().parents[1]


def _declared(header: str, prefix: str):
    text = (ROOT / "include" / header).read_text()
    return sorted(set(re.findall(rf"\b({prefix}\w+)\s*\(", text)))


def test_c_abi_exports_every_declared_symbol():
    from exl3_b200 import _lib

    lib = _lib.lib()
    declared = _declared("exl3cu.h", "exl3cu_")
    assert declared, "no declarations parsed"
    for name in declared:
        assert hasattr(lib, name), name
    assert set(declared) == set(_lib.EXPORTS)
    assert lib.exl3cu_abi_version() == 1


def test_ggml_adapter_exports():
    from exl3_b200 import _lib

    _lib.lib()
    g = ctypes.CDLL(str(_lib.GGML_LIB_PATH))
    names = _declared("exl3-block.h", "ggml_exl3_")
    assert {"ggml_exl3_mul_mat", "ggml_exl3_get_rows"} <= set(names)
    for name in names:
        assert hasattr(g, name), name


def test_status_strings_and_validation_without_gpu():
    from exl3_b200 import _lib

    lib = _lib.lib()
    assert lib.exl3cu_status_string(0) == b"ok"
    assert lib.exl3cu_status_string(1) == b"invalid argument"
    h = ctypes.c_void_p()
    buf = (ctypes.c_uint8 * 16)()
    # bad bitrate / shape / short buffer are rejected before any device work
    assert lib.exl3cu_weight_from_records(buf, 16, 256, 384, 9, 2, 0, 0, 0, ctypes.byref(h)) == _lib.INVALID_ARGUMENT
    assert lib.exl3cu_weight_from_records(buf, 16, 200, 384, 4, 2, 0, 0, 0, ctypes.byref(h)) == _lib.INVALID_ARGUMENT
    assert lib.exl3cu_weight_from_records(buf, 16, 256, 384, 4, 2, 0, 0, 0, ctypes.byref(h)) == _lib.INVALID_ARGUMENT
    assert b"record buffer" in lib.exl3cu_last_error()
    assert lib.exl3cu_hadamard128(None, 100, None) == _lib.INVALID_ARGUMENT
    assert lib.exl3cu_decode_codebook(None, 4, 3, None, None) == _lib.INVALID_ARGUMENT
    assert lib.exl3cu_decode_inner(None, 16, 16, 16, 16, 4, 2, None, None) == _lib.INVALID_ARGUMENT
    assert lib.exl3cu_decode_inner(None, 16, 16, 0, 16, 0, 2, None, None) == _lib.INVALID_ARGUMENT
    assert lib.exl3cu_mul_mat(None, None, 0, 1, 128, None, 128, None) == _lib.INVALID_ARGUMENT
    # ragged entries: bounds are checked before any device call
    assert lib.exl3cu_pack_ragged(0, None, None, 8, None, None, None, None) == _lib.INVALID_ARGUMENT
    assert lib.exl3cu_pack_ragged(4, None, None, 0, None, None, None, None) == _lib.INVALID_ARGUMENT
    assert lib.exl3cu_pack_ragged(70000, None, None, 8, None, None, None, None) == _lib.INVALID_ARGUMENT
    assert lib.exl3cu_mul_mat_ragged(None, None, 1, 128, None, 1, 8, None, 128, None) == _lib.INVALID_ARGUMENT
    assert lib.exl3cu_gemm_config(0, 48, 0) == _lib.INVALID_ARGUMENT  # tokens per CTA: multiples of 32
    assert lib.exl3cu_gemm_config(0, 0, 3) == _lib.INVALID_ARGUMENT   # splits: powers of two


@pytest.mark.parametrize("bits", range(1, 9))
def test_pack_records_matches_oracle(oracle, bits):
    from exl3_b200 import format as fmt

    k, n = kat.KAT_K, kat.KAT_N
    packed = kat.kat_packed(bits)
    suh, svh = kat.kat_scales()
    rec = fmt.pack_records(packed, suh, svh, bits)
    assert rec.nbytes == fmt.records_nbytes(k, n, bits)
    assert np.array_equal(rec, oracle.pack_records(packed, suh, svh, k, n, bits))
    t2, su2, sv2 = fmt.unpack_records(rec, k, n, bits)
    assert np.array_equal(t2, packed) and np.array_equal(su2, suh) and np.array_equal(sv2, svh)


def test_format_rejects_bad_geometry():
    from exl3_b200 import format as fmt

    with pytest.raises(ValueError):
        fmt.pack_records(np.zeros((8, 8, 64), np.uint16), np.zeros(128, np.uint16), np.zeros(128, np.uint16), 5)
    with pytest.raises(ValueError):
        fmt.unpack_records(np.zeros(10, np.uint8), 100, 128, 4)


def test_synthetic_is_seeded():
    from exl3_b200 import synthetic

    a = synthetic.matrix(256, 384, 4, seed=7)
    b = synthetic.matrix(256, 384, 4, seed=7)
    assert np.array_equal(a.trellis, b.trellis) and np.array_equal(a.svh, b.svh)
    sv = a.svh.view(np.float16).astype(np.float32)
    assert np.all((np.abs(sv) >= 0.0099) & (np.abs(sv) <= 0.0301))
    assert set(np.unique(a.suh.view(np.float16).astype(np.float32))) == {-1.0, 1.0}
    assert synthetic.algorithmic_bytes(2048, 6144, 4) == 6336512  # configs[0]


def test_package_imports_without_gpu():
    import exl3_b200
    from exl3_b200 import ops

    assert exl3_b200.ops is ops and exl3_b200.Exl3Weight is ops.Exl3Weight
