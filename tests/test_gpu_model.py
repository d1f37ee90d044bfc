"""The deployment loader on the GPU: every EXL3 matrix of a mixed-bit model
uploaded at its own bit width (decode bit-exact, mul_mat within the operator
tolerance, against the oracle fed the same file bytes), the tied-head
embedding (bit-exact against the oracle and the reference reader test's
known answer), plain tensors in the device arena, and exl3::Model from C++.
"""
import ctypes
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

import model_dir as md

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
TOL_MAX_ABS_REL = 2e-3
TOL_NMSE = 1e-5


@pytest.fixture(scope="module")
def mixed(cuda_lib, tmp_path_factory):
    from exl3_b200.model import Exl3Model
    from oracle.model_reader import read_model

    d = tmp_path_factory.mktemp("mixed")
    md.mixed_model().write(d)
    return Exl3Model(d, device=0), read_model(d)


def _records(oracle, info, name, k, n, bits):
    tr = info.array(name + ".trellis")
    su = info.array(name + ".suh").view(np.uint16)
    sv = info.array(name + ".svh").view(np.uint16)
    return oracle.pack_records(tr, su, sv, k, n, bits), tr


def test_every_matrix_decodes_bit_exact_and_multiplies(mixed, oracle):
    m, info = mixed
    assert [x.name for x in m.matrices()] == [x.name for x in info.matrices]
    for x in m.matrices():
        w = m.weight(x.name)
        assert (w.k, w.n, w.bits, w.codebook) == (x.k, x.n, x.bits, x.codebook)
        rec, tr = _records(oracle, info, x.name, x.k, x.n, x.bits)
        assert np.array_equal(w.decode_inner(), oracle.decode_inner(tr, x.k, x.n, x.bits, x.codebook)), x.name
        xin = np.random.default_rng(x.k + x.n).standard_normal((3, x.k)).astype(np.float16)
        y = w.mul_mat(torch.from_numpy(xin).cuda())
        torch.cuda.synchronize()
        ref = oracle.mul_mat(rec, x.bits, x.k, x.n, xin, codebook=x.codebook).astype(np.float64)
        yy = y.cpu().numpy().astype(np.float64)
        rel = np.max(np.abs(yy - ref)) / np.max(np.abs(ref))
        nmse = np.sum((yy - ref) ** 2) / np.sum(ref ** 2)
        assert rel <= TOL_MAX_ABS_REL and nmse < TOL_NMSE, (x.name, rel, nmse)


def test_embedding_matches_oracle(mixed, oracle):
    m, info = mixed
    k, n = m.hidden_size(), m.vocab_size()
    head = next(x for x in info.matrices if x.name == info.head)
    rec, _ = _records(oracle, info, head.name, k, n, head.bits)
    ids = np.array([0, 1, 127, 128, 300, n - 1], np.int32)
    ref = oracle.get_rows(rec, head.bits, k, n, ids, codebook=head.codebook)
    for i, t in enumerate(ids):
        e = m.embedding(int(t))
        assert e.dtype == np.uint16 and e.shape == (k,)
        assert np.array_equal(e.view(np.float16).astype(np.float32), ref[i]), t
    got = m.embed(torch.from_numpy(ids).cuda())
    torch.cuda.synchronize()
    assert np.array_equal(got.cpu().numpy(), ref)
    with pytest.raises(Exception, match="outside vocabulary"):
        m.embedding(n)


def test_plain_tensors_live_in_the_device_arena(mixed):
    m, info = mixed
    for t in m.tensors():
        part = any(t.name.startswith(x.name + ".") for x in info.matrices)
        if part:
            assert t.device_ptr == 0
            continue
        assert t.device_ptr and t.device_ptr % 256 == 0
        dev = m.tensor(t.name)
        assert tuple(dev.shape) == t.shape
        host = dev.cpu()
        want = info.array(t.name)
        if t.dtype == "BF16":
            assert np.array_equal(host.view(torch.int16).numpy().view(np.uint16), want)
        else:
            assert np.array_equal(host.numpy(), want)


def test_model_owned_weights_are_not_freed_alone(mixed):
    from exl3_b200 import _lib

    m, _ = mixed
    w = m.weight(m.head_name)
    assert _lib.lib().exl3cu_weight_free(w.handle) == _lib.INVALID_ARGUMENT
    assert b"belongs to a model" in _lib.lib().exl3cu_last_error()


def test_reference_reader_known_answer(cuda_lib, oracle, tmp_path):
    """tests/test_model_reader.cpp:44-50: zero trellis, unit scales -> row0[0] = fp16(code * 128),
    the rest of row 0 and all of row 1 zero; token 128 rejected."""
    from exl3_b200.model import Exl3Model

    md.reference_fixture().write(tmp_path)
    m = Exl3Model(tmp_path)
    code = float(oracle.codebook_table(2)[0:1].view(np.float16)[0])
    row0, row1 = m.embedding(0), m.embedding(1)
    assert np.array_equal(row0, m.embedding(0))
    assert row0[0] == np.float16(code * 128).view(np.uint16)
    assert np.all(row0[1:].view(np.float16) == 0) and np.all(row1.view(np.float16) == 0)
    with pytest.raises(Exception):
        m.embedding(128)
    m.close()


def test_cpp_model_class(cuda_lib, oracle, tmp_path):
    """exl3::Model (include/exl3_model.h) compiled as a C++ program, run on the reference's fixture
    and its four malformed variants."""
    import copy

    gxx = shutil.which("g++")
    if not gxx:
        pytest.skip("no g++")
    from exl3_b200 import _lib

    pkg = _lib.LIB_PATH.parent
    exe = tmp_path / "model_reader_check"
    subprocess.run([gxx, "-std=c++17", "-O1", f"-I{ROOT / 'include'}", str(ROOT / "tests" / "cpp" /
                    "model_reader_check.cpp"), "-o", str(exe), f"-L{pkg}", "-lexl3cu", f"-Wl,-rpath,{pkg}"],
                   check=True)
    d = md.reference_fixture()
    d.write(tmp_path / "ok")
    bad = []
    for i, mut in enumerate((lambda x: x.manifest.update(reference_parameter_count=1),
                             lambda x: x.header_patch.update({"lm_head.suh": {"data_offsets": [8190, 8446]}}),
                             lambda x: x.header_patch.update({"lm_head.suh": {"shape": [-128]}}),
                             lambda x: setattr(x, "truncate", 1))):
        b = copy.deepcopy(d)
        mut(b)
        b.write(tmp_path / f"bad{i}")
        bad.append(str(tmp_path / f"bad{i}"))
    code = float(oracle.codebook_table(2)[0:1].view(np.float16)[0])
    code16 = int(np.float16(code * 128).view(np.uint16))
    r = subprocess.run([str(exe), str(tmp_path / "ok"), str(code16), *bad], capture_output=True, text=True)
    assert r.returncode == 0 and "PASS" in r.stdout, r.stdout + r.stderr
