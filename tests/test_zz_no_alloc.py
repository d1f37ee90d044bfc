"""The allocation-free operator entry, exl3cu_mul_mat_noalloc.

It exists for callers that may not allocate device memory on their call path
(a framework that owns and budgets all device memory up front, or a loop that
cannot take cudaFree's device-wide synchronisation): its split-K scratch is a
fixed array inside the library.  This file checks, through the C ABI, that it
gives the same y as exl3cu_mul_mat on two calls in a row, for weights whose plan
really splits K (so the scratch is used), and that it refuses a weight whose
plan needs more scratch than the array holds.  Each output is also held to the
CPU restatement of the reference operator.  The kernel resets its own arrival
tickets, so the clear before each call only matters after an aborted launch.
The file is named to be collected last so a run that stops at the first
failure has run every other test first.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL_MAX_ABS_REL = 2e-3  # the operator tolerance used by the other parity tests


def _rel(y, ref):
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def _noalloc(lib, w, x, y):
    return lib.exl3cu_mul_mat_noalloc(w.handle, ctypes.c_void_p(x.data_ptr()), 1, x.shape[0], x.stride(0),
                                      ctypes.c_void_p(y.data_ptr()), y.stride(0),
                                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.fixture(scope="module")
def env(cuda_lib):
    from exl3_b200 import _lib, ops, synthetic

    return _lib, ops, synthetic


STATIC_SCRATCH_BYTES = 4 << 20  # the library's fixed array


@pytest.mark.parametrize("k,n,bits,rows", [(4096, 1024, 4, 1), (2048, 6144, 4, 1), (6144, 2048, 3, 5)])
def test_noalloc_matches_mul_mat_twice(env, oracle, k, n, bits, rows):
    _lib, ops, synthetic = env
    lib = _lib.lib()
    m = synthetic.matrix(k, n, bits, seed=k + n + bits)
    rec = m.records()
    w = ops.Exl3Weight.from_records(rec, k, n, bits)
    assert w.workspace_bytes > 0, "shape chosen so the split-K scratch is used"
    if w.workspace_bytes > STATIC_SCRATCH_BYTES:
        pytest.skip(f"this GPU's split-K plan needs {w.workspace_bytes} bytes, beyond the static array")
    xh = synthetic.activations(rows, k, seed=rows)
    x = torch.from_numpy(xh).cuda()
    ref = w.mul_mat(x).cpu().numpy()
    # the CPU restatement of the reference operator, so the bound is 2e-3 against it, not transitive
    ref_oracle = oracle.mul_mat(rec, bits, k, n, xh)
    outs = []
    for _ in range(2):  # two calls in a row share the static scratch
        y = torch.full((rows, n), float("nan"), dtype=torch.float32, device="cuda")
        _lib.check(_noalloc(lib, w, x, y))
        torch.cuda.synchronize()
        outs.append(y.cpu().numpy())
    for y in outs:
        assert np.all(np.isfinite(y))
        assert _rel(y, ref) <= TOL_MAX_ABS_REL
        assert _rel(y, ref_oracle) <= TOL_MAX_ABS_REL
    w.free()


def test_noalloc_rejects_plans_beyond_the_scratch(env, monkeypatch):
    _lib, ops, synthetic = env
    lib = _lib.lib()
    # one 16-row chunk per split: the plan needs 8 MiB of partials, beyond the 4 MiB array
    monkeypatch.setitem(os.environ, "EXL3CU_GEMV_CPS", "1")
    k, n = 4096, 1024
    m = synthetic.matrix(k, n, 4, seed=5)
    w = ops.Exl3Weight.from_records(m.records(), k, n, 4)
    x = torch.zeros((1, k), dtype=torch.float16, device="cuda")
    y = torch.zeros((1, n), dtype=torch.float32, device="cuda")
    rc = _noalloc(lib, w, x, y)
    assert rc == _lib.NO_SUPPORT
    assert b"static scratch" in lib.exl3cu_last_error()
    w.free()
