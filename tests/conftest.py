import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_DIR = ROOT / "xiaomi-hexagon-exl3_b200"
for p in (str(ROOT), str(PKG_DIR), str(ROOT / "tests" / "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")
    config.addinivalue_line("markers", "multigpu: needs 2 or more CUDA devices")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle, build

    if not (ROOT / "oracle" / "liboracle.so").exists():
        build()
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import Reference, have_reference

    if not have_reference():
        pytest.skip("oracle/_ref not built (reference sources absent)")
    return Reference()


@pytest.fixture(scope="session")
def golden():
    import json

    import numpy as np

    z = np.load(ROOT / "tests" / "golden" / "exl3_golden.npz")
    data = {k: z[k] for k in z.files}
    meta = json.loads(bytes(data.pop("meta_json")).decode())
    return data, meta


@pytest.fixture(scope="session")
def cuda_lib():
    """The shipped C-ABI library; GPU tests require a device."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from exl3_b200 import _lib

    return _lib.lib()


def pytest_collection_modifyitems(config, items):
    if os.environ.get("EXL3_ALLOW_NO_GPU"):
        return
