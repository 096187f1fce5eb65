"""Shared fixtures.

* ``pkg``    -- the product package (directory ``typhoon-ocr-server_b200``), imported by path.
* ``oracle`` -- the C restatement of the reference (oracle/liboracle.so); test infrastructure.
* ``ref``    -- the reference's own code built here (oracle/_ref), or skip when absent.
* ``lib``    -- the CUDA library, loaded; GPU tests only.

Tests that need a GPU carry ``@pytest.mark.gpu``; everything else runs on CPU.
"""

import importlib.util
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_DIR = ROOT / "typhoon-ocr-server_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(ROOT / "oracle"))


def load_pkg():
    name = "typhoon_ocr_server_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, PKG_DIR / "__init__.py",
                                                  submodule_search_locations=[str(PKG_DIR)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def pkg():
    return load_pkg()


@pytest.fixture(scope="session")
def oracle():
    import oracle as orc
    if not orc.ORACLE_LIB.exists():
        orc.build()
    return orc.Oracle()


@pytest.fixture(scope="session")
def ref():
    import oracle as orc
    if not orc.RefLib.available():
        pytest.skip("reference build oracle/_ref/libref_attn.so not present")
    return orc.RefLib()


@pytest.fixture(scope="session")
def golden():
    def _load(name):
        with np.load(GOLDEN / name) as z:
            return {k: z[k] for k in z.files}
    return _load


@pytest.fixture(scope="session")
def lib(pkg):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()
    return pkg.load_attention_lib()
