"""Shared test plumbing: the `gpu` marker, the backend package and the C oracle.

The oracle (oracle/liboracle.so) is the CPU restatement of the reference's
token loop; tests use it only as the checker of the CUDA path.
"""
import ctypes
import importlib.util
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "plamo-3-translate.c_b200")
ORACLE_DIR = os.path.join(ROOT, "oracle")
# Checkout of the reference project whose own tests pin the oracle, the loader and
# the tokenizer: $PLAMO_REFERENCE, else a "reference" directory beside this
# repository (absent on GPU hosts: those tests skip).
REF = os.environ.get("PLAMO_REFERENCE") or os.path.join(os.path.dirname(ROOT), "reference")
sys.path.insert(0, os.path.join(ROOT, "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def load_package():
    if "plamo_b200" in sys.modules:
        return sys.modules["plamo_b200"]
    spec = importlib.util.spec_from_file_location(
        "plamo_b200", os.path.join(PKG_DIR, "__init__.py"), submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["plamo_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


_oracle = None


def load_oracle():
    """ctypes handle of the C oracle, built on first use when missing."""
    global _oracle
    if _oracle is not None:
        return _oracle
    path = os.path.join(ORACLE_DIR, "liboracle.so")
    if not os.path.exists(path):
        subprocess.run(["make", "-C", ORACLE_DIR], check=True, capture_output=True)
    lib = ctypes.CDLL(path)
    P, U64 = ctypes.c_void_p, ctypes.c_uint64
    sig = {
        "plamo_forward": (ctypes.c_int, [P, U64]),
        "plamo_forward_hidden": (ctypes.c_int, [P, U64]),
        "plamo_prefill": (ctypes.c_int, [P, P, U64, P]),
        "plamo_bf16_matvec": (None, [P, P, P, U64, U64]),
        "plamo_argmax": (U64, [P, U64]),
        "plamo_rmsnorm": (None, [P, P, P, U64, ctypes.c_float, ctypes.c_float]),
        "plamo_exp": (ctypes.c_float, [ctypes.c_float]),
        "plamo_rope_table": (None, [P, U64, U64, P, P, ctypes.c_float]),
        "oracle_set_threads": (None, [ctypes.c_int]),
        "plamo_cache_rope": (None, [P, ctypes.c_float]),
        "oracle_synthetic_bf16": (None, [P, U64, U64, ctypes.c_float, ctypes.c_float, ctypes.c_int]),
        "oracle_set_matvec_lanes": (None, [ctypes.c_int]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    _oracle = lib
    return lib


def rel_l2(actual, expected):
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    den = float(np.sum(e * e))
    return float(np.sqrt(np.sum((a - e) ** 2) / (den if den else 1.0)))


def assert_close(actual, expected, name, rel=1e-4, absolute=1e-5):
    """The reference's GPU acceptance rule (reference tests/metal_decode.c:192-230):
    finite values, relative L2 <= 1e-4 and max |delta| <= 1e-5 * (1 + max |ref|)."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    assert a.shape == e.shape, name
    assert np.all(np.isfinite(a)) and np.all(np.isfinite(e)), f"{name}: non-finite values"
    r = rel_l2(a, e)
    m = float(np.max(np.abs(a - e))) if a.size else 0.0
    mag = float(np.max(np.abs(e))) if e.size else 0.0
    assert r <= rel and m <= absolute * (1 + mag), \
        f"{name}: relative L2 {r:.3g}, max error {m:.3g}, magnitude {mag:.3g}"


@pytest.fixture(scope="session")
def pkg():
    return load_package()


@pytest.fixture(scope="session")
def oracle():
    return load_oracle()


@pytest.fixture
def backend(pkg):
    b = pkg.Backend(device=0, max_context=4200, max_prefill=4096)
    yield b
    b.close()


def expect(backend, rc, want=1):
    """Assert a tri-state return code, reporting the backend's last note."""
    assert rc == want, f"returned {rc}, expected {want}: {backend.info().note.decode()}"
