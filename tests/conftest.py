import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))
GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: takes more than a few seconds")


def _gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


HAS_GPU = _gpu_available()


def pytest_collection_modifyitems(config, items):
    if HAS_GPU:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session", autouse=True)
def built():
    """Build the product and the CPU checkers if they are missing (no-op when
    the prebuilt libraries travelled with the tree)."""
    from tensoros_b200 import _build
    _build.build_synth()
    _build.build_oracle()
    if not _build.LIB_NN.exists() or os.environ.get("TOS_REBUILD"):
        _build.build_nn()
    return True


@pytest.fixture(scope="session")
def oracle():
    import pyoracle
    return pyoracle.oracle()


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN / "ops.npz")


@pytest.fixture(scope="session")
def lib():
    from tensoros_b200 import _ffi
    return _ffi.nn()


@pytest.fixture(scope="session")
def gpu(lib):
    """Initialises the library on cuda:0 (GPU tests only)."""
    st = lib.tos_init(0)
    assert st == 0, f"tos_init failed: {st}"
    return lib


def bits_equal(a, b) -> bool:
    """Bitwise equality of float32 arrays, NaN payloads ignored."""
    a = np.asarray(a, dtype=np.float32).ravel()
    b = np.asarray(b, dtype=np.float32).ravel()
    if a.shape != b.shape:
        return False
    nan = np.isnan(a) & np.isnan(b)
    return bool(np.all((a.view(np.uint32) == b.view(np.uint32)) | nan))


def first_diff(a, b):
    a = np.asarray(a, dtype=np.float32).ravel()
    b = np.asarray(b, dtype=np.float32).ravel()
    bad = np.nonzero((a.view(np.uint32) != b.view(np.uint32)) & ~(np.isnan(a) & np.isnan(b)))[0]
    if len(bad) == 0:
        return None
    i = int(bad[0])
    return f"{len(bad)} differ; first at {i}: {a[i]!r} vs {b[i]!r}"


FAST_TOL = 1e-4     # the FAST-arithmetic bound against the reference
FAST_FLOOR = 1e-3   # per-element part: elements with |ref| above this share of max|ref|


def fast_errors(got, ref):
    """The two halves of the FAST numerics contract: the normwise error
    max|got - ref| / max|ref|, and the largest per-element relative error
    |got - ref| / |ref| over the elements with |ref| > FAST_FLOOR * max|ref|."""
    got = np.asarray(got, dtype=np.float64).ravel()
    ref = np.asarray(ref, dtype=np.float64).ravel()
    d = np.abs(got - ref)
    scale = float(np.max(np.abs(ref))) if ref.size else 0.0
    norm = float(np.max(d)) / (scale if scale > 0 else 1.0) if ref.size else 0.0
    big = np.abs(ref) > FAST_FLOOR * scale
    elem = float(np.max(d[big] / np.abs(ref[big]))) if np.any(big) else 0.0
    return norm, elem


def assert_fast(got, ref, tol=FAST_TOL, what=""):
    """Both halves of the FAST bound: normwise <= tol and per-element <= tol
    where |ref| > 1e-3 * max|ref|."""
    norm, elem = fast_errors(got, ref)
    assert norm <= tol and elem <= tol, (what, "normwise", norm, "per-element", elem)
    return norm, elem

