"""The C-ABI library: loads, exports every entry point the public headers
declare, and fails loudly (no CPU fallback) where no GPU is present."""
import re
from pathlib import Path

import numpy as np
import pytest

from conftest import HAS_GPU, ROOT

HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_functions(path: Path):
    text = path.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^[A-Za-z_][\w \*]*?\b(tos_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_headers_declare_entry_points():
    names = declared_functions(ROOT / "include" / "tensoros_nn_gpu.h")
    assert "tos_gemv" in names and "tos_model_forward_token" in names
    assert len(names) >= 50


def test_library_exports_every_declared_symbol(lib):
    from tensoros_b200 import _ffi
    missing = []
    for h in HEADERS:
        target = _ffi.synth() if h.name == "tos_synth.h" else lib
        for name in declared_functions(h):
            if not hasattr(target, name):
                missing.append(f"{h.name}:{name}")
    assert not missing, missing


def test_ctypes_table_matches_header():
    from tensoros_b200 import _ffi
    declared = set(declared_functions(ROOT / "include" / "tensoros_nn_gpu.h"))
    assert declared <= set(_ffi.NN_FUNCS), sorted(declared - set(_ffi.NN_FUNCS))
    declared = set(declared_functions(ROOT / "include" / "tos_synth.h"))
    assert declared <= set(_ffi.SYNTH_FUNCS)


def test_library_has_sm100a_kernels_only():
    """The product library carries sm_100a device code and no other arch."""
    import subprocess
    from tensoros_b200 import _build
    out = subprocess.run(["nvcc", "--version"], capture_output=True, text=True)
    assert out.returncode == 0
    assert "compute_100a,code=sm_100a" in " ".join(_build.ARCH).replace(" ", "")


def test_status_strings(lib):
    assert lib.tos_status_string(0) == b"ok"
    assert lib.tos_status_string(-7) == b"no CUDA device"


@pytest.mark.skipif(HAS_GPU, reason="checks the no-GPU behaviour")
def test_no_gpu_fails_loudly(lib):
    """Without a device the drop-ins report TOS_ENODEV and leave zeros; no
    result is ever computed on the CPU."""
    assert lib.tos_init(0) == -7
    out = np.full(4, 7.0, np.float32)
    w = np.zeros(4 * 18, np.uint8)
    x = np.ones(32, np.float32)
    lib.tos_gemv(out.ctypes.data, w.ctypes.data, x.ctypes.data, 4, 32, 2)
    assert lib.tos_last_status() == -7
    assert np.all(out == 0)
    v = np.ones(8, np.float32)
    lib.tos_softmax(v.ctypes.data, 8)
    assert lib.tos_last_status() == -7
    assert np.all(v == 1)


def test_invalid_arguments_rejected_on_host(lib):
    """Argument checks happen before any device work."""
    import ctypes
    h = ctypes.c_void_p()
    assert lib.tos_model_create(ctypes.byref(h), None) == -1
    assert lib.tos_attention_workspace_bytes(0, 16) == 0


def test_gemm_workspace_covers_shorter_batches(lib):
    """tos_gemm_workspace_bytes(m, ...) is enough for every call with at
    most m rows (a caller sizes one workspace for its longest batch); the
    size is host arithmetic, so this runs without a GPU."""
    for n, k in ((4096, 4096), (22016, 4096), (4096, 11008), (288, 768), (32000, 4096)):
        sizes = [lib.tos_gemm_workspace_bytes(m, n, k) for m in range(1, 300)]
        assert all(s > 0 for s in sizes)
        assert all(b >= a for a, b in zip(sizes, sizes[1:])), (n, k)
    assert lib.tos_gemm_workspace_bytes(16, 4096, 4000) == 0   # in_dim not a multiple of 64
