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


def dequant(w: np.ndarray, t: int, rows: int, cols: int) -> np.ndarray:
    """GGUF Q4_0 / Q8_0 rows to float64 (llm.c:162-165, 199-200, 390-391)."""
    from tensoros_b200 import workloads as W
    nb = cols // 32
    if t == W.TYPE_Q4_0:
        b = w.reshape(rows, nb, 18)
        d = b[:, :, :2].copy().view(np.float16).astype(np.float64)
        q = b[:, :, 2:].astype(np.int64)
        vals = np.empty((rows, nb, 32), np.float64)
        vals[:, :, 0::2] = (q & 0xF) - 8
        vals[:, :, 1::2] = (q >> 4) - 8
    else:
        b = w.reshape(rows, nb, 34)
        d = b[:, :, :2].copy().view(np.float16).astype(np.float64)
        vals = b[:, :, 2:].copy().view(np.int8).astype(np.float64)
    return (vals * d).reshape(rows, cols)


FAST_TOL = 1e-4     # the FAST-arithmetic bound against the reference
FAST_FLOOR = 1e-3   # the literal per-element form: elements with |ref| above this share of max|ref|


def dequant_abs_matvec(w: np.ndarray, t: int, rows: int, cols: int, v) -> np.ndarray:
    """(|W| |v|)_i for a GGUF Q4_0 / Q8_0 matrix, in row chunks (float64):
    the magnitude of the terms each output element of W v sums."""
    v = np.abs(np.asarray(v, dtype=np.float64).ravel())
    bpr = (cols // 32) * (18 if t == 2 else 34)
    w2 = np.asarray(w).reshape(rows, bpr)
    out = np.empty(rows, np.float64)
    step = max(1, (1 << 24) // cols)
    for r0 in range(0, rows, step):
        r1 = min(rows, r0 + step)
        out[r0:r1] = np.abs(dequant(w2[r0:r1].ravel(), t, r1 - r0, cols)) @ v
    return out


def ref_expf64(x):
    """llm_expf (llm.c:123-131), (1 + x/256)^256, in float64."""
    x = np.asarray(x, np.float64)
    y = np.power(1.0 + x / 256.0, 256.0)
    return np.where(x > 88.0, 3.4e38, np.where(x < -88.0, 0.0, y))


def attention_abs_scale(q, kc, vc, kv_type, n_heads, n_kv, hd, pos) -> np.ndarray:
    """sum_t p_t |V_t[d]| for every output element of the decode attention
    (llm.c:683-714; p from the reference's exponential of s_t - max): the
    magnitude of the terms each element sums."""
    def rows(c):
        a = np.asarray(c)
        a = a.view(np.float16) if kv_type == 1 else a.view(np.float32)
        return a.astype(np.float64).reshape(-1, n_kv, hd)[:pos + 1]
    K, V = rows(kc), rows(vc)
    q = np.asarray(q, np.float64).reshape(n_heads, hd)
    g = n_heads // n_kv
    out = np.empty((n_heads, hd))
    for h in range(n_heads):
        s = K[:, h // g] @ q[h] / np.sqrt(hd)
        e = ref_expf64(s - s.max())
        out[h] = (e / e.sum()) @ np.abs(V[:, h // g])
    return out.ravel()


def logits_scale(synth, hidden) -> np.ndarray:
    """(|W_out| |x|)_i of the LM head (llm.c:737-742) for the normalised
    final hidden state x of a step (the oracle model's hidden())."""
    c = synth.cfg
    w, t = (synth.output, c["out_type"]) if synth.output is not None else (synth.token_embd, c["embd_type"])
    return dequant_abs_matvec(w, t, c["vocab_size"], c["dim"], hidden)


def fast_errors(got, ref, scale=None):
    """(normwise, per-element) errors of the FAST numerics contract.
    normwise = max|got - ref| / max|ref|.  per-element = max_i |got_i - ref_i|
    / scale_i, scale_i the magnitude of the terms element i sums (|W||x| for
    a GEMV row, sum_t p_t |V_t| for attention, the LM head's |W||x| for
    logits): the per-element error bound of any floating-point summation,
    which the reference's own fp32 result meets against the exact one.
    Without a scale the per-element figure is the literal form, over the
    elements with |ref| > FAST_FLOOR * max|ref|."""
    got = np.asarray(got, dtype=np.float64).ravel()
    ref = np.asarray(ref, dtype=np.float64).ravel()
    d = np.abs(got - ref)
    mx = float(np.max(np.abs(ref))) if ref.size else 0.0
    norm = float(np.max(d)) / (mx if mx > 0 else 1.0) if ref.size else 0.0
    if scale is not None:
        sc = np.asarray(scale, np.float64).ravel()
        elem = float(np.max(d / np.where(sc > 0, sc, 1.0))) if ref.size else 0.0
    else:
        big = np.abs(ref) > FAST_FLOOR * mx
        elem = float(np.max(d[big] / np.abs(ref[big]))) if np.any(big) else 0.0
    return norm, elem


def assert_fast(got, ref, tol=FAST_TOL, what="", scale=None):
    """The FAST bound: normwise <= tol and, given the terms' magnitudes,
    per-element |got_i - ref_i| <= tol * scale_i."""
    norm, elem = fast_errors(got, ref, scale)
    assert norm <= tol and (scale is None or elem <= tol), (what, "normwise", norm, "per-element", elem)
    return norm, elem
