"""The reference's GPU dispatch entry points (kernel/drivers/gpu/gpu.c:
155-225: gpu_tensor_matmul / attention / softmax / layernorm / elementwise,
stubs there) backed by the library: the results of the engine's CPU
operators (runtime/tensor/tensor_cpu.c), bit for bit
(tests/golden/engine.npz, the reference's outputs for the seeded cases of
tests/engine_cases.py), for tensors in host memory (device_id 0) and in
device memory (device_id 1)."""
import ctypes as C

import numpy as np
import pytest

import engine_cases as E
from conftest import GOLDEN, bits_equal, first_diff
from tensoros_b200 import _ffi

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN / "engine.npz")


class Tensors:
    """Descriptors over numpy arrays (host) or torch tensors (device)."""

    def __init__(self, device):
        self.device, self.keep = device, []

    def desc(self, a, shape=None):
        d = _ffi.TensorDesc()
        a = np.ascontiguousarray(a, np.float32) if not self.device else a
        shp = shape if shape is not None else a.shape
        d.ndim = len(shp)
        for i, v in enumerate(shp):
            d.shape[i] = v
        d.dtype = 0
        if self.device:
            d.data_virt = a.data_ptr()
            d.device_id = 1
        else:
            d.data_virt = a.ctypes.data
        d.size_bytes = int(np.prod(shp)) * 4
        self.keep.append(a)
        return d

    def array(self, a):
        if not self.device:
            return np.ascontiguousarray(a, np.float32)
        import torch
        return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()

    def empty(self, shape):
        if not self.device:
            return np.full(shape, np.nan, np.float32)
        import torch
        return torch.full(shape, float("nan"), device="cuda")

    def host(self, a):
        if not self.device:
            return a
        import torch
        torch.cuda.synchronize()
        return a.cpu().numpy()


@pytest.mark.parametrize("device", [0, 1])
def test_matmul(gpu, g, device):
    lib, T = _ffi.nn(), Tensors(device)
    for M, N, K in E.MATMUL:
        A, B = E.matmul_case(M, N, K)
        a, b, c = T.array(A), T.array(B), T.empty((M, N))
        dc = T.desc(c, (1,))   # tensor_matmul sets the output's shape
        assert lib.tos_gpu_tensor_matmul(0, C.byref(dc), C.byref(T.desc(a)), C.byref(T.desc(b))) == 0
        assert dc.ndim == 2 and dc.shape[0] == M and dc.shape[1] == N and dc.size_bytes == M * N * 4
        got = T.host(c)
        assert bits_equal(got, g[f"matmul_{M}_{N}_{K}"]), ((M, N, K), first_diff(got, g[f"matmul_{M}_{N}_{K}"]))


@pytest.mark.parametrize("device", [0, 1])
def test_softmax_layernorm_attention(gpu, g, device):
    lib, T = _ffi.nn(), Tensors(device)
    for rows, n in E.SOFTMAX:
        x = T.array(E.softmax_case(rows, n))
        o = T.empty((rows, n))
        assert lib.tos_gpu_tensor_softmax(0, C.byref(T.desc(o)), C.byref(T.desc(x)), -1) == 0
        assert bits_equal(T.host(o), g[f"softmax_{rows}_{n}"]), (rows, n)
    for rows, n in E.LAYERNORM:
        x = T.array(E.layernorm_case(rows, n))
        o = T.empty((rows, n))
        none = _ffi.TensorDesc()
        assert lib.tos_gpu_tensor_layernorm(0, C.byref(T.desc(o)), C.byref(T.desc(x)), C.byref(none), C.byref(none),
                                            E.EPS) == 0
        assert bits_equal(T.host(o), g[f"layernorm_{rows}_{n}"]), (rows, n)
    for seq, hd in E.ATTENTION:
        q, k, v = (T.array(t) for t in E.attention_case(seq, hd))
        o = T.empty((seq, hd))
        assert lib.tos_gpu_tensor_attention(0, C.byref(T.desc(o)), C.byref(T.desc(q)), C.byref(T.desc(k)),
                                            C.byref(T.desc(v)), 0.0) == 0
        got = T.host(o)
        assert bits_equal(got, g[f"attention_{seq}_{hd}"]), ((seq, hd), first_diff(got, g[f"attention_{seq}_{hd}"]))


def test_layernorm_affine_and_elementwise(gpu, g):
    """gamma / beta applied per element after the engine's normalisation
    (one fp32 multiply and add each), and the four element-wise ops: IEEE
    single precision, as numpy computes them."""
    lib, T = _ffi.nn(), Tensors(0)
    rows, n = E.LAYERNORM[0]
    x = E.layernorm_case(rows, n)
    gm = (np.arange(n, dtype=np.float32) / n + 0.5).astype(np.float32)
    bt = (np.arange(n, dtype=np.float32) / n - 0.25).astype(np.float32)
    o = T.empty((rows, n))
    assert lib.tos_gpu_tensor_layernorm(0, C.byref(T.desc(o)), C.byref(T.desc(x)), C.byref(T.desc(gm)),
                                        C.byref(T.desc(bt)), E.EPS) == 0
    want = (g[f"layernorm_{rows}_{n}"] * gm + bt).astype(np.float32)
    assert bits_equal(o, want)
    a, b = E.matmul_case(16, 16, 16)
    for op, f in enumerate([np.add, np.multiply, np.subtract, np.divide]):
        o = T.empty(a.shape)
        assert lib.tos_gpu_tensor_elementwise(0, C.byref(T.desc(o)), C.byref(T.desc(a)), C.byref(T.desc(b)), op) == 0
        assert bits_equal(o, f(a, b).astype(np.float32)), op


def test_rejects(gpu):
    lib, T = _ffi.nn(), Tensors(0)
    a = np.ones((4, 8), np.float32)
    b = np.ones((4, 8), np.float32)
    c = np.empty((4, 8), np.float32)
    assert lib.tos_gpu_tensor_matmul(0, C.byref(T.desc(c)), C.byref(T.desc(a)), C.byref(T.desc(b))) == -1   # K mismatch
    assert lib.tos_gpu_tensor_matmul(3, C.byref(T.desc(c)), C.byref(T.desc(a)), C.byref(T.desc(a.T.copy()))) == -1
    assert lib.tos_gpu_tensor_elementwise(0, C.byref(T.desc(c)), C.byref(T.desc(a)), C.byref(T.desc(b)), 4) == -1
