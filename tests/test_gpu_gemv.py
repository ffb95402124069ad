"""Q4_0 / Q8_0 GEMV on the GPU at the benchmark shapes, bit-exact against
the oracle (the restatement pinned to the reference by tests/golden)."""
import numpy as np
import pytest

from conftest import bits_equal, first_diff
from tensoros_b200 import ops
from tensoros_b200 import workloads as W

pytestmark = pytest.mark.gpu

SHAPES = [(W.TYPE_Q4_0, 4096, 4096)] + [(W.TYPE_Q8_0, r, c) for (r, c) in
                                        [(4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096)]]


@pytest.mark.parametrize("t,rows,cols", SHAPES)
def test_gemv_benchmark_shapes(gpu, oracle, t, rows, cols):
    w = W.quant(t, rows, cols, W.SEED, 500 + rows + cols)
    x = W.normal_f32(cols, W.SEED, 501)
    got = ops.gemv(w, x, rows, cols, t)
    ref = oracle.gemv_mt(w, x, rows, cols, t, threads=16)
    assert bits_equal(got, ref), first_diff(got, ref)


@pytest.mark.parametrize("t", [W.TYPE_Q4_0, W.TYPE_Q8_0])
@pytest.mark.parametrize("rows,cols", [(1, 32), (7, 64), (37, 288), (288, 768), (768, 288), (130, 8192), (3, 12288)])
def test_gemv_ragged_shapes(gpu, oracle, t, rows, cols):
    w = W.quant(t, rows, cols, W.SEED, 600 + rows)
    x = W.normal_f32(cols, W.SEED, 601 + cols)
    got = ops.gemv(w, x, rows, cols, t)
    assert bits_equal(got, oracle.gemv(w, x, rows, cols, t))


def test_gemv_special_values(gpu, oracle):
    """zero / subnormal / large scales and zero, subnormal, huge activations"""
    rows, cols = 24, 1024
    for t in (W.TYPE_Q4_0, W.TYPE_Q8_0):
        w = W.quant(t, rows, cols, 3, 700).copy()
        bs = W.BLOCK_BYTES[t]
        for i, h in enumerate([0x0000, 0x8000, 0x0001, 0x03FF, 0x7BFF, 0x0400]):
            w[bs * (i * 37)] = h & 0xFF
            w[bs * (i * 37) + 1] = h >> 8
        x = W.normal_f32(cols, 3, 701)
        x[:6] = [0.0, -0.0, 1e-40, -3e-39, 1e30, -1e30]
        got = ops.gemv(w, x, rows, cols, t)
        assert bits_equal(got, oracle.gemv(w, x, rows, cols, t))


def test_gemv_device_api_and_fused_norm(gpu, oracle):
    """tos_gemv_dev / tos_gemv_norm_dev with device pointers (torch tensors as
    plumbing) against oracle rmsnorm + gemv."""
    import ctypes
    import torch
    rows, cols, t = 1000, 4096, W.TYPE_Q4_0
    w = W.quant(t, rows, cols, 5, 800)
    x = W.normal_f32(cols, 5, 801)
    g = W.normal_f32(cols, 5, 802, 1.0, 0.1)
    h = ctypes.c_void_p()
    assert gpu.tos_weight_create(ctypes.byref(h), w.ctypes.data, rows, cols, t) == 0
    try:
        dx = torch.from_numpy(x).cuda()
        dg = torch.from_numpy(g).cuda()
        out = torch.empty(rows, device="cuda")
        s = torch.cuda.current_stream().cuda_stream
        assert gpu.tos_gemv_dev(h, dx.data_ptr(), out.data_ptr(), s) == 0
        torch.cuda.synchronize()
        assert bits_equal(out.cpu().numpy(), oracle.gemv(w, x, rows, cols, t))
        for eps in (1e-6, 1e-5):
            assert gpu.tos_gemv_norm_dev(h, dx.data_ptr(), dg.data_ptr(), eps, out.data_ptr(), s) == 0
            torch.cuda.synchronize()
            xn = oracle.rmsnorm(x, g, cols, 0, eps)
            assert bits_equal(out.cpu().numpy(), oracle.gemv(w, xn, rows, cols, t)), eps
    finally:
        gpu.tos_weight_destroy(h)


def test_weight_cache_tracks_pointer(gpu, oracle):
    """The drop-in caches registered weights by host pointer; clearing the
    cache picks up changed contents."""
    rows, cols, t = 64, 256, W.TYPE_Q8_0
    w = W.quant(t, rows, cols, 9, 900).copy()
    x = W.normal_f32(cols, 9, 901)
    assert bits_equal(ops.gemv(w, x, rows, cols, t), oracle.gemv(w, x, rows, cols, t))
    w[:] = W.quant(t, rows, cols, 9, 902)
    gpu.tos_weight_cache_clear()
    assert bits_equal(ops.gemv(w, x, rows, cols, t), oracle.gemv(w, x, rows, cols, t))
