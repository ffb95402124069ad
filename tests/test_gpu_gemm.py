"""Batched Q4_0 / Q8_0 GEMM on the tcgen05 tensor cores (prefill, batched
decode): Y = X W^T for M activation rows at once.  No counterpart in the
reference, which runs M GEMVs (llm.c:329-349); checked against the float64
product of the dequantised weights (normwise 1e-5; the hi/lo split and the
integer form for Q4_0 at up to 16 rows both deliver ~1e-6) and against the
oracle's GEMV rows (the 1e-4 FAST bound)."""
import ctypes

import numpy as np
import pytest

from conftest import assert_fast, dequant, dequant_abs_matvec
from tensoros_b200 import workloads as W

pytestmark = pytest.mark.gpu

TOL_TRUE = 1e-5   # vs the exact (float64) product
TOL_REF = 1e-4    # vs the reference GEMV, row by row


def normwise(got, ref):
    s = float(np.max(np.abs(ref)))
    return float(np.max(np.abs(got.astype(np.float64) - ref))) / (s if s > 0 else 1.0)


def run_gemm(gpu, w, t, n, k, x):
    import torch
    h = ctypes.c_void_p()
    assert gpu.tos_weight_create(ctypes.byref(h), w.ctypes.data, n, k, t) == 0
    try:
        m = x.shape[0]
        dx = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
        y = torch.empty((m, n), device="cuda")
        wsb = gpu.tos_gemm_workspace_bytes(m, n, k)
        ws = torch.empty(wsb + 256, dtype=torch.uint8, device="cuda")
        wp = (ws.data_ptr() + 255) & ~255
        s = torch.cuda.current_stream().cuda_stream
        outs = []
        for _ in range(2):
            assert gpu.tos_gemm_dev(h, dx.data_ptr(), m, y.data_ptr(), wp, wsb, s) == 0
            torch.cuda.synchronize()
            outs.append(y.cpu().numpy().copy())
    finally:
        gpu.tos_weight_destroy(h)
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32)), "deterministic"
    return outs[0]


@pytest.mark.parametrize("t,m,n,k", [
    (W.TYPE_Q4_0, 128, 4096, 4096),     # one prefill tile of the 7B q/o projections
    (W.TYPE_Q4_0, 16, 4096, 4096),      # batch-16 decode (integer form: Q4_0, <= 16 rows)
    (W.TYPE_Q4_0, 1, 4096, 4096),       # one row
    (W.TYPE_Q4_0, 16, 4096, 11008),     # batch-16 down projection
    (W.TYPE_Q4_0, 3, 19200, 512),       # 150 tiles: two cut into K slices, then the slice sum
    (W.TYPE_Q4_0, 12, 256, 384),        # three K chunks: a raw stage holding one
    (W.TYPE_Q4_0, 16, 4096, 4160),      # K not a multiple of 128: the fp16 hi / lo form
    (W.TYPE_Q4_0, 128, 4096, 11008),    # down projection
    (W.TYPE_Q4_0, 130, 2048, 4096),     # two M tiles, ragged
    (W.TYPE_Q4_0, 37, 288, 768),        # ragged N tile, short K
    (W.TYPE_Q8_0, 64, 4096, 4096),
    (W.TYPE_Q8_0, 5, 288, 288 // 64 * 64 + 64),
])
def test_gemm_matches_product(gpu, oracle, t, m, n, k):
    w = W.quant(t, n, k, W.SEED, 900 + n + k)
    x = np.stack([W.normal_f32(k, W.SEED, 950 + i) for i in range(m)])
    y = run_gemm(gpu, w, t, n, k, x)
    truth = x.astype(np.float64) @ dequant(w, t, n, k).T
    assert normwise(y, truth) <= TOL_TRUE, normwise(y, truth)
    for i in (0, m - 1):
        ref = oracle.gemv(w, x[i], n, k, t)
        assert_fast(y[i], ref, TOL_REF, ("gemm row", i), dequant_abs_matvec(w, t, n, k, x[i]))


def test_gemm_special_rows(gpu):
    """zero rows, rows of very different magnitudes, large scales"""
    t, m, n, k = W.TYPE_Q4_0, 8, 256, 512
    w = W.quant(t, n, k, 3, 990).copy()
    w[0:2] = np.frombuffer(np.float16(60.0).tobytes(), np.uint8)   # a large block scale in row 0
    x = np.stack([W.normal_f32(k, 3, 991 + i) for i in range(m)])
    x[1] = 0.0
    x[2] *= 1e-20
    x[3] *= 1e20
    x[4, ::7] *= 1000.0
    y = run_gemm(gpu, w, t, n, k, x)
    truth = x.astype(np.float64) @ dequant(w, t, n, k).T
    assert np.all(y[1] == 0.0)
    for i in range(m):
        if i != 1:
            assert normwise(y[i], truth[i]) <= TOL_TRUE, (i, normwise(y[i], truth[i]))
