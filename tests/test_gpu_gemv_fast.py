"""FAST GEMV arithmetic (TOS_GEMV_FAST): integer block dot products on 24-bit
fixed-point activations and tree row sums.  Bound: normwise relative error
max|gpu - ref| / max|ref| <= 1e-4 against the oracle (the restatement pinned to
the reference), deterministic results, and greedy decode identical to the
reference's."""
import ctypes

import numpy as np
import pytest

from conftest import GOLDEN, assert_fast, dequant_abs_matvec, logits_scale
from tensoros_b200 import ops
from tensoros_b200 import workloads as W

pytestmark = pytest.mark.gpu

TOL = 1e-4      # FAST-mode bound: max|gpu - ref| / max|ref|
TYPICAL = 2e-6  # what the arithmetic delivers on N(0,1) activations (~1e-7 measured)
FAST = 1

SHAPES = [(W.TYPE_Q4_0, 4096, 4096), (W.TYPE_Q4_0, 22016, 4096), (W.TYPE_Q4_0, 4096, 11008)] + \
         [(W.TYPE_Q8_0, r, c) for (r, c) in [(4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096)]]


def normwise(got, ref):
    scale = float(np.max(np.abs(ref)))
    return float(np.max(np.abs(got.astype(np.float64) - ref))) / (scale if scale > 0 else 1.0)


class DevGemv:
    """One registered weight and device buffers; calls tos_gemv_mode_dev."""

    def __init__(self, gpu, w, rows, cols, t):
        import torch
        self.torch, self.gpu, self.rows, self.cols = torch, gpu, rows, cols
        self.h = ctypes.c_void_p()
        assert gpu.tos_weight_create(ctypes.byref(self.h), w.ctypes.data, rows, cols, t) == 0

    def __call__(self, x, mode, norm_w=None, eps=1e-6):
        torch = self.torch
        dx = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()
        dg = torch.from_numpy(norm_w).cuda() if norm_w is not None else None
        out = torch.empty(self.rows, device="cuda")
        s = torch.cuda.current_stream().cuda_stream
        st = self.gpu.tos_gemv_mode_dev(self.h, dx.data_ptr(), dg.data_ptr() if dg is not None else None,
                                        eps, out.data_ptr(), mode, s)
        assert st == 0, st
        torch.cuda.synchronize()
        return out.cpu().numpy()

    def close(self):
        self.gpu.tos_weight_destroy(self.h)


@pytest.mark.parametrize("t,rows,cols", SHAPES)
def test_fast_gemv_shapes(gpu, oracle, t, rows, cols):
    w = W.quant(t, rows, cols, W.SEED, 500 + rows + cols)
    x = W.normal_f32(cols, W.SEED, 501)
    ref = oracle.gemv_mt(w, x, rows, cols, t, threads=16)
    g = DevGemv(gpu, w, rows, cols, t)
    try:
        a = g(x, FAST)
        b = g(x, FAST)
    finally:
        g.close()
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), "FAST results must be deterministic"
    err, _ = assert_fast(a, ref, TOL, (t, rows, cols), dequant_abs_matvec(w, t, rows, cols, x))
    assert err <= TYPICAL, err


@pytest.mark.parametrize("t", [W.TYPE_Q4_0, W.TYPE_Q8_0])
@pytest.mark.parametrize("rows,cols", [(1, 32), (7, 64), (37, 288), (288, 768), (768, 288), (130, 8192), (3, 12288)])
def test_fast_gemv_ragged(gpu, oracle, t, rows, cols):
    w = W.quant(t, rows, cols, W.SEED, 600 + rows)
    x = W.normal_f32(cols, W.SEED, 601 + cols)
    g = DevGemv(gpu, w, rows, cols, t)
    try:
        got = g(x, FAST)
    finally:
        g.close()
    assert_fast(got, oracle.gemv(w, x, rows, cols, t), TOL, (t, rows, cols), dequant_abs_matvec(w, t, rows, cols, x))


def test_fast_gemv_special_activations(gpu, oracle):
    """zero vector (exact zeros), outliers, subnormal and huge activations in
    one block, blocks of very different magnitudes"""
    rows, cols = 64, 1024
    for t in (W.TYPE_Q4_0, W.TYPE_Q8_0):
        w = W.quant(t, rows, cols, 3, 700)
        g = DevGemv(gpu, w, rows, cols, t)
        try:
            z = g(np.zeros(cols, np.float32), FAST)
            assert np.all(z == 0.0)
            x = W.normal_f32(cols, 3, 701)
            x[:6] = [0.0, -0.0, 1e-40, -3e-39, 1e30, -1e30]
            assert_fast(g(x, FAST), oracle.gemv(w, x, rows, cols, t), TOL, "special values",
                        dequant_abs_matvec(w, t, rows, cols, x))
            x = W.normal_f32(cols, 3, 702)
            x[::97] *= 100.0                 # outlier features
            x[256:512] *= 1e-6               # a quiet stretch
            assert_fast(g(x, FAST), oracle.gemv(w, x, rows, cols, t), TOL, "outliers",
                        dequant_abs_matvec(w, t, rows, cols, x))
        finally:
            g.close()


def test_fast_gemv_fused_norm(gpu, oracle):
    rows, cols, t = 1000, 4096, W.TYPE_Q4_0
    w = W.quant(t, rows, cols, 5, 800)
    x = W.normal_f32(cols, 5, 801)
    gw = W.normal_f32(cols, 5, 802, 1.0, 0.1)
    g = DevGemv(gpu, w, rows, cols, t)
    try:
        for eps in (1e-6, 1e-5):
            got = g(x, FAST, gw, eps)
            xn = oracle.rmsnorm(x, gw, cols, 0, eps)
            assert_fast(got, oracle.gemv(w, xn, rows, cols, t), TOL, ("fused norm", eps),
                        dequant_abs_matvec(w, t, rows, cols, xn))
        # EXACT through the same entry point is bit-identical to tos_gemv_norm_dev's contract
        exact = g(x, 0, gw, 1e-6)
        xn = oracle.rmsnorm(x, gw, cols, 0, 1e-6)
        assert np.array_equal(exact.view(np.uint32), oracle.gemv(w, xn, rows, cols, t).view(np.uint32))
    finally:
        g.close()


def test_fast_gemv_rejects_bad_mode(gpu):
    rows, cols, t = 8, 64, W.TYPE_Q8_0
    w = W.quant(t, rows, cols, 1, 1)
    g = DevGemv(gpu, w, rows, cols, t)
    try:
        import torch
        dx = torch.zeros(cols, device="cuda")
        out = torch.empty(rows, device="cuda")
        st = gpu.tos_gemv_mode_dev(g.h, dx.data_ptr(), None, 1e-6, out.data_ptr(), 7,
                                   torch.cuda.current_stream().cuda_stream)
        assert st != 0
    finally:
        g.close()


def test_tiny_llama_fast_greedy_matches_reference(gpu, oracle):
    """FAST GEMV + FAST attention: the greedy ids of the reference's own run
    (golden), and first-step logits within the bound (per-element scale:
    the LM head's terms, from the oracle's hidden state of the same step)."""
    g = np.load(GOLDEN / "tiny_llama.npz")
    m = W.make_model(W.TINY_LLAMA, int(g["seed"][0]))
    om = oracle.model(m)
    om.forward(int(g["prompt"][0]), 0)
    scale = logits_scale(m, om.hidden())
    om.close()
    model = ops.Model(m, attn_mode=1, gemv_mode=FAST)
    try:
        lg = model.forward(int(g["prompt"][0]), 0)
        assert_fast(lg, g["logits0"], TOL, "tiny-llama first logits", scale)
        model.reset()
        ids = model.generate_greedy(g["prompt"], len(g["ids"]))
        assert np.array_equal(ids, g["ids"]), np.nonzero(ids != g["ids"])[0][:5]
    finally:
        model.close()


def test_tiny_llama_fast_long_greedy(gpu, oracle):
    """256 greedy tokens (the tiny config's decode length) from a 16-token
    prompt: FAST ids equal the EXACT GPU ids and the oracle's."""
    cfg = W.TINY_LLAMA
    m = W.make_model(cfg, 11)
    prompt = W.tokens(16, cfg["vocab_size"], 11)
    ref = oracle.model(m).generate_greedy(prompt, 256)
    runs = {}
    for name, am, gm in [("exact", 0, 0), ("fast", 1, FAST)]:
        model = ops.Model(m, attn_mode=am, gemv_mode=gm)
        try:
            runs[name] = model.generate_greedy(prompt, 256)
        finally:
            model.close()
    assert np.array_equal(runs["exact"], ref), ("exact vs oracle", np.nonzero(runs["exact"] != ref)[0][:5])
    assert np.array_equal(runs["fast"], ref), ("fast vs oracle", np.nonzero(runs["fast"] != ref)[0][:5])


@pytest.mark.slow
def test_llama7b_fast_greedy_matches_exact(gpu):
    """Llama-2-7B-shaped Q4_0, fp16 KV: FAST decode gives the EXACT path's
    greedy ids (EXACT is bit-identical to the reference)."""
    cfg = dict(W.LLAMA2_7B)
    m = W.make_model(cfg, 5)
    prompt = W.tokens(8, cfg["vocab_size"], 5)
    exact = ops.Model(m)
    try:
        ref = exact.generate_greedy(prompt, 32)
    finally:
        exact.close()
    fast = ops.Model(m, attn_mode=1, gemv_mode=FAST)
    try:
        got = fast.generate_greedy(prompt, 32)
    finally:
        fast.close()
    assert np.array_equal(got, ref), np.nonzero(got != ref)[0][:5]
