"""The fp32 transformer engine (runtime/nn/transformer.c:92-366) on the GPU:
tos_tf_rmsnorm, tos_tf_swiglu_ffn, tos_tf_cached_attention and
tos_tf_forward_token give the reference engine's results bit for bit
(tests/golden/tf.npz: the reference's own outputs for the seeded cases of
tests/tf_cases.py): its fp32 weights, KV cache [layer][head][seq][head_dim],
eps 1e-5, and tensor_cpu.c's exponential, SiLU and softmax."""
import ctypes as C

import numpy as np
import pytest

import tf_cases as T
from conftest import GOLDEN, bits_equal, first_diff
from tensoros_b200 import _ffi

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN / "tf.npz")


def _p(a):
    return a.ctypes.data


def test_tf_rmsnorm(gpu, g):
    lib = _ffi.nn()
    for dim in T.RMS_DIMS:
        x, w = T.rms_case(dim)
        out = np.empty(dim, np.float32)
        lib.tos_tf_rmsnorm(_p(out), _p(x), _p(w), dim)
        assert lib.tos_last_status() == 0
        assert bits_equal(out, g[f"rms_{dim}_out"]), (dim, first_diff(out, g[f"rms_{dim}_out"]))


def test_tf_swiglu_ffn(gpu, g):
    lib = _ffi.nn()
    for dim, ff in T.FFN_SHAPES:
        x, w1, w2, w3 = T.ffn_case(dim, ff)
        out = np.empty(dim, np.float32)
        lib.tos_tf_swiglu_ffn(_p(out), _p(x), _p(w1), _p(w2), _p(w3), dim, ff)
        assert lib.tos_last_status() == 0
        assert bits_equal(out, g[f"ffn_{dim}_out"]), (dim, first_diff(out, g[f"ffn_{dim}_out"]))


class TfModel:
    def __init__(self, tf):
        self.lib, self.tf = _ffi.nn(), tf
        self.desc = tf.fill_desc(_ffi.TfDesc())
        self.h = C.c_void_p()
        assert self.lib.tos_tf_model_create(C.byref(self.h), C.byref(self.desc)) == 0

    def forward(self, tok, pos):
        d, v = self.tf.cfg["dim"], self.tf.cfg["vocab_size"]
        row = np.ascontiguousarray(self.tf.tok_embed[tok * d:(tok + 1) * d])
        out = np.empty(v, np.float32)
        assert self.lib.tos_tf_forward_token(self.h, _p(out), _p(row), pos) == 0
        return out

    def close(self):
        self.lib.tos_tf_model_destroy(self.h)


@pytest.mark.parametrize("tag", list(T.MODELS))
def test_tf_forward_token(gpu, g, tag):
    tf, toks = T.model_case(tag)
    m = TfModel(tf)
    try:
        for pos, t in enumerate(toks):
            lg = m.forward(int(t), pos)
            ref = g[f"model_{tag}_logits"][pos]
            assert bits_equal(lg, ref), (tag, pos, first_diff(lg, ref))
        # kv_cache_reset: the same sequence again from position 0
        assert m.lib.tos_tf_reset(m.h) == 0
        lg = m.forward(int(toks[0]), 0)
        assert bits_equal(lg, g[f"model_{tag}_logits"][0])
    finally:
        m.close()


def test_tf_cached_attention(gpu, g):
    tf, _ = T.model_case("small")
    m = TfModel(tf)
    try:
        qkv = T.attn_qkv()
        for p in range(T.ATTN["steps"]):
            out = np.empty(qkv.shape[2], np.float32)
            st = m.lib.tos_tf_cached_attention(m.h, _p(out), _p(np.ascontiguousarray(qkv[p, 0])),
                                               _p(np.ascontiguousarray(qkv[p, 1])), _p(np.ascontiguousarray(qkv[p, 2])),
                                               T.ATTN["layer"], T.ATTN["head"], p)
            assert st == 0
            assert bits_equal(out, g["attn_out"][p]), (p, first_diff(out, g["attn_out"][p]))
    finally:
        m.close()


def test_tf_rejects(gpu):
    lib = _ffi.nn()
    tf, _ = T.model_case("small")
    m = TfModel(tf)
    try:
        out = np.empty(16, np.float32)
        q = np.zeros(16, np.float32)
        assert lib.tos_tf_cached_attention(m.h, _p(out), _p(q), _p(q), _p(q), 9, 0, 0) == -1   # no layer 9
        assert lib.tos_tf_forward_token(m.h, None, _p(q), tf.cfg["max_seq"]) == -1
    finally:
        m.close()
