"""Whole-model decode (llm_forward_token + greedy generate) on the GPU:
greedy token ids and logits identical to the reference (golden) and to the
oracle restatement."""
import numpy as np
import pytest

from conftest import GOLDEN, bits_equal, first_diff
from tensoros_b200 import ops
from tensoros_b200 import workloads as W

pytestmark = pytest.mark.gpu


def test_tiny_llama_greedy_matches_reference(gpu):
    g = np.load(GOLDEN / "tiny_llama.npz")
    m = W.make_model(W.TINY_LLAMA, int(g["seed"][0]))
    model = ops.Model(m)
    try:
        lg = model.forward(int(g["prompt"][0]), 0)
        assert bits_equal(lg, g["logits0"]), first_diff(lg, g["logits0"])
        model.reset()
        ids = model.generate_greedy(g["prompt"], len(g["ids"]))
        assert np.array_equal(ids, g["ids"]), np.nonzero(ids != g["ids"])[0][:5]
    finally:
        model.close()


def test_tiny_llama_fp16_kv_and_fast_attention(gpu, oracle):
    """fp16 KV cache (no reference counterpart): equal to the restatement that
    rounds K/V to fp16 at the cache store.  FAST attention keeps the greedy
    ids of EXACT on this config."""
    cfg = W.TINY_LLAMA
    m = W.make_model(cfg, 3)
    prompt = W.tokens(16, cfg["vocab_size"], 3)
    ref = oracle.model(m, kv_type=W.TYPE_F16).generate_greedy(prompt, 64)
    model = ops.Model(m, kv_type=W.TYPE_F16)
    try:
        assert np.array_equal(model.generate_greedy(prompt, 64), ref)
    finally:
        model.close()
    fast = ops.Model(m, attn_mode=1, kv_type=W.TYPE_F16)
    try:
        got = fast.generate_greedy(prompt, 64)
        agree = int(np.sum(got == ref))
        assert agree == 64, agree
    finally:
        fast.close()


def test_logits_every_step_tiny(gpu, oracle):
    """Every decode step's logits are bit-identical to the restatement."""
    cfg = W.TINY_LLAMA
    m = W.make_model(cfg, 21)
    toks = W.tokens(40, cfg["vocab_size"], 21)
    om = oracle.model(m)
    model = ops.Model(m)
    try:
        for pos, t in enumerate(toks):
            a, b = model.forward(int(t), pos), om.forward(int(t), pos)
            assert bits_equal(a, b), (pos, first_diff(a, b))
    finally:
        model.close()
        om.close()


@pytest.mark.slow
def test_llama7b_short_matches_reference(gpu, oracle):
    """Llama-2-7B-shaped Q4_0 model with the reference's fp32 cache: logits of
    every step bit-exact vs the restatement, first logits and greedy ids vs
    the reference's golden run."""
    g = np.load(GOLDEN / "llama7b_short.npz")
    cfg = dict(W.LLAMA2_7B, kv_type=W.TYPE_F32, max_seq=16)
    m = W.make_model(cfg, int(g["seed"][0]))
    model = ops.Model(m)
    try:
        lg = model.forward(int(g["prompt"][0]), 0)
        assert bits_equal(lg, g["logits0"]), first_diff(lg, g["logits0"])
        model.reset()
        ids = model.generate_greedy(g["prompt"], len(g["ids"]))
        assert np.array_equal(ids, g["ids"])
    finally:
        model.close()


@pytest.mark.slow
def test_llama7b_fp16_kv_steps(gpu, oracle):
    """The benchmark configuration (fp16 KV, capacity 4096): a few steps'
    logits bit-exact vs the restatement."""
    cfg = dict(W.LLAMA2_7B)
    m = W.make_model(cfg, 5)
    toks = W.tokens(3, cfg["vocab_size"], 5)
    om = oracle.model(m, kv_type=W.TYPE_F16)
    model = ops.Model(m)
    try:
        for pos, t in enumerate(toks):
            a, b = model.forward(int(t), pos), om.forward(int(t), pos)
            assert bits_equal(a, b), (pos, first_diff(a, b))
    finally:
        model.close()
        om.close()
