"""Batched prompt pass (tos_model_prefill, tensor-core GEMMs) against the
token-by-token path that equals the reference (llm.c:1279-1281 runs the
prompt one llm_forward_token at a time): last-token logits within the 1e-4
normwise bound, the same greedy next token, and the same greedy ids when
decoding continues from the cache the prefill filled."""
import numpy as np
import pytest

from conftest import assert_fast
from tensoros_b200 import ops
from tensoros_b200 import workloads as W

pytestmark = pytest.mark.gpu
TOL = 1e-4


def normwise(got, ref):
    s = float(np.max(np.abs(ref)))
    return float(np.max(np.abs(got.astype(np.float64) - ref))) / (s if s > 0 else 1.0)


def stepwise(model, prompt):
    lg = None
    for i, t in enumerate(prompt):
        lg = model.forward(int(t), i)
    return int(np.argmax(lg)), lg


def check(cfg, layers, n_prompt, n_decode, seed=31, split=None, mode=0):
    synth = W.make_model(cfg, seed, n_layers=layers)
    prompt = W.tokens(n_prompt, cfg["vocab_size"], seed)
    ref_model = ops.Model(synth)
    try:
        nxt_ref, lg_ref = stepwise(ref_model, prompt)
        ids_ref = ref_model.decode(nxt_ref, n_prompt, n_decode)
    finally:
        ref_model.close()
    model = ops.Model(synth, attn_mode=mode, gemv_mode=mode)
    try:
        if split is None:
            nxt, lg = model.prefill(prompt, 0, logits=True)
        else:   # first part token by token, the rest batched from pos0 = split
            for i, t in enumerate(prompt[:split]):
                model.forward(int(t), i)
            nxt, lg = model.prefill(prompt[split:], split, logits=True)
        ids = model.decode(nxt, n_prompt, n_decode)
    finally:
        model.close()
    assert_fast(lg, lg_ref, TOL, "prefill last-token logits")
    assert nxt == nxt_ref
    assert np.array_equal(ids, ids_ref), np.nonzero(ids != ids_ref)[0][:5]


def test_prefill_small_gqa():
    check(W.SHARD_SMALL, None, 16, 24)


def test_prefill_7b_layers_128():
    check(W.LLAMA2_7B, 2, 128, 16)


def test_prefill_7b_layers_chunks_and_offset():
    check(W.LLAMA2_7B, 2, 200, 8)              # two 128-token chunks
    check(W.LLAMA2_7B, 2, 64, 8, split=40)     # continues a cache filled token by token


def test_prefill_fast_model():
    check(W.LLAMA2_7B, 2, 96, 8, mode=1)


def test_prefill_rejects_unsupported():
    synth = W.make_model(W.TINY_LLAMA, 3, n_layers=1)   # dim 288: not a multiple of 64
    model = ops.Model(synth)
    try:
        with pytest.raises(ops.TosError):
            model.prefill(W.tokens(4, W.TINY_LLAMA["vocab_size"], 3))
    finally:
        model.close()


@pytest.mark.slow
def test_prefill_7b_full_greedy():
    """the benchmark configuration: 128-token prefill, then greedy decode"""
    check(W.LLAMA2_7B, None, 128, 32)
