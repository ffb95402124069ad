"""Batched decode (tos_model_decode_batch): n <= 16 independent sequences,
one token each per step, each at its own position with its own KV cache;
projections as tensor-core GEMMs over the n tokens.  No counterpart in the
reference (one sequence, llm.c:641-743): every sequence must give the
reference's result for that sequence alone: logits within the FAST bound
(1e-4 normwise, and per element against the LM head's term magnitudes) of
the oracle's, greedy ids identical."""
import numpy as np
import pytest

from conftest import assert_fast, logits_scale
from tensoros_b200 import ops
from tensoros_b200 import workloads as W

pytestmark = pytest.mark.gpu
TOL = 1e-4


def normwise(got, ref):
    s = float(np.max(np.abs(ref)))
    return float(np.max(np.abs(got.astype(np.float64) - ref))) / (s if s > 0 else 1.0)


def run_batch(model, prompts, n_gen):
    """Sequence i (cache slot i) joins at step i, so positions differ within
    a batch and the rows of a batch change as sequences finish; each advances
    one token per step: its prompt, then its own greedy tokens.
    Returns per-sequence (generated ids, logits of every step)."""
    B = len(prompts)
    pos = [0] * B
    nxt = [None] * B
    gen = [[] for _ in range(B)]
    logs = [[] for _ in range(B)]
    step = 0
    while any(len(gen[i]) < n_gen for i in range(B)):
        alive = [i for i in range(B) if step >= i and len(gen[i]) < n_gen]
        toks = [int(prompts[i][pos[i]]) if pos[i] < len(prompts[i]) else int(nxt[i]) for i in alive]
        ids, lg = model.decode_batch(toks, [pos[i] for i in alive], slots=alive, logits=True)
        for k, i in enumerate(alive):
            logs[i].append(lg[k])
            if pos[i] >= len(prompts[i]):
                gen[i].append(toks[k])
            if pos[i] >= len(prompts[i]) - 1:
                nxt[i] = int(ids[k])
            pos[i] += 1
        step += 1
    return gen, logs


def test_batch_gqa_vs_oracle(gpu, oracle):
    cfg = W.SHARD_SMALL
    synth = W.make_model(cfg, 21)
    prompts = [W.tokens(3 + i, cfg["vocab_size"], 30 + i) for i in range(5)]
    n_gen = 6
    model = ops.Model(synth)
    try:
        gen, logs = run_batch(model, prompts, n_gen)
    finally:
        model.close()
    for i, p in enumerate(prompts):
        # the oracle consumes the same tokens: the prompt, then the ids the
        # batch produced; logits of every step within the bound
        ref = oracle.model(synth)
        consumed = list(p) + list(gen[i][:-1])
        try:
            want_next = []
            for t, tok in enumerate(consumed):
                lr = ref.forward(int(tok), t)
                assert_fast(logs[i][t], lr, TOL, ("batch", i, t), logits_scale(synth, ref.hidden()))
                if t >= len(p) - 1:
                    want_next.append((int(np.argmax(lr)), lr))
        finally:
            ref.close()
        # greedy ids: identical wherever the reference's choice is not a
        # near-tie within the FAST bound (the margin is reported otherwise)
        for k, (w, lr) in enumerate(want_next):
            top2 = np.sort(lr)[-2:]
            margin = float(top2[1] - top2[0]) / float(np.max(np.abs(lr)))
            assert gen[i][k] == w or margin <= 2 * TOL, (i, k, gen[i][k], w, margin)


def test_batch_7b_layers_sixteen(gpu):
    """16 sequences of the Llama-2-7B shape (2 layers, fp16 KV): sequences
    0, 7 and 15 against the single-sequence FAST path, step by step"""
    synth = W.make_model(W.LLAMA2_7B, 23, n_layers=2)
    prompts = [W.tokens(3, W.LLAMA2_7B["vocab_size"], 40 + i) for i in range(16)]
    model = ops.Model(synth)
    single = ops.Model(synth, attn_mode=1, gemv_mode=1)
    try:
        batch = [model.decode_batch([int(p[t]) for p in prompts], [t] * 16, logits=True) for t in range(3)]
        for i in (0, 7, 15):
            single.reset()
            for t in range(3):
                ls = single.forward(int(prompts[i][t]), t)
                ids, lg = batch[t]
                assert_fast(lg[i], ls, TOL, ("batch vs single", i, t))
            assert int(ids[i]) == int(np.argmax(ls))
    finally:
        model.close()
        single.close()


def test_batch_rejects(gpu):
    synth = W.make_model(W.SHARD_SMALL, 3)
    model = ops.Model(synth)
    try:
        with pytest.raises(ops.TosError):
            model.decode_batch([1] * 17, list(range(17)))
        with pytest.raises(ops.TosError):
            model.decode_batch([1, 2], [0, W.SHARD_SMALL["max_seq"]])
        with pytest.raises(ops.TosError):
            model.decode_batch([1, 2], [0, 0], slots=[3, 3])      # one slot twice
        with pytest.raises(ops.TosError):
            model.decode_batch([1], [0], slots=[16])
    finally:
        model.close()
    tiny = ops.Model(W.make_model(W.TINY_LLAMA, 3, n_layers=1))   # dim 288: not a multiple of 64
    try:
        with pytest.raises(ops.TosError):
            tiny.decode_batch([1], [0])
    finally:
        tiny.close()
