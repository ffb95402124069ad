"""Generate the golden vectors under tests/golden/ from the REFERENCE itself.

The reference (TensorOS runtime/nn, C) is compiled hosted from its own
unmodified sources by oracle/Makefile into oracle/_ref/libtos_ref.so; this
script feeds it seeded inputs and records its outputs.  The committed files
pin both the C restatement (oracle/tos_oracle.c) and the GPU path:

  ops.npz            per-operator inputs and reference outputs
  tiny_llama.npz     tiny-llama (6L/288d, Q8_0, fp32 KV) greedy ids + logits
  llama7b_short.npz  Llama-2-7B-shaped Q4_0 model, fp32 KV, 4 prompt + 4 greedy
  sample.npz         llm_sample's tokens for seeded logits, temperatures and
                     timestamp words (the reference's own sampler, its
                     timestamp read scripted: oracle/ref_llm_hosted.c)
  tf.npz             the fp32 transformer engine (runtime/nn/transformer.c):
                     tf_rmsnorm, tf_swiglu_ffn, tf_cached_attention and
                     tf_forward_token logits of two seeded models
  engine.npz         the tensor engine's CPU operators (runtime/tensor/
                     tensor_cpu.c: matmul, softmax, layer norm, attention)

Run from the repository root after building:  python tests/golden/make_golden.py
(`python tests/golden/make_golden.py sample` writes sample.npz alone)
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))

import pyoracle  # noqa: E402
from tensoros_b200 import workloads as W  # noqa: E402

OUT = Path(__file__).resolve().parent
SEED = 7


def edge_blocks(type_: int, n: int, stream: int) -> np.ndarray:
    """n GGUF blocks with a few hand-set scales: 0, -0, smallest subnormal,
    a subnormal, largest finite, 1.0."""
    b = W.quant(type_, 1, 32 * n, SEED, stream).copy()
    bs = W.BLOCK_BYTES[type_]
    specials = [0x0000, 0x8000, 0x0001, 0x03FF, 0x7BFF, 0x3C00, 0xBC00]
    for i, h in enumerate(specials):
        b[bs * i] = h & 0xFF
        b[bs * i + 1] = h >> 8
    return b


def edge_x(n: int, stream: int) -> np.ndarray:
    x = W.normal_f32(n, SEED, stream)
    x[:8] = np.array([0.0, -0.0, 1e-40, -1e-40, 3e38, -3e38, 1.0, -1.0], dtype=np.float32)
    return x


def main():
    R = pyoracle.reference()
    g = {}
    # --- per-block values (llm.c:148-216)
    for t, name in [(W.TYPE_Q4_0, "q4_0"), (W.TYPE_Q8_0, "q8_0")]:
        n = 96
        blocks = edge_blocks(t, n, 11 + t)
        x = edge_x(32 * n, 12 + t)
        bs = W.BLOCK_BYTES[t]
        fn = R.q4_0_dot32 if t == W.TYPE_Q4_0 else R.q8_0_dot32
        g[f"blocks_{name}"] = blocks
        g[f"blocks_{name}_x"] = x
        g[f"blocks_{name}_out"] = np.array([fn(blocks[bs * i:bs * i + bs], x[32 * i:32 * i + 32]) for i in range(n)],
                                           dtype=np.float32)
    # --- GEMV (llm.c:221-349), odd shapes incl. the F16/F32 row formats
    for t, (r, c), tag in [(W.TYPE_Q4_0, (37, 256), "q4_0"), (W.TYPE_Q8_0, (40, 288), "q8_0"),
                           (W.TYPE_Q4_0, (24, 4096), "q4_0_wide"), (W.TYPE_Q8_0, (9, 11008), "q8_0_wide")]:
        w = W.quant(t, r, c, SEED, 20 + len(g))
        x = W.normal_f32(c, SEED, 21 + len(g))
        g[f"gemv_{tag}_w"], g[f"gemv_{tag}_x"] = w, x
        g[f"gemv_{tag}_shape"] = np.array([r, c, t], dtype=np.int32)
        g[f"gemv_{tag}_out"] = R.gemv(w, x, r, c, t)
    # F32 rows are read with aligned 16-byte vector loads (llm.c:266-267), so
    # in_dim stays a multiple of 4; 100 = 12*8 + a 4-element tail
    wf = W.normal_f32(11 * 100, SEED, 30)
    xf = W.normal_f32(100, SEED, 31)
    g["gemv_f32_w"], g["gemv_f32_x"], g["gemv_f32_out"] = wf, xf, R.gemv(wf, xf, 11, 100, W.TYPE_F32)
    wh = W.normal_f16(13 * 102, SEED, 32, 0.0, 0.1)
    xh = W.normal_f32(102, SEED, 33)
    g["gemv_f16_w"], g["gemv_f16_x"], g["gemv_f16_out"] = wh, xh, R.gemv(wh, xh, 13, 102, W.TYPE_F16)
    # --- RMSNorm (llm.c:416-452): eps fixed at 1e-6 by the reference
    for dim in (288, 290, 4096):
        x = W.normal_f32(dim, SEED, 40 + dim)
        w = W.normal_f32(dim, SEED, 41 + dim, 1.0, 0.1)
        g[f"rmsnorm_{dim}_x"], g[f"rmsnorm_{dim}_w"] = x, w
        g[f"rmsnorm_{dim}_out"] = R.rmsnorm(x, w, dim)
    # --- RoPE (llm.c:460-500)
    positions = np.array([0, 1, 5, 100, 271, 1023, 2047, 4095, 4096, 8191], dtype=np.int32)
    for hd in (48, 128):
        v = W.normal_f32(hd, SEED, 50 + hd)
        g[f"rope_{hd}_v"] = v
        g[f"rope_{hd}_pos"] = positions
        g[f"rope_{hd}_out"] = np.stack([R.rope(v, int(p), hd, 10000.0) for p in positions])
    # --- softmax / silu (llm.c:506-544)
    for n in (1, 7, 1000):
        s = W.normal_f32(n, SEED, 60 + n, 0.0, 8.0)
        g[f"softmax_{n}_x"], g[f"softmax_{n}_out"] = s, R.softmax(s)
    s = np.concatenate([np.linspace(-100, 100, 401, dtype=np.float32), W.normal_f32(599, SEED, 70, 0, 3)])
    g["silu_x"], g["silu_out"] = s, R.silu(s)
    # --- dot / axpy / vadd / vmul (llm.c:551-632)
    for n in (48, 128, 131):
        a, b = W.normal_f32(n, SEED, 80 + n), W.normal_f32(n, SEED, 81 + n)
        g[f"dot_{n}_a"], g[f"dot_{n}_b"] = a, b
        g[f"dot_{n}_out"] = np.array([R.dot_f32(a, b)], dtype=np.float32)
    a, b = W.normal_f32(1001, SEED, 90), W.normal_f32(1001, SEED, 91)
    g["vec_a"], g["vec_b"] = a, b
    g["axpy_out"] = R.axpy_f32(a, np.float32(0.3710938), b)
    g["vadd_out"] = R.vadd_f32(a, b)
    g["vmul_out"] = R.vmul_f32(a, b)
    # --- argmax (llm.c:1129-1140): ties, NaN first / later, signed zeros
    cases = [
        np.array([1, 3, 3, 2], np.float32), np.array([np.nan, 5, 7], np.float32),
        np.array([1, np.nan, 7, 7], np.float32), np.array([-0.0, 0.0, -1.0], np.float32),
        np.array([-np.inf, -np.inf], np.float32), W.normal_f32(32000, SEED, 95),
    ]
    for i, c in enumerate(cases):
        g[f"argmax_{i}_x"] = c
        g[f"argmax_{i}_out"] = np.array([R.argmax(c)], dtype=np.int32)
    # --- embedding rows (llm.c:365-410)
    for t, dim, tag in [(W.TYPE_Q4_0, 4096, "q4_0"), (W.TYPE_Q8_0, 288, "q8_0")]:
        e = W.quant(t, 5, dim, SEED, 100 + t)
        g[f"embed_{tag}_w"] = e
        g[f"embed_{tag}_out"] = np.stack([R.embed(e, t, dim, tok) for tok in range(5)])
    ef = W.normal_f32(5 * 64, SEED, 110)
    g["embed_f32_w"], g["embed_f32_out"] = ef, np.stack([R.embed(ef, W.TYPE_F32, 64, t) for t in range(5)])
    eh = W.normal_f16(5 * 64, SEED, 111)
    g["embed_f16_w"], g["embed_f16_out"] = eh, np.stack([R.embed(eh, W.TYPE_F16, 64, t) for t in range(5)])
    # --- fp32-scale Q4 (quantize4.c:122-198)
    qb = W.q4f(8, 64, SEED, 120)
    qx = W.normal_f32(64, SEED, 121)
    g["q4f_w"], g["q4f_x"] = qb, qx
    g["q4f_gemv_out"] = R.q4_gemv(qb, qx, 8, 64)
    g["q4f_block_out"] = np.array([R.q4_dot_block(qb[20 * i:20 * i + 20], qx[:32]) for i in range(4)], np.float32)
    np.savez_compressed(OUT / "ops.npz", **g)
    print("ops.npz:", len(g), "arrays")

    # --- tiny-llama greedy decode (BASELINE tiny config; eps 1e-6 = reference)
    cfg = W.TINY_LLAMA
    m = W.make_model(cfg, W.SEED)
    prompt = W.prompt_tokens(cfg, W.SEED)
    rm = R.model(m)
    logits0 = rm.forward(int(prompt[0]), 0)
    rm.close()
    ids = R.model(m).generate_greedy(prompt, cfg["n_gen"])
    np.savez_compressed(OUT / "tiny_llama.npz", seed=np.array([W.SEED]), prompt=prompt, ids=ids,
                        logits0=logits0)
    print("tiny_llama.npz:", len(ids), "ids")

    # --- Llama-2-7B shape, fp32 KV (the reference's cache type), short run
    cfg7 = dict(W.LLAMA2_7B, kv_type=W.TYPE_F32, max_seq=16)
    m7 = W.make_model(cfg7, W.SEED)
    p7 = W.tokens(4, cfg7["vocab_size"], W.SEED)
    r7 = R.model(m7)
    l7 = r7.forward(int(p7[0]), 0)
    r7.close()
    ids7 = R.model(m7).generate_greedy(p7, 4)
    np.savez_compressed(OUT / "llama7b_short.npz", seed=np.array([W.SEED]), prompt=p7, ids=ids7,
                        logits0=l7)
    print("llama7b_short.npz:", ids7)


SAMPLE_TEMPS = [0.0005, 0.2, 0.7, 1.0, 1.9]
SAMPLE_WORDS = 24


def sample_cases():
    """Logit vectors for llm_sample (llm.c:1143-1246): plain, ties across the
    top-40 cut, ties exactly at the 40th value, signed zeros, fewer than 40
    candidates, many duplicates."""
    c0 = W.normal_f32(32000, SEED, 200, 0.0, 3.0)
    c1 = W.normal_f32(32000, SEED, 201).copy()
    c1[(np.arange(60) * 523 + 7) % 32000] = 4.0
    c2 = W.normal_f32(5000, SEED, 202).copy()
    c2[(np.arange(7) * 701 + 3) % 5000] = np.sort(c2)[-40]
    c3 = np.zeros(1000, np.float32)
    c3[::3] = -0.0
    c3[500] = 1.0
    c4 = W.normal_f32(17, SEED, 203, 0.0, 2.0)
    c5 = (np.round(W.normal_f32(32000, SEED, 204) * 4) / 4).astype(np.float32)
    return [c0, c1, c2, c3, c4, c5]


def sample_golden(R):
    cases = sample_cases()
    # timestamp words: a fixed LCG sequence (the reference mixes them itself)
    words = np.empty((len(cases), len(SAMPLE_TEMPS), SAMPLE_WORDS), np.uint32)
    v = 0x2545F491
    for idx in np.ndindex(words.shape):
        v = (v * 1664525 + 1013904223) & 0xFFFFFFFF
        words[idx] = v
    toks = np.empty(words.shape, np.int32)
    for ci, x in enumerate(cases):
        for ti, t in enumerate(SAMPLE_TEMPS):
            for k in range(SAMPLE_WORDS):
                toks[ci, ti, k] = R.sample_at(x, t, int(words[ci, ti, k]))
    if np.any(toks < 0):
        raise SystemExit("the timestamp read could not be scripted on this host")
    g = {f"x{i}": x for i, x in enumerate(cases)}
    np.savez_compressed(OUT / "sample.npz", temps=np.array(SAMPLE_TEMPS, np.float32), words=words, tokens=toks, **g)
    print("sample.npz:", toks.size, "draws")


def tf_golden(R):
    """The reference engine's outputs for the seeded cases of tests/tf_cases.py
    (inputs regenerated by the tests, not stored)."""
    sys.path.insert(0, str(ROOT / "tests"))
    import tf_cases as T
    g = {}
    for dim in T.RMS_DIMS:
        g[f"rms_{dim}_out"] = R.tf_rmsnorm(*T.rms_case(dim))
    for dim, ff in T.FFN_SHAPES:
        g[f"ffn_{dim}_out"] = R.tf_swiglu_ffn(*T.ffn_case(dim, ff), dim, ff)
    for tag in T.MODELS:
        tf, toks = T.model_case(tag)
        m = R.tf_model(tf)
        g[f"model_{tag}_logits"] = np.stack([m.forward(int(t), p) for p, t in enumerate(toks)])
    tf, _ = T.model_case("small")
    m = R.tf_model(tf)
    qkv = T.attn_qkv()
    g["attn_out"] = np.stack([m.cached_attention(qkv[p, 0], qkv[p, 1], qkv[p, 2], T.ATTN["layer"], T.ATTN["head"], p)
                              for p in range(T.ATTN["steps"])])
    np.savez_compressed(OUT / "tf.npz", **g)
    print("tf.npz:", len(g), "arrays")


def engine_golden(R):
    """The tensor engine's CPU operators (runtime/tensor/tensor_cpu.c) on the
    seeded cases of tests/engine_cases.py."""
    sys.path.insert(0, str(ROOT / "tests"))
    import engine_cases as E
    g = {}
    for M, N, K in E.MATMUL:
        g[f"matmul_{M}_{N}_{K}"] = R.engine_matmul(*E.matmul_case(M, N, K))
    for rows, n in E.SOFTMAX:
        g[f"softmax_{rows}_{n}"] = R.engine_softmax_rows(E.softmax_case(rows, n))
    for rows, n in E.LAYERNORM:
        g[f"layernorm_{rows}_{n}"] = R.engine_layernorm_rows(E.layernorm_case(rows, n), E.EPS)
    for seq, hd in E.ATTENTION:
        g[f"attention_{seq}_{hd}"] = R.engine_attention(*E.attention_case(seq, hd))
    np.savez_compressed(OUT / "engine.npz", **g)
    print("engine.npz:", len(g), "arrays")


if __name__ == "__main__":
    if sys.argv[1:] == ["engine"]:
        engine_golden(pyoracle.reference())
    elif sys.argv[1:] == ["sample"]:
        sample_golden(pyoracle.reference())
    elif sys.argv[1:] == ["tf"]:
        tf_golden(pyoracle.reference())
    else:
        main()
        sample_golden(pyoracle.reference())
        tf_golden(pyoracle.reference())
        engine_golden(pyoracle.reference())
