"""Seeded inputs of the fp32 transformer-engine parity cases
(runtime/nn/transformer.c), shared by tests/golden/make_golden.py, which
records the reference's outputs for them in tests/golden/tf.npz, and by the
tests, which regenerate the same inputs."""
import numpy as np

from tensoros_b200 import workloads as W

SEED = 7
RMS_DIMS = (64, 132, 512)            # the engine's vector loads need dim % 4 == 0
FFN_SHAPES = ((64, 128), (256, 688))
MODELS = {"small": (W.TF_SMALL, 3, 12), "medium": (W.TF_MEDIUM, 5, 6)}   # cfg, seed, steps
ATTN = dict(layer=1, head=2, steps=10)


def rms_case(dim):
    return W.normal_f32(dim, SEED, 300 + dim), W.normal_f32(dim, SEED, 301 + dim, 1.0, 0.1)


def ffn_case(dim, ff):
    return (W.normal_f32(dim, SEED, 310 + dim), W.normal_f32(ff * dim, SEED, 311 + dim, 0.0, dim ** -0.5),
            W.normal_f32(dim * ff, SEED, 312 + dim, 0.0, ff ** -0.5),
            W.normal_f32(ff * dim, SEED, 313 + dim, 0.0, dim ** -0.5))


def model_case(tag):
    cfg, seed, steps = MODELS[tag]
    return W.make_tf_model(cfg, seed), W.tokens(steps, cfg["vocab_size"], seed)


def attn_qkv():
    hd = W.TF_SMALL["dim"] // W.TF_SMALL["num_heads"]
    return W.normal_f32(ATTN["steps"] * 3 * hd, SEED, 330).reshape(ATTN["steps"], 3, hd)
