"""Seeded inputs of the tensor-engine dispatch parity cases (the reference's
gpu_tensor_* entry points backed by the engine's CPU operators,
runtime/tensor/tensor_cpu.c), shared by tests/golden/make_golden.py, which
records the reference's outputs in tests/golden/engine.npz, and the tests."""
import numpy as np

from tensoros_b200 import workloads as W

SEED = 11
# M, N, K: edges of the 4x4 micro-tiles and the 64/128 blocks; N a multiple
# of 4 (the reference's packed-B loads are aligned 16-byte loads of B's rows)
MATMUL = [(4, 4, 4), (67, 132, 130), (128, 64, 257), (5, 300, 7)]
SOFTMAX = [(3, 1000), (2, 7), (1, 32000)]                              # rows, n
LAYERNORM = [(4, 256), (3, 130), (2, 4097)]
EPS = 1e-5
# seq, head_dim: seq a multiple of 4 (the reference softmaxes the rows of its
# seq x seq score matrix with aligned 16-byte stores)
ATTENTION = [(16, 64), (132, 32)]


def matmul_case(M, N, K):
    return (W.normal_f32(M * K, SEED, 400 + M).reshape(M, K), W.normal_f32(K * N, SEED, 401 + N).reshape(K, N))


def softmax_case(rows, n):
    x = (W.normal_f32(rows * n, SEED, 410 + n) * 4.0).reshape(rows, n)
    if rows >= 2 and n >= 7:
        x[1, 3] = x[1, 5] = x[1].max() + 1.0        # a tie at the maximum
    return x


def layernorm_case(rows, n):
    return W.normal_f32(rows * n, SEED, 420 + n, 0.5, 2.0).reshape(rows, n)


def attention_case(seq, hd):
    return tuple(W.normal_f32(seq * hd, SEED, 430 + 3 * seq + k).reshape(seq, hd) for k in range(3))
