"""The seeded workload generator (libtos_synth): deterministic, independent
of thread count, with the distributions the benchmark configurations name."""
import numpy as np

from tensoros_b200 import _ffi
from tensoros_b200 import workloads as W


def _gen_q4(nb, threads):
    a = np.empty(nb * 18, np.uint8)
    _ffi.synth().tos_synth_q4_0(a.ctypes.data, nb, 5, 9, 0.02, threads)
    return a


def test_thread_count_independent():
    a, b = _gen_q4(10000, 1), _gen_q4(10000, 7)
    assert np.array_equal(a, b)
    x1 = np.empty(5000, np.float32)
    x2 = np.empty(5000, np.float32)
    _ffi.synth().tos_synth_normal_f32(x1.ctypes.data, 5000, 3, 4, 0.0, 1.0, 1)
    _ffi.synth().tos_synth_normal_f32(x2.ctypes.data, 5000, 3, 4, 0.0, 1.0, 5)
    assert np.array_equal(x1, x2)


def test_streams_differ_and_repeat():
    assert not np.array_equal(W.q4_0(8, 64, 1, 1), W.q4_0(8, 64, 1, 2))
    assert np.array_equal(W.q8_0(8, 64, 1, 3), W.q8_0(8, 64, 1, 3))


def test_q4_0_distribution():
    blocks = W.q4_0(256, 4096, 11, 1).reshape(-1, 18)
    scales = blocks[:, :2].copy().view(np.float16).astype(np.float32).ravel()
    assert np.all(scales >= 0)
    assert abs(np.sqrt(np.mean(scales.astype(np.float64) ** 2)) - 0.02) < 0.001
    nib = np.concatenate([blocks[:, 2:] & 0xF, blocks[:, 2:] >> 4]).ravel()
    counts = np.bincount(nib, minlength=16)
    assert counts.min() > 0.95 * counts.mean() and counts.max() < 1.05 * counts.mean()


def test_q8_0_distribution():
    blocks = W.q8_0(256, 4096, 11, 2).reshape(-1, 34)
    q = blocks[:, 2:].copy().view(np.int8).ravel()
    assert q.min() == -127 and q.max() == 127
    assert abs(q.mean()) < 0.5
    scales = blocks[:, :2].copy().view(np.float16).astype(np.float32).ravel()
    assert abs(np.sqrt(np.mean(scales.astype(np.float64) ** 2)) - 0.01) < 0.0005


def test_normal_and_f16():
    x = W.normal_f32(200000, 1, 1)
    assert abs(x.mean()) < 0.01 and abs(x.std() - 1) < 0.01
    h = W.normal_f16(200000, 1, 1)
    assert np.array_equal(h, x.astype(np.float16).view(np.uint16))


def test_f32_to_f16_matches_numpy():
    xs = np.concatenate([W.normal_f32(5000, 2, 2, 0, 2e4), W.normal_f32(5000, 2, 3, 0, 1e-6),
                         np.array([65504, 65520, 65519.9, 6e-8, 3e-8, 2.9802322e-8, -0.0, np.inf], np.float32)])
    got = np.array([W.f32_to_f16_bits(v) for v in xs], np.uint16)
    assert np.array_equal(got, xs.astype(np.float16).view(np.uint16))


def test_tokens_in_range():
    t = W.tokens(1000, 32000, 4)
    assert t.min() >= 0 and t.max() < 32000 and len(set(t.tolist())) > 900
