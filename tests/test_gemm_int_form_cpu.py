"""The arithmetic of the integer GEMM form (gemm_tc.cu, gemm_i8_kernel and
gemm_prep_i8_kernel: Q4_0 at up to 16 activation rows), restated in numpy
and checked on the CPU.

Per 32-element block the prep writes X = rint(x / s) (s a power of two,
|X| <= 2^22, as the FAST GEMV's make_xfix) as three signed byte limbs
X = L0 + 2^8 L1 + 2^16 L2, and the weights enter as the signed bytes n - 8
in the order q4_to_s8 produces.  The tensor core's exact integer sums per
limb then give Y = sum_k (n_k - 8) X_k, the block value of q4_0_dot32
(runtime/nn/llm.c:148-185) before its float roundings.  These checks cover
the limb split (range and reconstruction at the extremes), the byte trick
for n - 8, the K order shared by the weights and the limbs, and that the
limb sums fit the int32 accumulators."""
import numpy as np

from tensoros_b200 import workloads as W


def limbs(X):
    """gemm_prep_i8_kernel's balanced split: low byte as a signed byte, then
    the same on the rest."""
    X = np.asarray(X, np.int64)
    l0 = ((X & 0xFF) ^ 0x80) - 0x80
    r1 = (X - l0) >> 8
    l1 = ((r1 & 0xFF) ^ 0x80) - 0x80
    l2 = (r1 - l1) >> 8
    return l0, l1, l2


def q4_to_s8(w):
    """q4_to_s8: a quant word's low and high nibbles as bytes n - 8
    (n + 120 stays inside its byte; flipping bit 7 gives n - 8)."""
    w = np.uint32(w)
    lo = ((w & np.uint32(0x0F0F0F0F)) + np.uint32(0x78787878)) ^ np.uint32(0x80808080)
    hi = (((w >> np.uint32(4)) & np.uint32(0x0F0F0F0F)) + np.uint32(0x78787878)) ^ np.uint32(0x80808080)
    as_s8 = lambda v: np.frombuffer(np.uint32(v).tobytes(), np.int8).astype(np.int64)
    return as_s8(lo), as_s8(hi)


def test_limbs_reconstruct_and_fit_signed_bytes():
    rng = np.random.default_rng(W.SEED)
    X = np.concatenate([rng.integers(-(1 << 22), (1 << 22) + 1, 200000),
                        np.array([0, 1, -1, 127, 128, -128, -129, 255, 256, -256, 32767, 32768, -32768,
                                  (1 << 22), -(1 << 22), (1 << 22) - 1, -(1 << 22) + 1])])
    l0, l1, l2 = limbs(X)
    assert np.array_equal(l0 + 256 * l1 + 65536 * l2, X)
    for l in (l0, l1):
        assert l.min() >= -128 and l.max() <= 127
    assert np.abs(l2).max() <= 65


def test_q4_bytes_are_n_minus_8_in_the_shared_k_order():
    # quant byte b of a word holds elements 2b (low nibble) and 2b + 1
    # (llm.c:162-165); q4_to_s8's low word carries elements 0, 2, 4, 6 and
    # its high word 1, 3, 5, 7, which is the order the prep gives the limbs
    rng = np.random.default_rng(W.SEED + 1)
    for _ in range(2000):
        n = rng.integers(0, 16, 8)
        w = 0
        for b in range(4):
            w |= int(n[2 * b] | (n[2 * b + 1] << 4)) << (8 * b)
        lo, hi = q4_to_s8(w)
        assert np.array_equal(lo, n[0::2] - 8)
        assert np.array_equal(hi, n[1::2] - 8)


def test_block_value_from_limb_sums_is_exact():
    # one MMA of K = 32 per block: S_l = sum_k (n_k - 8) L_l,k for the three
    # limbs; Y = S0 + 2^8 S1 + 2^16 S2 in wrapping int32 equals the exact sum
    rng = np.random.default_rng(W.SEED + 2)
    for case in range(3000):
        n = rng.integers(0, 16, 32)
        X = rng.integers(-(1 << 22), (1 << 22) + 1, 32)
        if case % 5 == 0:
            n = np.full(32, 0 if case % 2 else 15)
            X = np.full(32, (1 << 22) if case % 3 else -(1 << 22))
        l0, l1, l2 = limbs(X)
        a = n - 8
        S = [int(np.dot(a, l)) for l in (l0, l1, l2)]
        assert max(abs(s) for s in S) <= 32 * 8 * 128       # the s32 accumulator columns
        Y = (S[0] + (S[1] << 8) + (S[2] << 16)) & 0xFFFFFFFF
        Y = Y - (1 << 32) if Y >> 31 else Y
        assert Y == int(np.dot(a, X))
