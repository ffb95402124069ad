"""Device sampling (tos_sample / tos_sample_dev) with a 32-bit entropy word
in place of the reference's timestamp: the reference's own llm_sample token
(llm.c:1143-1246, tests/golden/sample.npz, drawn with its timestamp read
scripted to the same word) for every committed case, and the oracle's
restatement on further random words: equal logits at the top-40 boundary,
+0.0 / -0.0, vocabularies shorter than 40 and the greedy limit."""
import numpy as np
import pytest

from conftest import GOLDEN
from tensoros_b200 import _ffi

pytestmark = pytest.mark.gpu


def test_sample_matches_reference_draws(gpu):
    lib = _ffi.nn()
    g = np.load(GOLDEN / "sample.npz")
    temps, words, toks = g["temps"], g["words"], g["tokens"]
    for ci in range(toks.shape[0]):
        x = np.ascontiguousarray(g[f"x{ci}"])
        for ti, t in enumerate(temps):
            for k in range(toks.shape[2]):
                got = lib.tos_sample(x.ctypes.data, len(x), float(t), int(words[ci, ti, k]))
                assert lib.tos_last_status() == 0
                assert got == toks[ci, ti, k], (ci, float(t), k, got, int(toks[ci, ti, k]))


def cases():
    rng = np.random.default_rng(5)
    yield rng.normal(0, 3, 32000).astype(np.float32)
    x = rng.normal(0, 1, 32000).astype(np.float32)
    x[rng.choice(32000, 60, replace=False)] = 4.0          # 60 equal maxima: ties across the cut
    yield x
    x = rng.normal(0, 1, 5000).astype(np.float32)
    top = np.sort(x)[-40]
    x[rng.choice(5000, 7, replace=False)] = top            # ties exactly at the 40th value
    yield x
    x = np.zeros(1000, np.float32)
    x[::3] = -0.0
    x[500] = 1.0
    yield x                                                # signed zeros compare equal
    yield rng.normal(0, 2, 17).astype(np.float32)          # fewer than 40 candidates
    yield np.round(rng.normal(0, 1, 32000) * 4).astype(np.float32) / 4   # many duplicates


@pytest.mark.parametrize("temperature", [0.0005, 0.2, 0.7, 1.0, 1.9])
def test_sample_matches_oracle(gpu, oracle, temperature):
    lib = _ffi.nn()
    rng = np.random.default_rng(11)
    for x in cases():
        for _ in range(24):
            ent = int(rng.integers(0, 2**32))
            got = lib.tos_sample(x.ctypes.data, len(x), temperature, ent)
            assert lib.tos_last_status() == 0
            want = oracle.sample(x, temperature, ent)
            assert got == want, (len(x), temperature, ent, got, want)


def test_sample_dev_on_stream(gpu, oracle):
    import torch
    lib = _ffi.nn()
    x = np.random.default_rng(3).normal(0, 2, 32000).astype(np.float32)
    dx = torch.from_numpy(x).cuda()
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    for ent in (0, 1, 12345, 2**32 - 1):
        assert lib.tos_sample_dev(dx.data_ptr(), len(x), 0.8, ent, out.data_ptr(), s) == 0
        torch.cuda.synchronize()
        assert int(out.item()) == oracle.sample(x, 0.8, ent)
