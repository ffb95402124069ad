"""Multi-GPU row sharding, host side, on CPU: the product's partition plan
(tos_shard_plan / tos_shard_range) tiles every projection exactly, and a
forward pass computed slice by slice on world_size 2 and 4 gloo ranks (the
oracle's operators on each rank's rows, all-gathers between them) reproduces
the one-device oracle's logits bit for bit."""
import socket

import numpy as np
import pytest

from tensoros_b200 import ops
from tensoros_b200 import workloads as W


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("cfg", [W.LLAMA2_7B, W.SHARD_SMALL])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_tiles_every_projection(cfg, world):
    if cfg is W.SHARD_SMALL and world == 8:
        pytest.skip("4 kv heads")
    hd = cfg["dim"] // cfg["n_heads"]
    plans = [ops.shard_plan(cfg, world, r) for r in range(world)]
    spans = {"q": ("q_row0", "n_q_rows", cfg["n_heads"] * hd), "kv": ("kv_row0", "n_kv_rows", cfg["n_kv_heads"] * hd),
             "rows": ("row0", "n_rows", cfg["dim"]), "ff": ("ff0", "n_ff", cfg["ff_dim"]),
             "vocab": ("vocab0", "n_vocab", cfg["vocab_size"]),
             "heads": ("head0", "n_heads", cfg["n_heads"]), "kvh": ("kv_head0", "n_kv_heads", cfg["n_kv_heads"])}
    for name, (b, n, total) in spans.items():
        pos = 0
        for r, p in enumerate(plans):
            assert p[b] == pos, (name, r)        # contiguous, in rank order (gather order)
            assert p[n] == total // world
            pos += p[n]
        assert pos == total, name
    for p in plans:
        assert p["q_row0"] == p["head0"] * hd and p["kv_row0"] == p["kv_head0"] * hd
        for b, n in [("row0", "n_rows"), ("ff0", "n_ff"), ("vocab0", "n_vocab")]:
            assert p[b] % 32 == 0 and p[n] % 32 == 0
        # grouped-query attention stays local: a rank's query heads use its kv heads
        g = cfg["n_heads"] // cfg["n_kv_heads"]
        assert p["head0"] // g == p["kv_head0"] and p["n_heads"] == g * p["n_kv_heads"]


def test_plan_rejects_uneven_splits(lib):
    import ctypes as C
    b, n = C.c_int(), C.c_int()
    assert lib.tos_shard_range(4096, 32, 3, 0, C.byref(b), C.byref(n)) == -6      # TOS_ENOTSUP
    assert lib.tos_shard_range(4096, 32, 2, 2, C.byref(b), C.byref(n)) == -1      # rank out of range
    assert lib.tos_shard_range(4096, 32, 4, 3, C.byref(b), C.byref(n)) == 0
    assert (b.value, n.value) == (3072, 1024)
    with pytest.raises(ops.TosError):
        ops.shard_plan(W.TINY_LLAMA, 2, 0)          # 288 = 9 units of 32


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_forward_gloo_matches_oracle(world, oracle, tmp_path):
    import torch.multiprocessing as mp
    import shard_ref
    seed, n_steps = 17, 4
    out = tmp_path / "logits.npy"
    mp.start_processes(shard_ref.gloo_rank_main, args=(world, _free_port(), n_steps, seed, str(out)),
                       nprocs=world, join=True, start_method="spawn")
    got = np.load(out)
    m = W.make_model(W.SHARD_SMALL, seed)
    om = oracle.model(m)
    try:
        toks = W.tokens(n_steps, m.cfg["vocab_size"], seed)
        for i, t in enumerate(toks):
            ref = om.forward(int(t), i)
            assert np.array_equal(got[i].view(np.uint32), ref.view(np.uint32)), i
    finally:
        om.close()
