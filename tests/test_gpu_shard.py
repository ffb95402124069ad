"""Row-sharded decoder on 2 GPUs (one process per GPU): every rank's logits
and greedy tokens equal the one-GPU model's, bit for bit, in EXACT and in
FAST arithmetic with a kernel per operator (NCCL all-gathers), and with the
fused FAST step, whose epilogues store each rank's rows into the peers'
vectors over NVLink and whose ranks meet at flag barriers (each row is
computed by the same arithmetic on the same inputs; the exchanges are
copies).  Needs two GPUs; skipped otherwise."""
import socket

import numpy as np
import pytest

from tensoros_b200 import ops
from tensoros_b200 import workloads as W

pytestmark = pytest.mark.gpu

WORLD = 2
N_STEPS = 6
N_DECODE = 12
CFGS = {"small": (W.SHARD_SMALL, None), "7b-2layer": (W.LLAMA2_7B, 2)}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(model, toks):
    logits = np.stack([model.forward(int(t), i) for i, t in enumerate(toks)])
    ids = model.decode(int(toks[-1]), len(toks), N_DECODE)
    return logits, ids


VARIANTS = {"exact": dict(attn_mode=0, gemv_mode=0), "fast": dict(attn_mode=1, gemv_mode=1),
            "fused": dict(attn_mode=1, gemv_mode=1, fused_step=1)}


def rank_main(rank, world, port, cfg_name, variant, out_path):
    import os
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import datetime
    import torch
    import torch.distributed as dist
    from tensoros_b200 import lib as _lib
    torch.cuda.set_device(rank)
    assert _lib().tos_init(rank) == 0
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    try:
        obj = [ops.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        cfg, layers = CFGS[cfg_name]
        synth = W.make_model(cfg, 23, n_layers=layers)
        model = ops.Model(synth, shard=(rank, world, obj[0]), **VARIANTS[variant])
        try:
            fused = model.fused
            toks = W.tokens(N_STEPS, cfg["vocab_size"], 23)
            logits, ids = _run(model, toks)
        finally:
            model.close()
        np.savez(f"{out_path}.{rank}.npz", logits=logits, ids=ids, fused=fused)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("cfg_name", list(CFGS))
@pytest.mark.parametrize("variant", list(VARIANTS))
def test_sharded_equals_one_gpu(gpu, cfg_name, variant, tmp_path):
    import torch
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    import torch.multiprocessing as mp
    out = str(tmp_path / "run")
    mp.start_processes(rank_main, args=(WORLD, _free_port(), cfg_name, variant, out), nprocs=WORLD, join=True,
                       start_method="spawn")
    cfg, layers = CFGS[cfg_name]
    synth = W.make_model(cfg, 23, n_layers=layers)
    model = ops.Model(synth, **VARIANTS[variant])
    try:
        assert model.fused == (variant == "fused")
        ref_logits, ref_ids = _run(model, W.tokens(N_STEPS, cfg["vocab_size"], 23))
    finally:
        model.close()
    for r in range(WORLD):
        got = np.load(f"{out}.{r}.npz")
        assert bool(got["fused"]) == (variant == "fused"), r
        assert np.array_equal(got["logits"].view(np.uint32), ref_logits.view(np.uint32)), r
        assert np.array_equal(got["ids"], ref_ids), r


def test_distributed_argmax_rule(gpu):
    """tos_argmax_sharded_dev (the sharded model's slice + pair kernels) on
    vectors where slices start with NaN, hold ties across slice borders, or
    are all NaN: the result is llm_argmax of the whole vector."""
    import torch
    from tensoros_b200 import lib as _lib
    rng = np.random.default_rng(5)
    n = 1024
    cases = []
    x = rng.standard_normal(n).astype(np.float32); cases.append(x)
    x = x.copy(); x[512] = np.nan; x[700] = 9.0; cases.append(x)              # NaN starts slice 1 of 2
    x = rng.standard_normal(n).astype(np.float32); x[0] = np.nan; cases.append(x)   # NaN at 0 wins
    x = np.zeros(n, np.float32); x[300] = x[800] = 3.0; cases.append(x)       # tie across slices
    x = np.full(n, np.nan, np.float32); x[5] = 1.0; cases.append(x)
    x = np.full(n, -np.inf, np.float32); x[900] = -1.0; cases.append(x)
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    for x in cases:
        # llm_argmax: first strict maximum starting from x[0]; NaN never beats it
        best, bv = 0, x[0]
        for i in range(1, n):
            if x[i] > bv:
                best, bv = i, x[i]
        want = best
        dx = torch.from_numpy(x).cuda()
        for world in (1, 2, 4, 8):
            assert _lib().tos_argmax_sharded_dev(dx.data_ptr(), n, world, out.data_ptr(),
                                                 torch.cuda.current_stream().cuda_stream) == 0
            torch.cuda.synchronize()
            assert int(out.item()) == want, (world, int(out.item()), want)
