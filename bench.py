#!/usr/bin/env python
"""Decode throughput of the B200 TensorOS decode path.

Workload: Llama-2-7B-shaped decoder (32 layers, d_model 4096, 32 heads, SwiGLU
11008, vocab 32000), random-init Q4_0 weights (GGUF layout, seeded), fp16 KV
cache of capacity 4096; a 128-token prompt is prefilled, then greedy decode at
batch 1.  A step is one decoded token.

  value      tokens/s with the model resident in HBM: K greedy steps chained on
             the device (tos_model_decode), timed with CUDA events on the
             model's stream.  --math fast (default): FAST GEMV and attention
             arithmetic (normwise error <= 1e-4), each token one fused
             persistent kernel (decode_step_kernel; --per-op: a kernel per
             operator); --math exact: bit-identical to the reference, a
             kernel per operator.  With fast, "exact" reports the bit-exact
             arithmetic's tokens/s on the same prompt and whether its greedy
             ids equal the fast run's.  Weights (3.7 GB per step) exceed L2 (126 MB), so
             no flush is needed.
  e2e        the same metric through tos_model_forward_argmax: every step
             copies token+position host->device (8 B, pinned) and the next
             token device->host (8 B).
  roofline   the dominant kernel: the fused step (one launch per token: all
             weight planes + the KV rows of the context per launch), or with
             a kernel per operator the Q4_0 GEMV.  gemv_roofline: that GEMV
             timed in isolation on the 4096x4096 shape (one launch streams
             9,469,952 algorithmic bytes), rotating 32 weight copies (303 MB)
             so every launch is L2-cold.
  cpu_baseline  the reference's own C implementation (runtime/nn/llm.c,
             compiled hosted) on one host core, rank 0 at N=1.

--impl reference times that reference CPU implementation alone.
With --gpus N > 1 (one process per GPU) the value is one sequence
row-sharded over the N GPUs (strong scaling): each token is one fused
kernel per GPU whose epilogues store their rows straight into the peers'
vectors over NVLink.  "sharded_check" compares its greedy ids and next-step
logits with the one-GPU model's (rank 0); "replicas" adds N data-parallel
replicas, each GPU decoding its own sequence with the whole model (weak
scaling; --replicas makes that the value).
batch_decode: 16 sequences per step through the tensor-core GEMMs.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

GEMV_BYTES_4096 = 4096 * 128 * 18 + 4096 * 4 + 4096 * 4   # 9,469,952 B per launch
METRIC = "decode tokens/sec (Llama-2-7B-shaped, Q4_0, batch 1)"
# dram__bytes_read.sum + dram__bytes_write.sum of one decode_step_kernel launch
# of the 32-layer model, from a full-size ncu capture at context 8 (the KV rows
# of a longer context add 16 KB per position and layer)
STEP_TRAFFIC = 3721505024 + 15383296


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        # nvidia-smi numbers GPUs physically; CUDA_VISIBLE_DEVICES may remap
        vis = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
        self.gpu = vis[gpu_index] if gpu_index < len(vis) else str(gpu_index)
        self.proc = None
        self.lines = []
        self.start = 0

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            # the sampler is running (first line out) before the region starts
            t0 = time.time()
            while not self.lines and time.time() - t0 < 5.0 and self.proc.poll() is None:
                time.sleep(0.01)
        except Exception:
            self.proc = None
        self.start = len(self.lines)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            # a region shorter than the 200 ms interval still gets the sample
            # that closes it
            t0 = time.time()
            while len(self.lines) <= self.start and time.time() - t0 < 1.0 and self.proc.poll() is None:
                time.sleep(0.01)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines[self.start:]:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_info() -> dict:
    """The host CPU the baselines ran on: model name, online CPUs, and the
    CPUs this process may use."""
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    try:
        usable = len(os.sched_getaffinity(0))
    except Exception:
        usable = os.cpu_count()
    return {"cpu_model": model, "nproc": os.cpu_count(), "usable_cpus": usable}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def ref_cpu_decode(synth, n_tokens: int, start_pos: int, warmup: int):
    """Times the reference's llm_forward_token on this host (1 core)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import pyoracle
    if pyoracle.reference_available():
        ops, kind = pyoracle.reference(), "reference"
        model = ops.model(synth)
    else:
        ops, kind = pyoracle.oracle(), "port"
        model = ops.model(synth, kv_type=0)
    saved = None
    try:
        saved = os.sched_getaffinity(0)
        os.sched_setaffinity(0, {sorted(saved)[0]})
    except Exception:
        pass
    try:
        tok = 1
        pos = start_pos
        for _ in range(warmup):
            model.forward(tok, pos)
            pos += 1
        t0 = time.perf_counter()
        for _ in range(n_tokens):
            lg = model.forward(tok, pos)
            tok = int(lg.argmax())
            pos += 1
        dt = time.perf_counter() - t0
    finally:
        model.close()
        if saved:
            os.sched_setaffinity(0, saved)   # the process's other work keeps all its CPUs
    return n_tokens / dt, kind, dt


def run_reference(args, world, rank):
    if rank != 0:
        return
    from tensoros_b200 import workloads as W
    cfg = dict(W.LLAMA2_7B, kv_type=W.TYPE_F32)
    synth = W.make_model(cfg, W.SEED)
    # a bounded sample: at ~3 s per token on one core, the run times n
    # tokens after w warm-up tokens (the line reports those counts)
    n = max(1, min(args.steps, args.ref_tokens))
    w = min(args.warmup, 1)
    value, kind, dt = ref_cpu_decode(synth, n, args.prefill, w)
    sample = (f"{n} decode tokens (after {w} warm-up) at positions {args.prefill + w}.. of the 7B Q4_0 model, "
              f"fp32 KV cache (the reference's only cache type), prefix positions left zero instead of a "
              f"{args.prefill}-token CPU prefill; reference runtime/nn/llm.c built hosted, 1 core, {dt:.1f} s")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": n, "warmup": w, "steps_requested": args.steps, "ms_per_step": 1000.0 / value,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, random-init weights)",
        "config": {"workload": "llama2-7b-shape-q4_0 decode, batch 1", "global_batch": 1,
                   "seq_len": args.prefill, "parallelism": "none (CPU)"},
        "cpu_baseline": dict({"value": value, "unit": "tokens/s", "cores": 1, "kind": kind, "sample": sample},
                             **cpu_info()),
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def gemv_roofline(lib, torch, mode, n_copies=32, reps=4):
    """Isolated Q4_0 GEMV 4096x4096, L2-cold by rotating weight copies."""
    from tensoros_b200 import workloads as W
    return time_gemv(lib, torch, W.TYPE_Q4_0, 4096, 4096, (mode,), n_copies, reps)[mode]


def time_gemv(lib, torch, t, rows, cols, modes, n_copies, reps=4):
    """{mode: ms per launch} of one GEMV (tos_gemv_mode_dev) in a CUDA graph
    of back-to-back launches over n_copies weight copies (L2-cold when the
    copies exceed L2)."""
    import ctypes
    from tensoros_b200 import workloads as W
    hs = []
    try:
        for c in range(n_copies):
            w = W.quant(t, rows, cols, W.SEED, 9000 + c)
            h = ctypes.c_void_p()
            assert lib.tos_weight_create(ctypes.byref(h), w.ctypes.data, rows, cols, t) == 0
            hs.append(h)
        x = torch.from_numpy(W.normal_f32(cols, W.SEED, 9999)).cuda()
        y = torch.empty(rows, device="cuda")
        s = torch.cuda.Stream()
        res = {}
        for mode in modes:
            with torch.cuda.stream(s):
                sp = s.cuda_stream
                for h in hs[:4]:
                    assert lib.tos_gemv_mode_dev(h, x.data_ptr(), None, 0.0, y.data_ptr(), mode, sp) == 0
                s.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    for _ in range(reps):
                        for h in hs:
                            lib.tos_gemv_mode_dev(h, x.data_ptr(), None, 0.0, y.data_ptr(), mode, sp)
                g.replay()
                s.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(s)
                g.replay()
                e1.record(s)
                e1.synchronize()
            res[mode] = e0.elapsed_time(e1) / (reps * n_copies)
            del g
        return res
    finally:
        for h in hs:
            lib.tos_weight_destroy(h)


L2_BYTES = 126 << 20
ROTATE_BYTES = 256 << 20   # rotated inputs: more than twice L2, so every launch is L2-cold


def q8_0_sweep(lib, torch, peak):
    """The Q8_0 GEMV shapes of the weight sweep (batch 1, fp32 in/out), FAST
    and EXACT arithmetic: algorithmic bytes R*(C/32)*34 + 4C + 4R per
    launch, L2-cold."""
    from tensoros_b200 import workloads as W
    out = []
    for rows, cols in [(4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096)]:
        wbytes = rows * (cols // 32) * 34
        copies = max(2, -(-ROTATE_BYTES // wbytes))
        ms = time_gemv(lib, torch, W.TYPE_Q8_0, rows, cols, (1, 0), copies, reps=3)
        alg = wbytes + 4 * cols + 4 * rows
        row = {"rows": rows, "cols": cols, "algorithmic_bytes": alg, "copies_rotated": copies}
        for name, mode in (("fast", 1), ("exact", 0)):
            gbs = alg / (ms[mode] / 1000.0) / 1e9
            row[name] = {"launch_us": ms[mode] * 1000.0, "GB/s": gbs, "frac": gbs / peak}
        out.append(row)
    return out


def attention_sweep(lib, torch, peak):
    """Single-query decode attention, 32 heads x 128, fp16 KV cache at
    contexts 512 / 2048 / 4096 (tos_attention_dev, EXACT and FAST): K and V
    rows read once per call, L2-cold by rotating cache copies; seeded
    N(0,1) data."""
    nh, hd = 32, 128
    g = torch.Generator(device="cuda")
    g.manual_seed(1234)
    res = []
    s = torch.cuda.Stream()
    for ctx in (512, 2048, 4096):
        kvb = 2 * ctx * nh * hd * 2
        copies = max(2, -(-ROTATE_BYTES // kvb))
        ks = [torch.randn(ctx * nh * hd, generator=g, device="cuda").half() for _ in range(copies)]
        vs = [torch.randn(ctx * nh * hd, generator=g, device="cuda").half() for _ in range(copies)]
        q = torch.randn(nh * hd, generator=g, device="cuda")
        out = torch.empty(nh * hd, device="cuda")
        wsb = lib.tos_attention_workspace_bytes(nh, ctx)
        ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
        row = {"ctx": ctx, "heads": nh, "head_dim": hd, "algorithmic_bytes": kvb + 2 * nh * hd * 4,
               "copies_rotated": copies}
        for name, mode in (("exact", 0), ("fast", 1)):
            with torch.cuda.stream(s):
                def call(c):
                    return lib.tos_attention_dev(out.data_ptr(), q.data_ptr(), ks[c].data_ptr(), vs[c].data_ptr(), 1,
                                                 nh, nh, hd, ctx - 1, ctx, mode, ws.data_ptr(), wsb, s.cuda_stream)
                for c in range(copies):
                    assert call(c) == 0
                s.synchronize()
                reps = 3
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=s):
                    for _ in range(reps):
                        for c in range(copies):
                            call(c)
                gr.replay()
                s.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(s)
                gr.replay()
                e1.record(s)
                e1.synchronize()
            us = e0.elapsed_time(e1) * 1000.0 / (reps * copies)
            gbs = row["algorithmic_bytes"] / (us * 1e-6) / 1e9
            row[name] = {"call_us": us, "GB/s": gbs, "frac": gbs / peak}
            del gr
        res.append(row)
        del ks, vs
    return res


def tiny_llama_run(torch):
    """The tiny Llama config: the reference's golden 16-token prompt, then 256
    greedy tokens; the ids are compared with the reference's own golden run
    and the decode is timed (device-chained steps, CUDA events)."""
    import numpy as np
    from tensoros_b200 import ops
    from tensoros_b200 import workloads as W
    g = np.load(ROOT / "tests" / "golden" / "tiny_llama.npz")
    synth = W.make_model(W.TINY_LLAMA, int(g["seed"][0]))
    prompt, want = [int(t) for t in g["prompt"]], [int(t) for t in g["ids"]]
    res = {"prompt_tokens": len(prompt), "generated": len(want)}
    for name, kw in (("exact", {}), ("fast", dict(attn_mode=1, gemv_mode=1, fused_step=1))):
        model = ops.Model(synth, **kw)
        try:
            nxt = 0
            for i, t in enumerate(prompt):
                nxt = model.forward_argmax(t, i)
            stream = torch.cuda.ExternalStream(model.stream())
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            toks = model.decode(nxt, len(prompt), len(want) - 1)
            e1.record(stream)
            e1.synchronize()
            ms = e0.elapsed_time(e1)
            ids = [nxt] + [int(t) for t in toks]
            res[name] = {"tokens_per_s": (len(want) - 1) / (ms / 1000.0), "ms": ms,
                         "ids_identical_to_reference": ids == want, "fused": model.fused}
        finally:
            model.close()
    return res


def long_context_run(synth, torch, weight_bytes, peak, K=32):
    """The 7B model deep into its 4096-position fp16 cache: prefill to
    position 2048 and ~4000 (tensor-core prefill), then K greedy steps
    chained on the device (fused FAST step) at each; bytes per token =
    weights + the K and V rows of the context."""
    from tensoros_b200 import ops
    from tensoros_b200 import workloads as W
    cfg = synth.cfg
    L = cfg["n_layers"]
    prompt = [int(t) for t in W.tokens(4000, cfg["vocab_size"], W.SEED + 7)]
    model = ops.Model(synth, attn_mode=1, gemv_mode=1, fused_step=1)
    out = []
    try:
        nxt = model.prefill(prompt[:2048], 0)
        stream = torch.cuda.ExternalStream(model.stream())
        for start in (2048, 4000 - K):
            if start > 2048:
                nxt = model.prefill(prompt[2048 + K:start], 2048 + K)
            model.decode(nxt, start, 1)   # warm-up: the same graph, one step
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            toks = model.decode(nxt, start, K)
            e1.record(stream)
            e1.synchronize()
            ms = e0.elapsed_time(e1)
            ctx_mid = start + K // 2
            step_bytes = weight_bytes + L * 2 * (ctx_mid + 1) * cfg["dim"] * 2
            us = ms * 1000.0 / K
            out.append({"positions": [start, start + K - 1], "tokens_per_s": K / (ms / 1000.0), "ms_per_step": ms / K,
                        "GB/s": step_bytes / (us * 1e-6) / 1e9, "frac": step_bytes / (us * 1e-6) / 1e9 / peak,
                        "kv_bytes_per_step": L * 2 * (ctx_mid + 1) * cfg["dim"] * 2})
            nxt = int(toks[-1])
    finally:
        model.close()
    return out


def cpu_batch_worker(n_seq: int, n_tokens: int, start_pos: int):
    """Batch-16 CPU baseline: n_seq independent single-core runs of the
    reference's llm_forward_token on the 7B model, one process per CPU, run
    at the same time; forked from this process, which never touches CUDA.
    Prints one JSON line."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import pyoracle
    from tensoros_b200 import workloads as W
    cfg = dict(W.LLAMA2_7B, kv_type=W.TYPE_F32, max_seq=start_pos + n_tokens + 8)
    synth = W.make_model(cfg, W.SEED)
    kind = "reference" if pyoracle.reference_available() else "port"
    cpus = sorted(os.sched_getaffinity(0))
    n = min(n_seq, len(cpus))
    kids = []
    for i in range(n):
        r, w = os.pipe()
        pid = os.fork()
        if pid == 0:
            os.close(r)
            try:
                os.sched_setaffinity(0, {cpus[i]})
                ops = pyoracle.reference() if kind == "reference" else pyoracle.oracle()
                model = ops.model(synth) if kind == "reference" else ops.model(synth, kv_type=0)
                tok, pos = 1 + i, start_pos
                model.forward(tok, pos)   # warm-up
                pos += 1
                t0 = time.perf_counter()
                for _ in range(n_tokens):
                    tok = int(model.forward(tok, pos).argmax())
                    pos += 1
                os.write(w, json.dumps({"s": time.perf_counter() - t0}).encode())
            finally:
                os._exit(0)
        os.close(w)
        kids.append((pid, r))
    secs = []
    for pid, r in kids:
        data = b""
        while True:
            chunk = os.read(r, 4096)
            if not chunk:
                break
            data += chunk
        os.close(r)
        os.waitpid(pid, 0)
        if data:
            secs.append(json.loads(data)["s"])
    total = len(secs) * n_tokens / max(secs) if secs else None
    print(json.dumps({"value": total, "unit": "tokens/s", "cores": len(secs), "kind": kind,
                      "sample": f"{len(secs)} independent sequences, one process and one core each, run "
                                f"concurrently: {n_tokens} decode tokens each (after 1 warm-up) at positions "
                                f"{start_pos + 1}.. of the 7B Q4_0 model (fp32 KV, prefix positions zero); "
                                f"aggregate = sequences x tokens / the slowest sequence's time",
                      "per_sequence_s": secs}), flush=True)


def cpu_batch_baseline(n_seq=16, n_tokens=2, start_pos=128):
    """Runs cpu_batch_worker in a fresh CUDA-free process."""
    try:
        r = subprocess.run([sys.executable, str(Path(__file__).resolve()), "--cpu-batch-worker",
                            str(n_seq), str(n_tokens), str(start_pos)], capture_output=True, text=True, timeout=900)
        line = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
        return dict(json.loads(line[-1]), **cpu_info()) if line else {"error": r.stderr[-500:]}
    except Exception as e:   # the baseline is reported, not required
        return {"error": str(e)}


def run_gemv_only(args, local):
    import torch
    from tensoros_b200 import lib as _lib
    torch.cuda.set_device(local)
    lib = _lib()
    assert lib.tos_init(local) == 0, "tos_init failed"
    mode = int(args.math == "fast")
    ms = gemv_roofline(lib, torch, mode, n_copies=args.gemv_copies)
    peak, peak_kind = peaks()
    gbs = GEMV_BYTES_4096 / (ms / 1000.0) / 1e9
    print(json.dumps({"kernel": f"gemv Q4_0 4096x4096 {args.math}", "launch_us": ms * 1000.0, "GB/s": gbs,
                      "frac": gbs / peak, "peak_source": peak_kind, "copies": args.gemv_copies}), flush=True)


def time_batch(model, B, start, K, vocab, torch):
    """Batched decode (tos_model_decode_batch): B independent sequences, one
    token each per step, at positions start.. (the earlier cache rows of the
    batch caches are zeros); host-driven steps, CUDA events on the model's
    stream around K steps after 3 warm-up steps."""
    import numpy as np
    stream = torch.cuda.ExternalStream(model.stream())
    toks = [(17 * i + 5) % vocab for i in range(B)]
    pos = start
    for _ in range(3):
        toks = list(model.decode_batch(toks, [pos] * B))
        pos += 1
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(K):
        toks = list(model.decode_batch(toks, [pos] * B))
        pos += 1
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    return {"sequences": B, "steps": K, "ms_per_step": ms / K, "tokens_per_s": B * K / (ms / 1000.0),
            "positions": [start + 3, pos - 1],
            "note": "B greedy sequences per step, projections as tcgen05 GEMMs over the B tokens; "
                    "host-driven steps (8*B bytes in, 4*B out per step)"}


def time_prefill(model, prompt, prompt_next, torch):
    """The prompt as one batched pass (tos_model_prefill: tensor-core GEMMs),
    against the token-by-token pass the decode measurement ran."""
    stream = torch.cuda.ExternalStream(model.stream())
    times = []
    nxt = None
    for rep in range(3):
        model.reset()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        nxt = model.prefill(prompt, 0)
        e1.record(stream)
        e1.synchronize()
        if rep:
            times.append(e0.elapsed_time(e1))
    ms = min(times)
    return {"tokens": len(prompt), "ms": ms, "tokens_per_s": len(prompt) / (ms / 1000.0),
            "stepwise_ms": prompt_next["stepwise_s"] * 1000.0,
            "next_token_identical_to_stepwise": nxt == prompt_next["token"]}


def attention_once(lib, torch, ctx, calls=5):
    """FAST decode attention, 32 heads x 128, fp16 cache of ctx positions:
    `calls` calls on one cache (L2-warm after the first), the last timed."""
    nh, hd = 32, 128
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    k = torch.randn(ctx * nh * hd, generator=g, device="cuda").half()
    v = torch.randn(ctx * nh * hd, generator=g, device="cuda").half()
    q = torch.randn(nh * hd, generator=g, device="cuda")
    out = torch.empty(nh * hd, device="cuda")
    wsb = lib.tos_attention_workspace_bytes(nh, ctx)
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for i in range(calls):
        if i == calls - 1:
            e0.record(s)
        assert lib.tos_attention_dev(out.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), 1, nh, nh, hd,
                                     ctx - 1, ctx, 1, ws.data_ptr(), wsb, s.cuda_stream) == 0
    e1.record(s)
    e1.synchronize()
    return {"kernel": f"FAST attention 32x128 fp16, context {ctx}", "calls": calls,
            "last_call_us": e0.elapsed_time(e1) * 1000.0}


def gemm_roofline(lib, torch, m=128, n=22016, k=4096, reps=10):
    """Isolated tensor-core GEMM of the prefill (gate|up shape)."""
    import ctypes
    from tensoros_b200 import workloads as W
    w = W.q4_0(n, k, W.SEED, 9500)
    h = ctypes.c_void_p()
    assert lib.tos_weight_create(ctypes.byref(h), w.ctypes.data, n, k, W.TYPE_Q4_0) == 0
    try:
        x = torch.randn(m, k, device="cuda")
        y = torch.empty(m, n, device="cuda")
        wsb = lib.tos_gemm_workspace_bytes(m, n, k)
        ws = torch.empty(wsb + 256, dtype=torch.uint8, device="cuda")
        wp = (ws.data_ptr() + 255) & ~255
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            for _ in range(3):
                assert lib.tos_gemm_dev(h, x.data_ptr(), m, y.data_ptr(), wp, wsb, s.cuda_stream) == 0
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for _ in range(reps):
                lib.tos_gemm_dev(h, x.data_ptr(), m, y.data_ptr(), wp, wsb, s.cuda_stream)
            e1.record(s)
            e1.synchronize()
        us = e0.elapsed_time(e1) * 1000.0 / reps
    finally:
        lib.tos_weight_destroy(h)
    return us, 2.0 * m * n * k


def run_ours(args, world, rank, local):
    import numpy as np
    import torch
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        # no NVLink multicast (NVLS) objects: a rank that dies while bound to
        # one can fault its peers
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    from tensoros_b200 import lib as _lib
    from tensoros_b200 import ops
    from tensoros_b200 import workloads as W
    lib = _lib()
    assert lib.tos_init(local) == 0, "tos_init failed"
    cfg = dict(W.LLAMA2_7B)
    if args.layers:
        cfg["n_layers"] = args.layers   # profiling of a small case only; the metric is the 32-layer model
    t_gen = time.perf_counter()
    synth = W.make_model(cfg, W.SEED)
    fast = args.math == "fast"
    t_gen = time.perf_counter() - t_gen
    # several GPUs: one sequence row-sharded over them (strong scaling), or
    # with --replicas independent replicas, each decoding its own sequence
    replicas = world > 1 and args.replicas
    prompt = W.tokens(args.prefill, cfg["vocab_size"], W.SEED + (rank if replicas else 0))
    warm = max(3, args.warmup)
    K = args.steps
    if args.prefill + warm + 2 * K + 2 > cfg["max_seq"]:
        raise SystemExit("steps too large for the 4096-position cache")

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    prompt_next = {}

    def timed_decode(model, clk=None, prompt=prompt):
        """prompt token by token, W warm-up steps, then K chained steps
        (value) and K host round-trip steps (e2e); returns (ms, e2e ms, the
        2K greedy ids)"""
        nxt = 0
        t0 = time.perf_counter()
        for i, t in enumerate(prompt):
            nxt = model.forward_argmax(int(t), i)
        prompt_next["stepwise_s"] = time.perf_counter() - t0
        prompt_next["token"] = nxt
        pos = args.prefill
        toks = model.decode(nxt, pos, warm)
        nxt, pos = int(toks[-1]), pos + warm
        stream = torch.cuda.ExternalStream(model.stream())
        # the clock sampler starts (and delivers its first sample) before the
        # ranks meet: its start-up time differs from rank to rank, and a rank
        # that starts its steps early waits inside the sharded step for the
        # others, which the max over ranks would count
        if clk:
            clk.__enter__()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.cudart().cudaProfilerStart()
        e0.record(stream)
        toks = model.decode(nxt, pos, K)
        e1.record(stream)
        e1.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        if clk:
            clk.__exit__()
        barrier()
        ids = [int(t) for t in toks]
        nxt, pos = ids[-1], pos + K
        e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2.record(stream)
        for _ in range(K):
            nxt = model.forward_argmax(nxt, pos)
            ids.append(int(nxt))
            pos += 1
        e3.record(stream)
        e3.synchronize()
        barrier()
        return e0.elapsed_time(e1), e2.elapsed_time(e3), ids

    def shard(force=False):
        """row-sharding over the ranks (one sequence); a fresh communicator
        id for every model"""
        if world == 1 or (replicas and not force):
            return None
        obj = [ops.nccl_unique_id() if rank == 0 else None]
        torch.distributed.broadcast_object_list(obj, src=0)
        return (rank, world, obj[0])

    def untimed_sequence(model, prompt=prompt):
        """the token sequence timed_decode produces, on one GPU, untimed:
        the prompt, warm-up and chained steps, then host-driven steps"""
        nxt = 0
        for i, t in enumerate(prompt):
            nxt = model.forward_argmax(int(t), i)
        pos = args.prefill
        toks = model.decode(nxt, pos, warm)
        nxt, pos = int(toks[-1]), pos + warm
        ids = [int(t) for t in model.decode(nxt, pos, K)]
        nxt, pos = ids[-1], pos + K
        for _ in range(K):
            nxt = model.forward_argmax(nxt, pos)
            ids.append(int(nxt))
            pos += 1
        return ids

    # ---- value / e2e: the selected arithmetic
    clk = ClockSampler(local)
    model = ops.Model(synth, attn_mode=int(fast), gemv_mode=int(fast), shard=shard(),
                      fused_step=int(fast and not args.per_op))
    fused = model.fused
    t_ms, t_e2e, ids = timed_decode(model, clk)
    prefill = None
    if world == 1 and not args.no_prefill:
        prefill = time_prefill(model, prompt, prompt_next, torch)
    sharded_check = None
    if world > 1 and not replicas:
        # the sharded model's next-step logits (every rank takes part), then
        # on rank 0 the one-GPU model over the same tokens: greedy ids and
        # logits compared
        next_pos = args.prefill + warm + 2 * K
        lg_sharded = model.forward(ids[-1], next_pos)
        barrier()
        if rank == 0:
            one = ops.Model(synth, attn_mode=int(fast), gemv_mode=int(fast), fused_step=int(fast and not args.per_op))
            ids_one = untimed_sequence(one)
            lg_one = one.forward(ids_one[-1], next_pos)
            one.close()
            d = float(np.max(np.abs(lg_sharded.astype(np.float64) - lg_one)))
            sharded_check = {"ids_identical_to_one_gpu": ids_one == ids, "ids_compared": len(ids),
                             "next_logits_max_abs_diff": d,
                             "next_logits_bitwise_equal": bool(np.array_equal(lg_sharded.view(np.uint32),
                                                                                lg_one.view(np.uint32)))}
        barrier()
    model.close()
    batch = None
    if world == 1 and args.batch > 1:
        bmodel = ops.Model(synth)
        batch = time_batch(bmodel, args.batch, args.prefill, 16, cfg["vocab_size"], torch)
        bmodel.close()
    # ---- the bit-exact path on the same prompt: its speed, and whether the
    # greedy ids agree (EXACT equals the reference bit for bit)
    exact_ms, exact_ids = None, None
    if fast and not args.no_exact:
        model = ops.Model(synth, shard=shard())
        exact_ms, _, exact_ids = timed_decode(model)
        model.close()
    # beside the value: the other multi-GPU mode (data-parallel replicas
    # beside the sharded value, or the sharded sequence beside replicas)
    other_ms = None
    if world > 1 and not args.no_replicas:
        if replicas:
            model = ops.Model(synth, attn_mode=int(fast), gemv_mode=int(fast), shard=shard(force=True),
                              fused_step=int(fast and not args.per_op))
            # one sequence: every rank feeds the same prompt
            other_ms, _, _ = timed_decode(model, prompt=W.tokens(args.prefill, cfg["vocab_size"], W.SEED))
        else:
            model = ops.Model(synth, attn_mode=int(fast), gemv_mode=int(fast),
                              fused_step=int(fast and not args.per_op))
            other_ms, _, _ = timed_decode(model, prompt=W.tokens(args.prefill, cfg["vocab_size"], W.SEED + rank))
        model.close()
    if world > 1:
        tt = torch.tensor([t_ms, t_e2e, exact_ms or 0.0, other_ms or 0.0], device="cuda")
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.MAX)
        t_ms, t_e2e = float(tt[0]), float(tt[1])
        exact_ms = float(tt[2]) if exact_ms is not None else None
        other_ms = float(tt[3]) if other_ms is not None else None
    # tokens of the whole job: one sequence per replica, or one sequence
    # row-sharded over all GPUs
    seqs = world if replicas else 1
    value = seqs * K / (t_ms / 1000.0)
    e2e = seqs * K / (t_e2e / 1000.0)

    res = {}
    if rank == 0:
        gemv_ms = gemv_roofline(lib, torch, int(fast))
        if prefill is not None:
            g_us, g_flops = gemm_roofline(lib, torch)
            tpeak = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["bf16_tflops"] \
                if (ROOT / "MEASURED_PEAKS.json").exists() else 1590.0
            prefill["gemm_roofline"] = {
                "bound": "tensor", "kernel": "gemm_tc_kernel<Q4_0> 128x22016x4096", "launch_us": g_us,
                "achieved": g_flops / (g_us * 1e-6) / 1e12, "peak": tpeak, "unit": "TFLOP/s",
                "frac": g_flops / (g_us * 1e-6) / 1e12 / tpeak,
                "note": "algorithmic 2MNK; the exact fp16 hi/lo split issues 3 MMAs per product"}
        peak, peak_kind = peaks()
        achieved = GEMV_BYTES_4096 / (gemv_ms / 1000.0) / 1e9
        L = cfg["n_layers"]
        per_layer = 1 + 2 + 3   # QKV GEMV, attention (2 kernels), o / gate-up / down GEMVs
        launches = K if fused else K * (1 + L * per_layer + 3)
        weight_bytes = (L * (4096 * 128 * 18 * 4 + 3 * 11008 * 128 * 18) + 32000 * 128 * 18)
        # fused step: its own roofline, algorithmic bytes of one token = every
        # weight plane + the KV rows read and written (fp16) + the embedding
        # row, norms and the small vectors (<1 MB, ignored)
        ctx = args.prefill + warm + K // 2
        step_bytes = weight_bytes + L * 2 * (ctx + 1) * 4096 * 2
        gemv_rl = {"bound": "hbm", "kernel": f"tos_gemv_kernel<Q4_0, {args.math}> 4096x4096 (isolated, L2-cold)",
                   "achieved": achieved, "peak": peak, "peak_source": peak_kind, "unit": "GB/s",
                   "frac": achieved / peak,
                   # dram__bytes_read.sum + dram__bytes_write.sum of one launch
                   # of this kernel and shape, from an ncu capture of each
                   # arithmetic
                   "traffic": 9482496 if args.math == "fast" else 9485568,
                   "algorithmic_bytes_per_launch": GEMV_BYTES_4096, "launch_us": gemv_ms * 1000.0}
        step_us = t_ms / K * 1000.0
        # sharded: each GPU's launch streams its 1/N of the weights and KV rows
        shards = world if (world > 1 and not replicas) else 1
        launch_bytes = step_bytes / shards
        step_rl = {"bound": "hbm", "kernel": "decode_step_kernel (one launch per token, all layers)"
                   + (f", one of {shards} row-sharded launches" if shards > 1 else ""),
                   "achieved": launch_bytes / (step_us * 1e-6) / 1e9, "peak": peak, "peak_source": peak_kind,
                   "unit": "GB/s", "frac": launch_bytes / (step_us * 1e-6) / 1e9 / peak,
                   # dram bytes of one (one-GPU) launch at context 8 from an ncu
                   # capture, plus the KV rows of this context; no capture of a
                   # multi-rank launch exists (ncu never wraps a multi-rank run)
                   "traffic": STEP_TRAFFIC + L * 2 * (ctx - 8) * 4096 * 2 if shards == 1 else None,
                   "algorithmic_bytes_per_launch": launch_bytes, "launch_us": step_us}
        extra = {}
        if world == 1 and not args.no_extra:
            extra["q8_0_gemv_sweep"] = q8_0_sweep(lib, torch, peak)
            extra["attention"] = attention_sweep(lib, torch, peak)
            extra["tiny_llama"] = tiny_llama_run(torch)
            extra["long_context"] = long_context_run(synth, torch, weight_bytes, peak)
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            v, kind, dt = ref_cpu_decode(synth, args.ref_tokens, args.prefill, 1)
            cpu = dict({"value": v, "unit": "tokens/s", "cores": 1, "kind": kind,
                        "sample": f"{args.ref_tokens} decode tokens of the same 7B Q4_0 model (fp32 KV, the "
                                  f"reference's cache type) at positions {args.prefill + 1}.., one host core, "
                                  f"{dt:.1f} s"}, **cpu_info())
            if args.batch > 1 and not args.no_extra:
                # the batch-16 decode's baseline: 16 single-core reference runs
                cpu["batch16"] = cpu_batch_baseline(16, 2, args.prefill)
        res = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K,
            "warmup": warm, "ms_per_step": t_ms / K, "higher_is_better": True,
            "scaling": "weak" if replicas else "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init Q4_0 weights; BASELINE distributions)",
            "config": {"workload": "llama2-7b-shape-q4_0 greedy decode, batch 1, after a 128-token prefill",
                       "model": cfg["name"], "global_batch": 1, "seq_len": args.prefill,
                       "kv_cache": "fp16, capacity 4096", "arithmetic": args.math,
                       "step": "one fused kernel per token" if fused else "a kernel per operator (CUDA graph)",
                       "positions": [args.prefill + warm, args.prefill + warm + K - 1],
                       "parallelism": (f"{world} data-parallel replicas, one sequence each" if replicas else
                                       f"row-sharded x{world} (heads, rows, vocabulary; rows stored into the "
                                       "peers' vectors over NVLink inside the fused step)"
                                       if world > 1 else "single GPU"),
                       "l2": "inputs larger than L2 (3.72 GB of weights per step)"},
            "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8},
            "gpu_launches": launches,
            # the dominant kernel: the fused step when it runs, else the GEMV
            "roofline": step_rl if fused else gemv_rl,
            "gemv_roofline": gemv_rl,
            "decode_weight_gbs": weight_bytes * value / 1e9,   # all GPUs together
            "prefill": prefill,
            "batch_decode": batch,
            "clocks": clk.summary(),
            "sharded": None if not (replicas and other_ms) else {
                "value": K / (other_ms / 1000.0), "unit": "tokens/s", "ms_per_step": other_ms / K,
                "scaling": "strong", "note": f"one sequence row-sharded over {world} GPUs"},
            "replicas": None if (replicas or not other_ms) else {
                "value": world * K / (other_ms / 1000.0), "unit": "tokens/s", "ms_per_step": other_ms / K,
                "scaling": "weak", "note": f"{world} data-parallel replicas, one sequence each, the whole model "
                                           "on every GPU (slowest rank's time)"},
            "sharded_check": sharded_check,
            "exact": None if exact_ms is None else {
                "value": K / (exact_ms / 1000.0), "unit": "tokens/s", "ms_per_step": exact_ms / K,
                "greedy_ids_identical": exact_ids == ids, "ids_compared": len(ids)},
            "cpu_baseline": cpu,
            "setup_s": round(t_gen, 1),
        }
        res.update(extra)
        print(json.dumps(res), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--prefill", type=int, default=128)
    ap.add_argument("--math", default="fast", choices=["exact", "fast"],
                    help="exact: bit-identical to the reference; fast: FAST GEMV and attention "
                         "(normwise error <= 1e-4, greedy ids identical)")
    ap.add_argument("--ref-tokens", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--shard", action="store_true",
                    help="with several GPUs, row-shard one sequence over them (the default)")
    ap.add_argument("--replicas", action="store_true",
                    help="with several GPUs, one data-parallel replica per GPU as the value instead")
    ap.add_argument("--no-replicas", action="store_true", help="skip the second multi-GPU mode beside the value")
    ap.add_argument("--batch", type=int, default=16,
                    help="also time batched decode of this many sequences (0/1: skip)")
    ap.add_argument("--layers", type=int, default=0,
                    help="decoder layers (default: the 32 of the workload; fewer only to profile a small case)")
    ap.add_argument("--per-op", action="store_true",
                    help="fast arithmetic with a kernel per operator instead of the one fused kernel per token")
    ap.add_argument("--no-exact", action="store_true", help="skip the EXACT-arithmetic comparison run")
    ap.add_argument("--no-prefill", action="store_true", help="skip the batched-prefill measurement")
    ap.add_argument("--gemv-only", action="store_true",
                    help="time only the isolated Q4_0 4096x4096 GEMV (the roofline leg) and print it")
    ap.add_argument("--gemv-copies", type=int, default=32)
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the other workloads (Q8_0 GEMV sweep, attention, tiny llama, long context, "
                         "batch-16 CPU baseline)")
    ap.add_argument("--cpu-batch-worker", nargs=3, type=int, metavar=("SEQS", "TOKENS", "POS"),
                    help=argparse.SUPPRESS)
    ap.add_argument("--gemm-only", action="store_true",
                    help="time only the prefill tensor-core GEMM (128x22016x4096 Q4_0) and print it")
    ap.add_argument("--gemm-m", type=int, default=128,
                    help="--gemm-only: token rows of the gate|up GEMM (16 = a batch-16 decode step)")
    ap.add_argument("--attention-only", type=int, default=0, metavar="CTX",
                    help="time only FAST decode attention (32 heads x 128, fp16 cache) at this context: "
                         "five calls on one cache (the small case for a profiler capture)")
    args = ap.parse_args()
    if args.cpu_batch_worker:
        cpu_batch_worker(*args.cpu_batch_worker)
        return
    world, rank, local = dist_setup(args)
    if args.gemv_only:
        run_gemv_only(args, local)
    elif args.attention_only:
        import torch
        from tensoros_b200 import lib as _lib
        torch.cuda.set_device(local)
        lib = _lib()
        assert lib.tos_init(local) == 0, "tos_init failed"
        print(json.dumps(attention_once(lib, torch, args.attention_only)), flush=True)
    elif args.gemm_only:
        import torch
        from tensoros_b200 import lib as _lib
        torch.cuda.set_device(local)
        lib = _lib()
        assert lib.tos_init(local) == 0, "tos_init failed"
        us, flops = gemm_roofline(lib, torch, m=args.gemm_m)
        print(json.dumps({"kernel": f"gemm_tc Q4_0 {args.gemm_m}x22016x4096", "launch_us": us,
                          "TFLOP/s": flops / (us * 1e-6) / 1e12,
                          "weight_GB/s": 22016 * 4096 // 32 * 18 / (us * 1e-6) / 1e9}), flush=True)
    elif args.impl == "reference":
        run_reference(args, world, rank)
    else:
        run_ours(args, world, rank, local)


if __name__ == "__main__":
    main()
