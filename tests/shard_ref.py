"""Test helper: one forward step of a row-sharded decoder restated with the
oracle's operators on one rank's rows, all-gathers through torch.distributed
(gloo on CPU).  The row ranges come from the product's plan
(tos_shard_plan), so the tests check the plan and the order of the
exchanges the sharded model uses (runtime/nn/llm.c:641-743 per row)."""
import numpy as np

from tensoros_b200 import workloads as W


def rows(w: np.ndarray, r0: int, n: int, cols: int, type_: int) -> np.ndarray:
    """Rows [r0, r0+n) of a GGUF-layout matrix (row-major, whole blocks)."""
    rb = (cols // 32) * W.BLOCK_BYTES[type_]
    return w[r0 * rb:(r0 + n) * rb]


class ShardedRef:
    def __init__(self, orc, synth, plan: dict, gather):
        self.orc, self.m, self.p, self.gather = orc, synth, plan, gather
        c = synth.cfg
        self.hd = c["dim"] // c["n_heads"]
        L, S = c["n_layers"], c["max_seq"]
        self.kc = [np.zeros((S, plan["n_kv_rows"]), np.float32) for _ in range(L)]
        self.vc = [np.zeros((S, plan["n_kv_rows"]), np.float32) for _ in range(L)]

    def forward(self, tok: int, pos: int) -> np.ndarray:
        o, m, p, c, hd = self.orc, self.m, self.p, self.m.cfg, self.hd
        dim, ff, wt, eps, base = c["dim"], c["ff_dim"], c["wtype"], c["norm_eps"], c["rope_base"]
        qd = c["n_heads"] * hd
        r0, nr = p["row0"], p["n_rows"]
        x = o.embed(m.token_embd, c["embd_type"], dim, tok)
        for l, Lw in enumerate(m.layers):
            xn = o.rmsnorm(x, Lw["attn_norm"], dim, 0, eps)
            q = o.gemv(rows(Lw["wq"], p["q_row0"], p["n_q_rows"], dim, wt), xn, p["n_q_rows"], dim, wt)
            k = o.gemv(rows(Lw["wk"], p["kv_row0"], p["n_kv_rows"], dim, wt), xn, p["n_kv_rows"], dim, wt)
            v = o.gemv(rows(Lw["wv"], p["kv_row0"], p["n_kv_rows"], dim, wt), xn, p["n_kv_rows"], dim, wt)
            for h in range(p["n_heads"]):
                q[h * hd:(h + 1) * hd] = o.rope(q[h * hd:(h + 1) * hd], pos, hd, base)
            for h in range(p["n_kv_heads"]):
                k[h * hd:(h + 1) * hd] = o.rope(k[h * hd:(h + 1) * hd], pos, hd, base)
            self.kc[l][pos] = k
            self.vc[l][pos] = v
            att = self.gather(o.attention(q, self.kc[l], self.vc[l], W.TYPE_F32, p["n_heads"], p["n_kv_heads"],
                                          hd, pos))
            y = o.gemv(rows(Lw["wo"], r0, nr, qd, wt), att, nr, qd, wt)
            x = self.gather(o.vadd_f32(x[r0:r0 + nr], y))
            xn = o.rmsnorm(x, Lw["ffn_norm"], dim, 0, eps)
            g = o.gemv(rows(Lw["wgate"], p["ff0"], p["n_ff"], dim, wt), xn, p["n_ff"], dim, wt)
            u = o.gemv(rows(Lw["wup"], p["ff0"], p["n_ff"], dim, wt), xn, p["n_ff"], dim, wt)
            hv = self.gather(o.vmul_f32(o.silu(g), u))
            y = o.gemv(rows(Lw["wdown"], r0, nr, ff, wt), hv, nr, ff, wt)
            x = self.gather(o.vadd_f32(x[r0:r0 + nr], y))
        xn = o.rmsnorm(x, m.output_norm, dim, 0, eps)
        lg = o.gemv(rows(m.output, p["vocab0"], p["n_vocab"], dim, c["out_type"]), xn, p["n_vocab"], dim,
                    c["out_type"])
        return self.gather(lg)


def gloo_rank_main(rank: int, world: int, port: int, n_steps: int, seed: int, out_path: str):
    """Child process: sharded forward steps; rank 0 saves the gathered logits."""
    import os
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root))
    sys.path.insert(0, str(root / "oracle"))
    import torch
    import torch.distributed as dist
    import pyoracle
    from tensoros_b200 import ops
    os.environ.setdefault("GLOO_SOCKET_IFNAME", "lo")
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        m = W.make_model(W.SHARD_SMALL, seed)
        plan = ops.shard_plan(m, world, rank)

        def gather(local):
            parts = [torch.empty(len(local), dtype=torch.float32) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(local, dtype=np.float32)))
            return np.concatenate([t.numpy() for t in parts])

        ref = ShardedRef(pyoracle.oracle(), m, plan, gather)
        toks = W.tokens(n_steps, m.cfg["vocab_size"], seed)
        out = np.stack([ref.forward(int(t), i) for i, t in enumerate(toks)])
        if rank == 0:
            np.save(out_path, out)
    finally:
        dist.destroy_process_group()
