"""Seeded synthetic workloads for the TensorOS decode path (host numpy arrays).

Distributions follow the benchmark configurations of the decode path:
  * Q4_0 matrices: GGUF blocks, scale fp16(|N(0, 0.02)|), nibbles uniform 0..15
  * Q8_0 matrices: scale fp16(|N(0, 0.01)|), int8 uniform in [-127, 127]
  * activations N(0, 1) fp32; fp16 KV caches N(0, 1)
  * RMSNorm weights 1 + 0.1*N(0, 1) (F32)
Every tensor has its own stream id, so any tensor can be regenerated alone.
The generator is libtos_synth (host C, counter-based, thread-count
independent).
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass, field

import numpy as np

from . import _ffi

TYPE_F32, TYPE_F16, TYPE_Q4_0, TYPE_Q8_0 = 0, 1, 2, 8
BLOCK_BYTES = {TYPE_Q4_0: 18, TYPE_Q8_0: 34}
SEED = 20261201


def _threads() -> int:
    return max(1, min(64, os.cpu_count() or 1))


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def q4_0(rows: int, cols: int, seed: int = SEED, stream: int = 0, scale_std: float = 0.02) -> np.ndarray:
    nb = rows * (cols // 32)
    a = np.empty(nb * 18, dtype=np.uint8)
    _ffi.synth().tos_synth_q4_0(_ptr(a), nb, seed, stream, scale_std, _threads())
    return a


def q8_0(rows: int, cols: int, seed: int = SEED, stream: int = 0, scale_std: float = 0.01) -> np.ndarray:
    nb = rows * (cols // 32)
    a = np.empty(nb * 34, dtype=np.uint8)
    _ffi.synth().tos_synth_q8_0(_ptr(a), nb, seed, stream, scale_std, _threads())
    return a


def quant(type_: int, rows: int, cols: int, seed: int = SEED, stream: int = 0) -> np.ndarray:
    if type_ == TYPE_Q4_0:
        return q4_0(rows, cols, seed, stream)
    if type_ == TYPE_Q8_0:
        return q8_0(rows, cols, seed, stream)
    raise ValueError(f"unsupported quant type {type_}")


def q4f(rows: int, cols: int, seed: int = SEED, stream: int = 0, scale_std: float = 0.05) -> np.ndarray:
    nb = rows * (cols // 32)
    a = np.empty(nb * 20, dtype=np.uint8)
    _ffi.synth().tos_synth_q4f(_ptr(a), nb, seed, stream, scale_std, _threads())
    return a


def normal_f32(n: int, seed: int = SEED, stream: int = 0, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    a = np.empty(n, dtype=np.float32)
    _ffi.synth().tos_synth_normal_f32(_ptr(a), n, seed, stream, mean, std, _threads())
    return a


def normal_f16(n: int, seed: int = SEED, stream: int = 0, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    """fp16 bit patterns (uint16) of N(mean, std) values"""
    a = np.empty(n, dtype=np.uint16)
    _ffi.synth().tos_synth_normal_f16(_ptr(a), n, seed, stream, mean, std, _threads())
    return a


def tokens(n: int, vocab: int, seed: int = SEED, stream: int = 2_000_000) -> np.ndarray:
    a = np.empty(n, dtype=np.int32)
    _ffi.synth().tos_synth_tokens(_ptr(a), n, vocab, seed, stream)
    return a


def f32_to_f16_bits(x: float) -> int:
    return int(_ffi.synth().tos_synth_f32_to_f16(float(x)))


# --------------------------------------------------------------------- configs

GEMV_Q4_0 = dict(name="q4_0_gemv_4096x4096", type=TYPE_Q4_0, rows=4096, cols=4096)
Q8_0_SWEEP = [dict(name=f"q8_0_gemv_{r}x{c}", type=TYPE_Q8_0, rows=r, cols=c)
              for (r, c) in [(4096, 4096), (11008, 4096), (4096, 11008), (32000, 4096)]]
ATTENTION = dict(n_heads=32, n_kv=32, head_dim=128, ctxs=(512, 2048, 4096), rope_base=10000.0)

TINY_LLAMA = dict(name="tiny-llama-6L-288d-q8_0", dim=288, n_layers=6, n_heads=6, n_kv_heads=6,
                  ff_dim=768, vocab_size=32000, wtype=TYPE_Q8_0, embd_type=TYPE_Q8_0,
                  out_type=TYPE_Q8_0, kv_type=TYPE_F32, max_seq=288, rope_base=10000.0,
                  norm_eps=1e-6, n_prompt=16, n_gen=256)

LLAMA2_7B = dict(name="llama2-7b-shape-q4_0", dim=4096, n_layers=32, n_heads=32, n_kv_heads=32,
                 ff_dim=11008, vocab_size=32000, wtype=TYPE_Q4_0, embd_type=TYPE_Q4_0,
                 out_type=TYPE_Q4_0, kv_type=TYPE_F16, max_seq=4096, rope_base=10000.0,
                 norm_eps=1e-6, n_prompt=128, n_gen=256)

# A small grouped-query decoder whose every dimension splits over 1/2/4 ranks
# in 32-row units (8 heads of 32, 4 kv heads): the multi-GPU parity case.
SHARD_SMALL = dict(name="shard-small-2L-256d-gqa-q8_0", dim=256, n_layers=2, n_heads=8, n_kv_heads=4,
                   ff_dim=512, vocab_size=1024, wtype=TYPE_Q8_0, embd_type=TYPE_Q8_0,
                   out_type=TYPE_Q8_0, kv_type=TYPE_F32, max_seq=64, rope_base=10000.0,
                   norm_eps=1e-6, n_prompt=8, n_gen=16)


def stream_id(layer: int, what: str) -> int:
    names = ["wq", "wk", "wv", "wo", "wgate", "wup", "wdown", "attn_norm", "ffn_norm"]
    if layer < 0:
        return {"token_embd": 1_000_001, "output": 1_000_002, "output_norm": 1_000_003}[what]
    return 100 * layer + 1 + names.index(what)


@dataclass
class SynthModel:
    cfg: dict
    seed: int
    layers: list = field(default_factory=list)   # per layer dict of arrays
    token_embd: np.ndarray = None
    output: np.ndarray = None
    output_norm: np.ndarray = None
    _keep: list = field(default_factory=list)

    @property
    def head_dim(self) -> int:
        return self.cfg["dim"] // self.cfg["n_heads"]

    def _ptr_array(self, key: str):
        arr = (C.c_void_p * len(self.layers))(*[_ptr(l[key]) for l in self.layers])
        self._keep.append(arr)
        return arr

    def fill_desc(self, desc, attn_mode: int = 0, kv_type: int | None = None, gemv_mode: int = 0):
        """Fill a ctypes struct with tos_model_desc_t / orc_model_desc_t fields."""
        c = self.cfg
        desc.dim = c["dim"]; desc.n_layers = c["n_layers"]; desc.n_heads = c["n_heads"]
        desc.n_kv_heads = c["n_kv_heads"]; desc.ff_dim = c["ff_dim"]; desc.vocab_size = c["vocab_size"]
        desc.max_seq = c["max_seq"]; desc.rope_base = c["rope_base"]; desc.norm_eps = c["norm_eps"]
        desc.kv_type = c["kv_type"] if kv_type is None else kv_type
        if hasattr(desc, "attn_mode"):
            desc.attn_mode = attn_mode
        if hasattr(desc, "gemv_mode"):
            desc.gemv_mode = gemv_mode
        desc.wtype = c["wtype"]; desc.embd_type = c["embd_type"]; desc.out_type = c["out_type"]
        desc.token_embd = _ptr(self.token_embd)
        desc.output_weight = _ptr(self.output) if self.output is not None else None
        desc.output_norm = _ptr(self.output_norm)
        for key in ["attn_norm", "ffn_norm", "wq", "wk", "wv", "wo", "wgate", "wup", "wdown"]:
            setattr(desc, key, C.cast(self._ptr_array(key), C.POINTER(C.c_void_p)))
        return desc


def make_model(cfg: dict, seed: int = SEED, n_layers: int | None = None) -> SynthModel:
    cfg = dict(cfg)
    if n_layers is not None:
        cfg["n_layers"] = n_layers
    dim, ff, hd = cfg["dim"], cfg["ff_dim"], cfg["dim"] // cfg["n_heads"]
    qd, kvd = cfg["n_heads"] * hd, cfg["n_kv_heads"] * hd
    wt = cfg["wtype"]
    m = SynthModel(cfg=cfg, seed=seed)
    for l in range(cfg["n_layers"]):
        m.layers.append(dict(
            wq=quant(wt, qd, dim, seed, stream_id(l, "wq")),
            wk=quant(wt, kvd, dim, seed, stream_id(l, "wk")),
            wv=quant(wt, kvd, dim, seed, stream_id(l, "wv")),
            wo=quant(wt, dim, qd, seed, stream_id(l, "wo")),
            wgate=quant(wt, ff, dim, seed, stream_id(l, "wgate")),
            wup=quant(wt, ff, dim, seed, stream_id(l, "wup")),
            wdown=quant(wt, dim, ff, seed, stream_id(l, "wdown")),
            attn_norm=normal_f32(dim, seed, stream_id(l, "attn_norm"), 1.0, 0.1),
            ffn_norm=normal_f32(dim, seed, stream_id(l, "ffn_norm"), 1.0, 0.1),
        ))
    m.token_embd = quant(cfg["embd_type"], cfg["vocab_size"], dim, seed, stream_id(-1, "token_embd"))
    m.output = quant(cfg["out_type"], cfg["vocab_size"], dim, seed, stream_id(-1, "output"))
    m.output_norm = normal_f32(dim, seed, stream_id(-1, "output_norm"), 1.0, 0.1)
    return m


def prompt_tokens(cfg: dict, seed: int = SEED) -> np.ndarray:
    return tokens(cfg["n_prompt"], cfg["vocab_size"], seed)


# The fp32 transformer engine (runtime/nn/transformer.c): no quantisation,
# tied output embedding, eps 1e-5.  Parity shapes within the engine's
# raised harness limits (dim <= 512, max_seq <= 1024).
TF_SMALL = dict(name="tf-engine-2L-64d", dim=64, num_heads=4, ff_dim=128, num_layers=2, vocab_size=32, max_seq=128)
TF_MEDIUM = dict(name="tf-engine-4L-256d", dim=256, num_heads=8, ff_dim=688, num_layers=4, vocab_size=1000,
                 max_seq=512)


@dataclass
class TfModel:
    cfg: dict
    seed: int
    layers: list = field(default_factory=list)
    tok_embed: np.ndarray = None
    rms_final: np.ndarray = None
    _keep: list = field(default_factory=list)

    def fill_desc(self, desc):
        """Fill a ctypes struct with tos_tf_desc_t / the harness's ref_tf_desc_t fields."""
        c = self.cfg
        for k in ("dim", "num_heads", "ff_dim", "num_layers", "vocab_size", "max_seq"):
            setattr(desc, k, c[k])
        for key in ("wq", "wk", "wv", "wo", "w1", "w2", "w3", "rms_att", "rms_ffn"):
            arr = (C.c_void_p * len(self.layers))(*[_ptr(l[key]) for l in self.layers])
            self._keep.append(arr)
            setattr(desc, key, C.cast(arr, C.POINTER(C.c_void_p)))
        desc.tok_embed = _ptr(self.tok_embed)
        desc.rms_final = _ptr(self.rms_final)
        return desc


def make_tf_model(cfg: dict, seed: int = SEED) -> TfModel:
    """fp32 weights ~N(0, 1/dim) (rows of a projection keep activations near
    unit scale), norm weights 1 + 0.1 N(0,1), embeddings N(0,1)."""
    d, f = cfg["dim"], cfg["ff_dim"]
    m = TfModel(cfg=dict(cfg), seed=seed)
    s_d, s_f = 1.0 / np.sqrt(d), 1.0 / np.sqrt(f)
    for l in range(cfg["num_layers"]):
        base = 3_000_000 + 100 * l
        m.layers.append(dict(
            wq=normal_f32(d * d, seed, base + 0, 0.0, s_d), wk=normal_f32(d * d, seed, base + 1, 0.0, s_d),
            wv=normal_f32(d * d, seed, base + 2, 0.0, s_d), wo=normal_f32(d * d, seed, base + 3, 0.0, s_d),
            w1=normal_f32(f * d, seed, base + 4, 0.0, s_d), w2=normal_f32(d * f, seed, base + 5, 0.0, s_f),
            w3=normal_f32(f * d, seed, base + 6, 0.0, s_d),
            rms_att=normal_f32(d, seed, base + 7, 1.0, 0.1), rms_ffn=normal_f32(d, seed, base + 8, 1.0, 0.1)))
    m.tok_embed = normal_f32(cfg["vocab_size"] * d, seed, 3_999_000)
    m.rms_final = normal_f32(d, seed, 3_999_001, 1.0, 0.1)
    return m
