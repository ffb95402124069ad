"""Host-buffer mirror of runtime/nn/llm.c's operators, bound to the C-ABI.

Each function calls the library's drop-in of the same reference operator
(tos_gemv for llm_gemv, tos_rmsnorm for llm_rmsnorm, ...) on numpy buffers
and raises TosError when the call's status is not TOS_OK.  In-place
operators of the reference (softmax, silu, rope, axpy, vadd, vmul) return a
new array rather than mutating the argument.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _ffi

_STATUS = {0: "ok", -1: "invalid argument", -2: "out of memory", -3: "CUDA error",
           -4: "collective error", -5: "device wait timed out", -6: "not supported",
           -7: "no CUDA device"}


class TosError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        super().__init__(f"{what}: {_STATUS.get(status, status)} ({status})")


def _lib():
    return _ffi.nn()


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _check(what: str, status: int | None = None):
    st = _lib().tos_last_status() if status is None else status
    if st != 0:
        raise TosError(st, what)


def init(device: int = 0):
    _check("tos_init", _lib().tos_init(device))


def _forget_weights():
    """tos_gemv / tos_vec_dot cache a quantised matrix by its host address, as
    the reference uses GGUF tensors in place.  A numpy buffer can be freed and
    its address reused by another array, so these wrappers drop the cache
    after every call (the C drop-ins keep it for callers whose weights stay
    put)."""
    _lib().tos_weight_cache_clear()


def gemv(weight: np.ndarray, x, out_dim: int, in_dim: int, type_: int) -> np.ndarray:
    out = np.empty(out_dim, dtype=np.float32)
    x = _f32(x)
    w = np.ascontiguousarray(weight)
    _lib().tos_gemv(_p(out), _p(w), _p(x), out_dim, in_dim, type_)
    st = _lib().tos_last_status()
    _forget_weights()
    _check("tos_gemv", st)
    return out


def vec_dot(weight: np.ndarray, x, n: int, type_: int) -> float:
    x = _f32(x)
    r = _lib().tos_vec_dot(_p(np.ascontiguousarray(weight)), _p(x), n, type_)
    st = _lib().tos_last_status()
    _forget_weights()
    _check("tos_vec_dot", st)
    return np.float32(r)


def q4_0_dot32(block: np.ndarray, x) -> np.float32:
    x = _f32(x)
    r = _lib().tos_q4_0_dot32(_p(np.ascontiguousarray(block)), _p(x))
    _check("tos_q4_0_dot32")
    return np.float32(r)


def q8_0_dot32(block: np.ndarray, x) -> np.float32:
    x = _f32(x)
    r = _lib().tos_q8_0_dot32(_p(np.ascontiguousarray(block)), _p(x))
    _check("tos_q8_0_dot32")
    return np.float32(r)


def embed(embd: np.ndarray, type_: int, dim: int, token: int) -> np.ndarray:
    out = np.empty(dim, dtype=np.float32)
    _lib().tos_embed(_p(out), _p(np.ascontiguousarray(embd)), type_, dim, token)
    _check("tos_embed")
    return out


def rmsnorm(x, w: np.ndarray, dim: int, wtype: int = 0) -> np.ndarray:
    x = _f32(x)
    out = np.empty(dim, dtype=np.float32)
    _lib().tos_rmsnorm(_p(out), _p(x), _p(np.ascontiguousarray(w)), dim, wtype)
    _check("tos_rmsnorm")
    return out


def rope(vec, pos: int, head_dim: int, base: float) -> np.ndarray:
    v = _f32(vec).copy()
    _lib().tos_rope(_p(v), pos, head_dim, base)
    _check("tos_rope")
    return v


def _inplace(name: str, x, *extra) -> np.ndarray:
    v = _f32(x).copy()
    getattr(_lib(), name)(_p(v), *extra)
    _check(name)
    return v


def softmax(x) -> np.ndarray:
    return _inplace("tos_softmax", x, len(x))


def silu(x) -> np.ndarray:
    return _inplace("tos_silu", x, len(x))


def dot_f32(a, b) -> np.float32:
    a, b = _f32(a), _f32(b)
    r = _lib().tos_dot_f32(_p(a), _p(b), len(a))
    _check("tos_dot_f32")
    return np.float32(r)


def axpy_f32(dst, scale: float, src) -> np.ndarray:
    d = _f32(dst).copy()
    s = _f32(src)
    _lib().tos_axpy_f32(_p(d), scale, _p(s), len(d))
    _check("tos_axpy_f32")
    return d


def vadd_f32(dst, src) -> np.ndarray:
    d = _f32(dst).copy()
    s = _f32(src)
    _lib().tos_vadd_f32(_p(d), _p(s), len(d))
    _check("tos_vadd_f32")
    return d


def vmul_f32(dst, src) -> np.ndarray:
    d = _f32(dst).copy()
    s = _f32(src)
    _lib().tos_vmul_f32(_p(d), _p(s), len(d))
    _check("tos_vmul_f32")
    return d


def argmax(logits) -> int:
    x = _f32(logits)
    r = _lib().tos_argmax(_p(x), len(x))
    _check("tos_argmax")
    return int(r)


def q4_dot_block(block20: np.ndarray, x) -> np.float32:
    x = _f32(x)
    r = _lib().tos_q4_dot_block(_p(np.ascontiguousarray(block20)), _p(x))
    _check("tos_q4_dot_block")
    return np.float32(r)


def q4_gemv(blocks20: np.ndarray, x, out_dim: int, in_dim: int) -> np.ndarray:
    out = np.empty(out_dim, dtype=np.float32)
    x = _f32(x)
    _lib().tos_q4_gemv(_p(out), _p(np.ascontiguousarray(blocks20)), _p(x), out_dim, in_dim)
    _check("tos_q4_gemv")
    return out


class Model:
    """tos_model_t built from a workloads.SynthModel (or any arrays with the
    same fields); mirrors llm_forward_token / greedy llm_generate."""

    def __init__(self, synth, attn_mode: int = 0, kv_type: int | None = None, gemv_mode: int = 0,
                 shard: tuple | None = None, fused_step: int = 0):
        """shard = (rank, world, nccl_id bytes): this process's rows of a model
        row-sharded over `world` GPUs (tos_model_create_sharded).
        fused_step = 1 runs each token as one fused persistent kernel where the
        model allows it (FAST arithmetic on one GPU)."""
        self.synth = synth
        self.desc = _ffi.ModelDesc()
        synth.fill_desc(self.desc, attn_mode=attn_mode, kv_type=kv_type, gemv_mode=gemv_mode)
        self.desc.fused_step = fused_step
        h = C.c_void_p()
        if shard is None:
            st = _lib().tos_model_create(C.byref(h), C.byref(self.desc))
            _check("tos_model_create", st)
        else:
            rank, world, nid = shard
            buf = C.create_string_buffer(bytes(nid), 128)
            st = _lib().tos_model_create_sharded(C.byref(h), C.byref(self.desc), rank, world, buf)
            _check("tos_model_create_sharded", st)
        self.h = h
        self.vocab = synth.cfg["vocab_size"]

    def close(self):
        if getattr(self, "h", None):
            _lib().tos_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        _check("tos_model_reset", _lib().tos_model_reset(self.h))

    def forward(self, token: int, pos: int, logits: bool = True):
        out = np.empty(self.vocab, dtype=np.float32) if logits else None
        st = _lib().tos_model_forward_token(self.h, _p(out) if logits else None, token, pos)
        _check("tos_model_forward_token", st)
        return out

    def forward_argmax(self, token: int, pos: int) -> int:
        nxt = C.c_int()
        _check("tos_model_forward_argmax", _lib().tos_model_forward_argmax(self.h, token, pos, C.byref(nxt)))
        return nxt.value

    def generate_greedy(self, prompt, n_gen: int) -> np.ndarray:
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(n_gen, 1), dtype=np.int32)
        n = _lib().tos_model_generate_greedy(self.h, _p(p), len(p), n_gen, _p(out))
        if n < 0:
            raise TosError(n, "tos_model_generate_greedy")
        return out[:n]

    def prefill(self, tokens, pos0: int = 0, logits: bool = False):
        """Batched prompt pass (tos_model_prefill): the greedy next token,
        and the last token's logits when asked."""
        p = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty(self.vocab, dtype=np.float32) if logits else None
        nxt = C.c_int()
        _check("tos_model_prefill", _lib().tos_model_prefill(self.h, _p(p), len(p), pos0,
                                                             _p(out) if logits else None, C.byref(nxt)))
        return (nxt.value, out) if logits else nxt.value

    def decode_batch(self, tokens, positions, slots=None, logits: bool = False):
        """One greedy step of len(tokens) independent sequences
        (tos_model_decode_batch); slots[i] is the KV-cache slot of sequence i
        (default 0..n-1).  The next token of each, and the logits when asked."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        p = np.ascontiguousarray(positions, dtype=np.int32)
        n = len(t)
        s = np.ascontiguousarray(range(n) if slots is None else slots, dtype=np.int32)
        out = np.empty((n, self.vocab), dtype=np.float32) if logits else None
        nxt = np.zeros(n, dtype=np.int32)
        _check("tos_model_decode_batch", _lib().tos_model_decode_batch(self.h, _p(s), _p(t), _p(p), n,
                                                                       _p(out) if logits else None, _p(nxt)))
        return (nxt, out) if logits else nxt

    def decode(self, token: int, pos: int, n_steps: int) -> np.ndarray:
        out = np.zeros(max(n_steps, 1), dtype=np.int32)
        _check("tos_model_decode", _lib().tos_model_decode(self.h, token, pos, n_steps, _p(out)))
        return out[:n_steps]

    def stream(self) -> int:
        return int(_lib().tos_model_stream(self.h) or 0)

    def device_bytes(self) -> int:
        return int(_lib().tos_model_device_bytes(self.h))

    @property
    def fused(self) -> bool:
        """True when each token runs as the one fused kernel (decode_step.cu)."""
        return bool(_lib().tos_model_fused(self.h))


def nccl_unique_id() -> bytes:
    """A fresh NCCL unique id (128 bytes) for tos_model_create_sharded."""
    buf = C.create_string_buffer(128)
    _check("tos_nccl_unique_id", _lib().tos_nccl_unique_id(buf, 128))
    return buf.raw


def shard_plan(synth_or_cfg, world: int, rank: int) -> dict:
    """The rows rank `rank` of `world` keeps (tos_shard_plan)."""
    d = _ffi.ModelDesc()
    cfg = synth_or_cfg.cfg if hasattr(synth_or_cfg, "cfg") else synth_or_cfg
    d.dim, d.n_layers, d.n_heads, d.n_kv_heads = cfg["dim"], cfg["n_layers"], cfg["n_heads"], cfg["n_kv_heads"]
    d.ff_dim, d.vocab_size, d.max_seq = cfg["ff_dim"], cfg["vocab_size"], cfg["max_seq"]
    p = _ffi.ShardPlan()
    _check("tos_shard_plan", _lib().tos_shard_plan(C.byref(d), world, rank, C.byref(p)))
    return {name: getattr(p, name) for name, _ in _ffi.ShardPlan._fields_}
