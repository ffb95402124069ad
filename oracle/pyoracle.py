"""ctypes binding of the CPU checkers (TEST INFRASTRUCTURE ONLY).

  Oracle     - the C restatement oracle/tos_oracle.c (oracle/_build/liboracle.so)
  Reference  - the reference's own runtime/nn sources compiled hosted
               (oracle/_ref/libtos_ref.so); present only where the reference
               tree was available at build time.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module; the product library never loads either .so.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "liboracle.so"
REF_SO = HERE / "_ref" / "libtos_ref.so"

vp, i32, f32 = C.c_void_p, C.c_int, C.c_float


class _Desc(C.Structure):
    """orc_model_desc_t"""
    _fields_ = [
        ("dim", i32), ("n_layers", i32), ("n_heads", i32), ("n_kv_heads", i32),
        ("ff_dim", i32), ("vocab_size", i32), ("max_seq", i32),
        ("rope_base", f32), ("norm_eps", f32),
        ("wtype", i32), ("embd_type", i32), ("out_type", i32), ("kv_type", i32),
        ("token_embd", vp), ("output_weight", vp), ("output_norm", vp),
        ("attn_norm", C.POINTER(vp)), ("ffn_norm", C.POINTER(vp)),
        ("wq", C.POINTER(vp)), ("wk", C.POINTER(vp)), ("wv", C.POINTER(vp)), ("wo", C.POINTER(vp)),
        ("wgate", C.POINTER(vp)), ("wup", C.POINTER(vp)), ("wdown", C.POINTER(vp)),
    ]


class _RefDesc(C.Structure):
    """ref_model_desc_t of oracle/ref_llm_hosted.c"""
    _fields_ = [
        ("dim", i32), ("n_layers", i32), ("n_heads", i32), ("n_kv_heads", i32),
        ("ff_dim", i32), ("vocab_size", i32), ("max_seq", i32),
        ("rope_base", f32),
        ("wtype", i32), ("embd_type", i32), ("out_type", i32),
        ("token_embd", vp), ("output_weight", vp), ("output_norm", vp),
        ("attn_norm", C.POINTER(vp)), ("ffn_norm", C.POINTER(vp)),
        ("wq", C.POINTER(vp)), ("wk", C.POINTER(vp)), ("wv", C.POINTER(vp)), ("wo", C.POINTER(vp)),
        ("wgate", C.POINTER(vp)), ("wup", C.POINTER(vp)), ("wdown", C.POINTER(vp)),
    ]


def _p(a):
    return None if a is None else a.ctypes.data


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


class _Ops:
    """Common operator surface; prefix 'orc_' (restatement) or 'ref_'."""

    def __init__(self, path: Path, prefix: str):
        if not path.exists():
            raise FileNotFoundError(f"{path} not built")
        self.lib = C.CDLL(str(path))
        self.px = prefix
        sig = {
            "fp16_to_fp32": (f32, [C.c_uint16]),
            "expf": (f32, [f32]),
            "sqrtf": (f32, [f32]),
            "q4_0_dot32": (f32, [vp, vp]),
            "q8_0_dot32": (f32, [vp, vp]),
            "vec_dot": (f32, [vp, vp, i32, i32]),
            "gemv": (None, [vp, vp, vp, i32, i32, i32]),
            "softmax": (None, [vp, i32]),
            "silu": (None, [vp, i32]),
            "dot_f32": (f32, [vp, vp, i32]),
            "axpy_f32": (None, [vp, f32, vp, i32]),
            "vadd_f32": (None, [vp, vp, i32]),
            "vmul_f32": (None, [vp, vp, i32]),
            "argmax": (i32, [vp, i32]),
            "rope": (None, [vp, i32, i32, f32]),
            "model_free": (None, [vp]),
            "forward_token": (None, [vp, vp, i32, i32]),
            "generate_greedy": (i32, [vp, vp, i32, i32, vp]),
        }
        for name, (res, args) in sig.items():
            f = getattr(self.lib, prefix + name)
            f.restype, f.argtypes = res, args
        self.f = lambda name: getattr(self.lib, prefix + name)

    # scalar helpers
    def fp16_to_fp32(self, h): return np.float32(self.f("fp16_to_fp32")(int(h)))
    def expf(self, x): return np.float32(self.f("expf")(float(x)))

    def q4_0_dot32(self, block, x):
        return np.float32(self.f("q4_0_dot32")(_p(np.ascontiguousarray(block)), _p(_f32(x))))

    def q8_0_dot32(self, block, x):
        return np.float32(self.f("q8_0_dot32")(_p(np.ascontiguousarray(block)), _p(_f32(x))))

    def vec_dot(self, w, x, n, t):
        return np.float32(self.f("vec_dot")(_p(np.ascontiguousarray(w)), _p(_f32(x)), n, t))

    def gemv(self, w, x, out_dim, in_dim, t):
        out = np.empty(out_dim, dtype=np.float32)
        self.f("gemv")(_p(out), _p(np.ascontiguousarray(w)), _p(_f32(x)), out_dim, in_dim, t)
        return out

    def _inpl(self, name, x, *extra):
        v = _f32(x).copy()
        self.f(name)(_p(v), *extra)
        return v

    def softmax(self, x): return self._inpl("softmax", x, len(x))
    def silu(self, x): return self._inpl("silu", x, len(x))
    def rope(self, v, pos, hd, base): return self._inpl("rope", v, pos, hd, base)

    def dot_f32(self, a, b):
        return np.float32(self.f("dot_f32")(_p(_f32(a)), _p(_f32(b)), len(a)))

    def axpy_f32(self, d, s, src):
        v = _f32(d).copy()
        self.f("axpy_f32")(_p(v), s, _p(_f32(src)), len(v))
        return v

    def vadd_f32(self, d, s):
        v = _f32(d).copy()
        self.f("vadd_f32")(_p(v), _p(_f32(s)), len(v))
        return v

    def vmul_f32(self, d, s):
        v = _f32(d).copy()
        self.f("vmul_f32")(_p(v), _p(_f32(s)), len(v))
        return v

    def argmax(self, x): return int(self.f("argmax")(_p(_f32(x)), len(x)))


class Oracle(_Ops):
    def __init__(self):
        super().__init__(ORACLE_SO, "orc_")
        L = self.lib
        L.orc_fp32_to_fp16.restype, L.orc_fp32_to_fp16.argtypes = C.c_uint16, [f32]
        L.orc_gemv_threads.restype, L.orc_gemv_threads.argtypes = None, [vp, vp, vp, i32, i32, i32, i32]
        L.orc_embed.restype, L.orc_embed.argtypes = None, [vp, vp, i32, i32, i32]
        L.orc_rmsnorm.restype, L.orc_rmsnorm.argtypes = None, [vp, vp, vp, i32, i32, f32]
        L.orc_rope_cs.restype, L.orc_rope_cs.argtypes = None, [i32, i32, i32, f32, C.POINTER(f32), C.POINTER(f32)]
        L.orc_rope_rows.restype, L.orc_rope_rows.argtypes = None, [vp, i32, i32, i32, vp, f32]
        L.orc_attention.restype, L.orc_attention.argtypes = None, [vp, vp, vp, vp, i32, i32, i32, i32, i32]
        L.orc_q4f_dot_block.restype, L.orc_q4f_dot_block.argtypes = f32, [vp, vp]
        L.orc_q4f_gemv.restype, L.orc_q4f_gemv.argtypes = None, [vp, vp, vp, i32, i32]
        L.orc_model_create.restype, L.orc_model_create.argtypes = vp, [C.POINTER(_Desc)]
        L.orc_model_kcache.restype, L.orc_model_kcache.argtypes = vp, [vp, i32]
        L.orc_model_vcache.restype, L.orc_model_vcache.argtypes = vp, [vp, i32]
        L.orc_model_hidden.restype, L.orc_model_hidden.argtypes = C.POINTER(f32), [vp]
        L.orc_sample.restype, L.orc_sample.argtypes = i32, [vp, i32, f32, C.c_uint32]

    def fp32_to_fp16(self, x): return int(self.lib.orc_fp32_to_fp16(float(x)))

    def sample(self, logits, temperature, entropy):
        return int(self.lib.orc_sample(_p(_f32(logits)), len(logits), float(temperature), int(entropy) & 0xFFFFFFFF))

    def gemv_mt(self, w, x, out_dim, in_dim, t, threads=8):
        out = np.empty(out_dim, dtype=np.float32)
        self.lib.orc_gemv_threads(_p(out), _p(np.ascontiguousarray(w)), _p(_f32(x)), out_dim, in_dim, t, threads)
        return out

    def embed(self, embd, t, dim, tok):
        out = np.empty(dim, dtype=np.float32)
        self.lib.orc_embed(_p(out), _p(np.ascontiguousarray(embd)), t, dim, tok)
        return out

    def rmsnorm(self, x, w, dim, wtype=0, eps=1e-6):
        out = np.empty(dim, dtype=np.float32)
        self.lib.orc_rmsnorm(_p(out), _p(_f32(x)), _p(np.ascontiguousarray(w)), wtype, dim, eps)
        return out

    def rope_cs(self, pos, i, hd, base):
        c, s = f32(), f32()
        self.lib.orc_rope_cs(pos, i, hd, base, C.byref(c), C.byref(s))
        return np.float32(c.value), np.float32(s.value)

    def rope_rows(self, rows, hd, positions, base):
        r = _f32(rows).copy()
        pos = np.ascontiguousarray(positions, dtype=np.int32)
        self.lib.orc_rope_rows(_p(r), r.shape[0], r.shape[1], hd, _p(pos), base)
        return r

    def attention(self, q, kc, vc, kv_type, n_heads, n_kv, hd, pos):
        out = np.empty(n_heads * hd, dtype=np.float32)
        self.lib.orc_attention(_p(out), _p(_f32(q)), _p(np.ascontiguousarray(kc)), _p(np.ascontiguousarray(vc)),
                               kv_type, n_heads, n_kv, hd, pos)
        return out

    def q4_dot_block(self, b, x):
        return np.float32(self.lib.orc_q4f_dot_block(_p(np.ascontiguousarray(b)), _p(_f32(x))))

    def q4_gemv(self, b, x, out_dim, in_dim):
        out = np.empty(out_dim, dtype=np.float32)
        self.lib.orc_q4f_gemv(_p(out), _p(np.ascontiguousarray(b)), _p(_f32(x)), out_dim, in_dim)
        return out

    def model(self, synth, kv_type=None):
        return _Model(self, synth, _Desc, "orc_", kv_type)


class Reference(_Ops):
    def __init__(self):
        super().__init__(REF_SO, "ref_")
        L = self.lib
        L.ref_embed.restype, L.ref_embed.argtypes = None, [vp, vp, i32, i32, i32]
        L.ref_rmsnorm.restype, L.ref_rmsnorm.argtypes = None, [vp, vp, vp, i32, i32]
        L.ref_model_create.restype, L.ref_model_create.argtypes = vp, [C.POINTER(_RefDesc)]
        L.q4_dot_block.restype, L.q4_dot_block.argtypes = f32, [vp, vp]
        L.q4_gemv.restype, L.q4_gemv.argtypes = None, [vp, vp, vp, i32, i32]
        L.ref_sample_at.restype, L.ref_sample_at.argtypes = i32, [vp, i32, f32, C.c_uint32]
        L.ref_tf_rmsnorm.restype, L.ref_tf_rmsnorm.argtypes = None, [vp, vp, vp, i32]
        L.ref_tf_swiglu_ffn.restype, L.ref_tf_swiglu_ffn.argtypes = None, [vp, vp, vp, vp, vp, i32, i32]
        L.ref_tf_model_init.restype, L.ref_tf_model_init.argtypes = i32, [vp]
        L.ref_tf_forward_token.restype, L.ref_tf_forward_token.argtypes = None, [vp, vp, i32]
        L.ref_tf_cached_attention.restype, L.ref_tf_cached_attention.argtypes = None, [vp, vp, vp, vp, i32, i32, i32]
        L.ref_tf_reset.restype, L.ref_tf_reset.argtypes = None, []

    # ---- the tensor engine's CPU operators (runtime/tensor/tensor_cpu.c) and
    # its routing rule (tensor_engine.c:28-67), their own code
    def _engine_bind(self):
        L = self.lib
        if getattr(self, "_eng", False):
            return L
        L.tensor_cpu_matmul.restype, L.tensor_cpu_matmul.argtypes = None, [vp, vp, vp, i32, i32, i32]
        L.tensor_cpu_softmax.restype, L.tensor_cpu_softmax.argtypes = None, [vp, vp, i32]
        L.tensor_cpu_layernorm.restype, L.tensor_cpu_layernorm.argtypes = None, [vp, vp, i32, f32]
        L.tensor_cpu_attention.restype, L.tensor_cpu_attention.argtypes = None, [vp, vp, vp, vp, i32, i32]
        L.ref_select_backend.restype, L.ref_select_backend.argtypes = i32, [i32, vp, i32, i32]
        self._eng = True
        return L

    def engine_matmul(self, A, B):
        L = self._engine_bind()
        A, B = _f32(A), _f32(B)
        M, K = A.shape
        N = B.shape[1]
        C_ = np.empty((M, N), np.float32)
        L.tensor_cpu_matmul(_p(C_), _p(A), _p(B), M, N, K)
        return C_

    def engine_softmax_rows(self, X):
        L = self._engine_bind()
        X = _f32(X)
        out = np.empty_like(X)
        for i in range(X.shape[0]):
            row = np.array(X[i], np.float32, copy=True)   # a fresh, 16-byte aligned buffer
            o = np.empty_like(row)
            L.tensor_cpu_softmax(_p(o), _p(row), len(row))
            out[i] = o
        return out

    def engine_layernorm_rows(self, X, eps):
        L = self._engine_bind()
        X = _f32(X)
        out = np.empty_like(X)
        for i in range(X.shape[0]):
            row = np.array(X[i], np.float32, copy=True)   # a fresh, 16-byte aligned buffer
            o = np.empty_like(row)
            L.tensor_cpu_layernorm(_p(o), _p(row), len(row), float(eps))
            out[i] = o
        return out

    def engine_attention(self, Q, K, V):
        L = self._engine_bind()
        Q, K, V = _f32(Q), _f32(K), _f32(V)
        seq, hd = Q.shape
        out = np.empty((seq, hd), np.float32)
        L.tensor_cpu_attention(_p(out), _p(Q), _p(K), _p(V), seq, hd)
        return out

    def select_backend(self, op, sizes, gpu_count):
        L = self._engine_bind()
        a = np.ascontiguousarray(sizes, dtype=np.uint64)
        return int(L.ref_select_backend(int(op), _p(a), len(a), int(gpu_count)))

    # ---- the fp32 transformer engine (runtime/nn/transformer.c), its own code
    def tf_rmsnorm(self, x, w):
        x, w = _f32(x), _f32(w)
        out = np.empty(len(x), np.float32)
        self.lib.ref_tf_rmsnorm(_p(out), _p(x), _p(w), len(x))
        return out

    def tf_swiglu_ffn(self, x, w1, w2, w3, dim, ff_dim):
        out = np.empty(dim, np.float32)
        self.lib.ref_tf_swiglu_ffn(_p(out), _p(_f32(x)), _p(_f32(w1)), _p(_f32(w2)), _p(_f32(w3)), dim, ff_dim)
        return out

    def tf_model(self, tf):
        """The engine over a workloads.TfModel (one at a time: its KV store is
        static)."""
        return _TfRef(self, tf)

    def sample_at(self, logits, temperature, tsc_lo):
        """The reference's own llm_sample with its timestamp read returning
        tsc_lo (oracle/ref_llm_hosted.c); -1 where the timestamp cannot be
        scripted on this host."""
        x = _f32(logits)
        return int(self.lib.ref_sample_at(_p(x), len(x), float(temperature), int(tsc_lo) & 0xFFFFFFFF))

    def embed(self, embd, t, dim, tok):
        out = np.empty(dim, dtype=np.float32)
        self.lib.ref_embed(_p(out), _p(np.ascontiguousarray(embd)), t, dim, tok)
        return out

    def rmsnorm(self, x, w, dim, wtype=0):
        out = np.empty(dim, dtype=np.float32)
        self.lib.ref_rmsnorm(_p(out), _p(_f32(x)), _p(np.ascontiguousarray(w)), dim, wtype)
        return out

    def q4_dot_block(self, b, x):
        return np.float32(self.lib.q4_dot_block(_p(np.ascontiguousarray(b)), _p(_f32(x))))

    def q4_gemv(self, b, x, out_dim, in_dim):
        out = np.empty(out_dim, dtype=np.float32)
        self.lib.q4_gemv(_p(out), _p(np.ascontiguousarray(b)), _p(_f32(x)), out_dim, in_dim)
        return out

    def model(self, synth):
        return _Model(self, synth, _RefDesc, "ref_", None)


class _Model:
    def __init__(self, ops, synth, desc_cls, px, kv_type):
        self.ops, self.px = ops, px
        d = desc_cls()
        if hasattr(d, "norm_eps"):
            synth.fill_desc(d, kv_type=kv_type)
        else:
            _fill_ref(d, synth)
        self.desc = d
        self.vocab = synth.cfg["vocab_size"]
        self.h = getattr(ops.lib, px + "model_create")(C.byref(d))
        if not self.h:
            raise MemoryError("model_create failed")

    def close(self):
        if self.h:
            getattr(self.ops.lib, self.px + "model_free")(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, token, pos):
        out = np.empty(self.vocab, dtype=np.float32)
        getattr(self.ops.lib, self.px + "forward_token")(self.h, _p(out), token, pos)
        return out

    def hidden(self):
        """The last step's normalised final hidden state (the LM head's
        input); restatement models only."""
        dim = self.desc.dim
        ptr = getattr(self.ops.lib, self.px + "model_hidden")(self.h)
        return np.ctypeslib.as_array(ptr, (dim,)).copy()

    def generate_greedy(self, prompt, n_gen):
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(1, n_gen), dtype=np.int32)
        n = getattr(self.ops.lib, self.px + "generate_greedy")(self.h, _p(p), len(p), n_gen, _p(out))
        return out[:n]


class _TfRef:
    def __init__(self, ref, tf):
        from tensoros_b200 import _ffi
        self.ref, self.tf = ref, tf
        self.desc = tf.fill_desc(_ffi.TfDesc())
        if ref.lib.ref_tf_model_init(C.byref(self.desc)) != 0:
            raise ValueError("shape beyond the harness limits")

    def forward(self, token, pos):
        c = self.tf.cfg
        row = np.ascontiguousarray(self.tf.tok_embed[token * c["dim"]:(token + 1) * c["dim"]])
        out = np.empty(c["vocab_size"], np.float32)
        self.ref.lib.ref_tf_forward_token(_p(out), _p(row), pos)
        return out

    def cached_attention(self, q, k, v, layer, head, pos):
        out = np.empty(len(q), np.float32)
        self.ref.lib.ref_tf_cached_attention(_p(out), _p(_f32(q)), _p(_f32(k)), _p(_f32(v)), layer, head, pos)
        return out

    def reset(self):
        self.ref.lib.ref_tf_reset()


def _fill_ref(d, synth):
    c = synth.cfg
    d.dim, d.n_layers, d.n_heads, d.n_kv_heads = c["dim"], c["n_layers"], c["n_heads"], c["n_kv_heads"]
    d.ff_dim, d.vocab_size, d.max_seq, d.rope_base = c["ff_dim"], c["vocab_size"], c["max_seq"], c["rope_base"]
    d.wtype, d.embd_type, d.out_type = c["wtype"], c["embd_type"], c["out_type"]
    d.token_embd = _p(synth.token_embd)
    d.output_weight = _p(synth.output)
    d.output_norm = _p(synth.output_norm)
    for key in ["attn_norm", "ffn_norm", "wq", "wk", "wv", "wo", "wgate", "wup", "wdown"]:
        setattr(d, key, C.cast(synth._ptr_array(key), C.POINTER(C.c_void_p)))


def oracle() -> Oracle:
    return Oracle()


def reference_available() -> bool:
    return REF_SO.exists()


def reference() -> Reference:
    return Reference()
