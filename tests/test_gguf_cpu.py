"""GGUF container reader and the llama tensor mapping (tos_gguf_*; the
reference's runtime/nn/gguf.c:204-423 and llm.c:1374-1448, 1521-1545), on
files written by tests/gguf_writer.py: metadata and tensor infos read back
exactly, tensor data used in place, the model descriptor filled as the
reference maps it, malformed files rejected.  No GPU needed."""
import ctypes as C

import numpy as np
import pytest

from gguf_writer import gguf_bytes
from tensoros_b200 import _ffi
from tensoros_b200 import workloads as W

EINVAL, ENOTSUP = -1, -6


@pytest.fixture(scope="module")
def lib(built):
    return _ffi.nn()


def open_bytes(lib, blob):
    buf = C.create_string_buffer(blob, len(blob))
    h = C.c_void_p()
    st = lib.tos_gguf_open(C.byref(h), buf, len(blob))
    return st, h, buf


def small():
    return W.make_model(dict(W.SHARD_SMALL, n_layers=2), 7)


def test_gguf_metadata_and_tensors(lib):
    synth = small()
    blob = gguf_bytes(synth)
    st, h, buf = open_bytes(lib, blob)
    assert st == 0
    try:
        assert lib.tos_gguf_version(h) == 3
        assert lib.tos_gguf_n_tensors(h) == 3 + 9 * 2
        assert lib.tos_gguf_n_kv(h) == 11
        v = C.c_uint32()
        assert lib.tos_gguf_get_u32(h, b"llama.embedding_length", C.byref(v)) == 0 and v.value == 256
        f = C.c_float()
        assert lib.tos_gguf_get_f32(h, b"llama.rope.freq_base", C.byref(f)) == 0 and f.value == 10000.0
        assert lib.tos_gguf_get_u32(h, b"llama.rope.freq_base", C.byref(v)) == EINVAL   # not an integer
        assert lib.tos_gguf_get_u32(h, b"no.such.key", C.byref(v)) == EINVAL
        s, n = C.c_char_p(), C.c_uint64()
        assert lib.tos_gguf_get_str(h, b"general.name", C.byref(s), C.byref(n)) == 0
        assert C.string_at(s, n.value).decode() == synth.cfg["name"]
        i = lib.tos_gguf_find_tensor(h, b"blk.1.ffn_down.weight")
        assert i >= 0 and lib.tos_gguf_find_tensor(h, b"blk.9.ffn_down.weight") == -1
        name, t, nd = C.c_char_p(), C.c_int(), C.c_int()
        dims, data, nbytes = (C.c_uint64 * 4)(), C.c_void_p(), C.c_uint64()
        assert lib.tos_gguf_tensor_info(h, i, C.byref(name), C.byref(t), C.byref(nd), dims, C.byref(data),
                                        C.byref(nbytes)) == 0
        assert name.value == b"blk.1.ffn_down.weight" and t.value == W.TYPE_Q8_0 and nd.value == 2
        assert list(dims) == [512, 256, 1, 1]
        src = bytes(synth.layers[1]["wdown"])
        assert nbytes.value == len(src) and C.string_at(data, len(src)) == src
        # in place: the pointer lies inside the caller's buffer
        assert C.addressof(buf) <= data.value < C.addressof(buf) + len(blob)
    finally:
        lib.tos_gguf_close(h)


def read_desc(lib, h):
    d = _ffi.ModelDesc()
    st = lib.tos_gguf_model_desc(h, C.byref(d))
    return st, d


@pytest.mark.parametrize("tied,alignment,norm_f16", [(False, None, False), (True, 64, False), (False, 128, True)])
def test_gguf_model_desc(lib, tied, alignment, norm_f16):
    synth = small()
    c = synth.cfg
    blob = gguf_bytes(synth, alignment=alignment, tied=tied, norm_f16=norm_f16)
    st, h, buf = open_bytes(lib, blob)
    assert st == 0
    try:
        st, d = read_desc(lib, h)
        assert st == 0
        for k in ("dim", "n_layers", "n_heads", "n_kv_heads", "ff_dim", "vocab_size", "max_seq"):
            assert getattr(d, k) == c[k], k
        assert d.rope_base == c["rope_base"] and abs(d.norm_eps - c["norm_eps"]) < 1e-12
        assert d.wtype == c["wtype"] and d.embd_type == c["embd_type"]
        if tied:
            assert not d.output_weight and d.out_type == c["embd_type"]
        else:
            assert C.string_at(d.output_weight, len(bytes(synth.output))) == bytes(synth.output)
        assert C.string_at(d.token_embd, 64) == bytes(synth.token_embd)[:64]
        if alignment:
            assert d.token_embd % alignment == C.addressof(buf) % alignment
        for l in range(c["n_layers"]):
            q = bytes(synth.layers[l]["wq"])
            assert C.string_at(d.wq[l], len(q)) == q
            g = np.ctypeslib.as_array(C.cast(d.attn_norm[l], C.POINTER(C.c_float)), (c["dim"],))
            want = np.asarray(synth.layers[l]["attn_norm"], np.float32)
            if norm_f16:
                want = want.astype(np.float16).astype(np.float32)
            assert np.array_equal(g, want)
    finally:
        lib.tos_gguf_close(h)


def test_gguf_rejects_malformed(lib):
    blob = gguf_bytes(small())
    assert open_bytes(lib, b"GGUX" + blob[4:])[0] == EINVAL
    assert open_bytes(lib, blob[:4] + (4).to_bytes(4, "little") + blob[8:])[0] == ENOTSUP
    huge = blob[:8] + (1 << 60).to_bytes(8, "little") + blob[16:]
    assert open_bytes(lib, huge)[0] == EINVAL
    for cut in (20, 100, 700, len(blob) // 2, len(blob) - 1):
        assert open_bytes(lib, blob[:cut])[0] == EINVAL, cut
    # a file without the llama keys parses but does not describe a model
    st, h, buf = open_bytes(lib, gguf_bytes(small())[:24] + b"")
    assert st == EINVAL


def _desc_status(lib, blob):
    st, h, buf = open_bytes(lib, blob)
    if st != 0:
        return st
    try:
        return read_desc(lib, h)[0]
    finally:
        lib.tos_gguf_close(h)


def test_gguf_desc_rejects_tensors_smaller_than_the_model(lib):
    """Every tensor the model maps must have the shape the descriptor
    implies: a file whose tensors are smaller than its header says passes the
    container's range check, and the model upload would then read past them."""
    synth = small()
    c = synth.cfg
    dim, ff = c["dim"], c["ff_dim"]
    wt = c["wtype"]
    rb = (dim // 32) * (18 if wt == W.TYPE_Q4_0 else 34)
    norm = np.asarray(synth.layers[0]["attn_norm"], np.float32)
    assert _desc_status(lib, gguf_bytes(synth)) == 0
    cases = {
        # a norm 32 elements short
        "short attn_norm": {"blk.0.attn_norm.weight": ([dim - 32], 0, norm[:dim - 32].tobytes())},
        # q with one row fewer than n_heads * head_dim
        "short attn_q": {"blk.1.attn_q.weight": ([dim, dim - 1], wt, bytes(synth.layers[1]["wq"])[:rb * (dim - 1)])},
        # down with the input and output dimensions swapped
        "swapped ffn_down": {"blk.0.ffn_down.weight": ([dim, ff], wt, bytes(synth.layers[0]["wdown"]))},
        # a third dimension
        "3-d output": {"output.weight": ([dim, c["vocab_size"] // 2, 2], c["out_type"], bytes(synth.output))},
    }
    for what, ov in cases.items():
        assert _desc_status(lib, gguf_bytes(synth, override=ov)) == EINVAL, what
    # a well-formed norm of a quantised type: valid but not supported
    ov = {"output_norm.weight": ([dim], W.TYPE_Q8_0, b"\0" * ((dim // 32) * 34))}
    assert _desc_status(lib, gguf_bytes(synth, override=ov)) == ENOTSUP
    # a vocab_size key larger than the embedding's row count
    big = [("llama.vocab_size", 4, c["vocab_size"] + 32)]
    assert _desc_status(lib, gguf_bytes(synth, extra_kv=big)) == EINVAL
    ok = [("llama.vocab_size", 4, c["vocab_size"])]
    assert _desc_status(lib, gguf_bytes(synth, extra_kv=ok)) == 0


def test_gguf_rejects_wrapping_byte_size(lib):
    """An F32 tensor whose element count fits in 64 bits but whose byte size
    does not: its size must not wrap to a small value that passes the range
    check."""
    synth = small()
    n = (1 << 62) + 1                      # 4 * n wraps past 2^64
    ov = {"output_norm.weight": ([n], 0, b"\0" * 4)}
    st = _desc_status(lib, gguf_bytes(synth, override=ov))
    assert st == EINVAL


def test_gguf_file_mapping(lib, tmp_path):
    synth = small()
    p = tmp_path / "m.gguf"
    p.write_bytes(gguf_bytes(synth))
    h = C.c_void_p()
    assert lib.tos_gguf_open_file(C.byref(h), str(p).encode()) == 0
    try:
        st, d = read_desc(lib, h)
        assert st == 0 and d.dim == 256
        assert C.string_at(d.wdown[0], 34) == bytes(synth.layers[0]["wdown"])[:34]
    finally:
        lib.tos_gguf_close(h)
    assert lib.tos_gguf_open_file(C.byref(h), str(tmp_path / "missing.gguf").encode()) == EINVAL
