"""A model created from a GGUF file (tos_gguf_model_desc, tensors used in
place) decodes exactly as the model created from the same tensors directly:
bitwise-equal logits in EXACT arithmetic, equal to the oracle's."""
import ctypes as C

import numpy as np
import pytest

from gguf_writer import gguf_bytes
from tensoros_b200 import _ffi, ops
from tensoros_b200 import workloads as W

pytestmark = pytest.mark.gpu


def test_gguf_model_matches_direct(gpu, oracle):
    synth = W.make_model(dict(W.SHARD_SMALL, n_layers=2), 9)
    blob = gguf_bytes(synth, tied=True)
    buf = C.create_string_buffer(blob, len(blob))
    lib = _ffi.nn()
    g = C.c_void_p()
    assert lib.tos_gguf_open(C.byref(g), buf, len(blob)) == 0
    try:
        d = _ffi.ModelDesc()
        assert lib.tos_gguf_model_desc(g, C.byref(d)) == 0
        d.kv_type = W.TYPE_F32
        d.max_seq = 64
        h = C.c_void_p()
        assert lib.tos_model_create(C.byref(h), C.byref(d)) == 0
        try:
            # the direct model with the same (tied) output
            synth.output = None
            synth.cfg = dict(synth.cfg, out_type=synth.cfg["embd_type"])
            direct = ops.Model(synth)
            ref = oracle.model(synth)
            try:
                for pos, tok in enumerate(W.tokens(5, synth.cfg["vocab_size"], 9)):
                    a = np.empty(synth.cfg["vocab_size"], np.float32)
                    assert lib.tos_model_forward_token(h, a.ctypes.data, int(tok), pos) == 0
                    b = direct.forward(int(tok), pos)
                    r = ref.forward(int(tok), pos)
                    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
                    assert np.array_equal(a.view(np.uint32), r.view(np.uint32))
            finally:
                direct.close()
                ref.close()
        finally:
            lib.tos_model_destroy(h)
    finally:
        lib.tos_gguf_close(g)
