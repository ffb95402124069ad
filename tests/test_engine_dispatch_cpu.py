"""The tensor engine's routing rule (select_backend,
runtime/tensor/tensor_engine.c:28-67) as the library states it
(tos_tensor_select_backend) against the reference's own function, run from
its hosted build: the same backend for every opcode, total size and GPU
count.  No GPU needed."""
import ctypes as C

import numpy as np
import pytest

from tensoros_b200 import _ffi


def test_select_backend_matches_reference():
    import pyoracle
    if not pyoracle.reference_available():
        pytest.skip("reference library not built here")
    R = pyoracle.reference()
    lib = _ffi.nn()
    rng = np.random.default_rng(3)
    edges = [0, 1, 4095, 4096, 4097, 32768, 32769, 65536, 65537, 1 << 20]
    for op in range(0, 30):
        for gpus in (0, 1, 8):
            for total in edges + list(rng.integers(0, 1 << 21, 20)):
                parts = [int(total) // 2, int(total) - int(total) // 2]
                descs = (_ffi.TensorDesc * 2)()
                for d, sz in zip(descs, parts):
                    d.size_bytes = sz
                got = lib.tos_tensor_select_backend(op, descs, 2, gpus)
                want = R.select_backend(op, parts, gpus)
                assert got == want, (op, gpus, total, got, want)


def test_tensor_desc_layout():
    """tos_tensor_desc_t has tensor_desc_t's layout (kernel/core/kernel.h:30-40)."""
    d = _ffi.TensorDesc
    assert C.sizeof(d) == 4 + 4 + 8 * 8 + 8 * 8 + 4 + 4 + 8 * 3 + 4 + 4
    assert d.shape.offset == 8 and d.dtype.offset == 136 and d.data_virt.offset == 152 and d.device_id.offset == 168
