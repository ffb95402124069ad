"""B200 (sm_100a) drop-in for TensorOS runtime/nn's GGUF decode path.

The product is the C-ABI library libtensoros_nn.so (include/tensoros_nn_gpu.h):
hand-written sm_100a kernels behind a C11 host runtime.  This package builds
it in-tree (`_build`), binds it (`_ffi`), mirrors the reference operators
for host numpy buffers (`ops`), and generates seeded workloads (`workloads`).
"""
from . import _ffi  # noqa: F401

TYPE_F32, TYPE_F16, TYPE_Q4_0, TYPE_Q8_0 = 0, 1, 2, 8
ATTN_EXACT, ATTN_FAST = 0, 1

TOS_OK, TOS_EINVAL, TOS_ENOMEM, TOS_ECUDA, TOS_ENCCL, TOS_ETIMEOUT, TOS_ENOTSUP, TOS_ENODEV = (
    0, -1, -2, -3, -4, -5, -6, -7)


def lib():
    """The bound libtensoros_nn.so (raises ImportError if it is not built)."""
    return _ffi.nn()
