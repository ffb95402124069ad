"""tos_attention_noalloc_dev: the allocation-free attention entry point.

It exists for callers that cannot allocate device memory while they run a
decode step (the reference's static-scratch loop allocates nothing either):
its workspace is a fixed 4 MiB device array inside the library.  These checks
call it through the C-ABI and compare it with tos_attention_dev, which takes a
caller-allocated workspace, on two calls in a row (the shared array keeps the
previous call's contents, which must not leak into the next result).  This
file is collected last on purpose.
"""
import pytest

from conftest import bits_equal, first_diff
from tensoros_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _inputs(nh, nkv, hd, ctx, kv_type, seed):
    q = W.normal_f32(nh * hd, seed, 1)
    if kv_type == W.TYPE_F16:
        kc = W.normal_f16(ctx * nkv * hd, seed, 2)
        vc = W.normal_f16(ctx * nkv * hd, seed, 3)
    else:
        kc = W.normal_f32(ctx * nkv * hd, seed, 2)
        vc = W.normal_f32(ctx * nkv * hd, seed, 3)
    return q, kc, vc


def _run_both(gpu, torch, q, kc, vc, kv_type, nh, nkv, hd, pos, max_ctx, mode):
    dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, kc, vc))
    ref = torch.empty(nh * hd, device="cuda")
    got = torch.full((nh * hd,), float("nan"), device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    wsb = gpu.tos_attention_workspace_bytes(nh, max_ctx)
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    assert gpu.tos_attention_dev(ref.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), kv_type, nh, nkv,
                                 hd, pos, max_ctx, mode, ws.data_ptr(), wsb, stream) == 0
    torch.cuda.synchronize()
    st = gpu.tos_attention_noalloc_dev(got.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), kv_type, nh,
                                       nkv, hd, pos, max_ctx, mode, stream)
    assert st == 0, st
    torch.cuda.synchronize()
    return got.cpu().numpy(), ref.cpu().numpy()


@pytest.mark.parametrize("mode", [0, 1])
def test_noalloc_matches_allocating_entry_point(gpu, mode):
    import torch
    # two calls in a row with different shapes and contents: the second must
    # not see anything the first left in the shared array
    cases = [(32, 32, 128, 2048, W.TYPE_F16, 2047, 31), (8, 2, 64, 700, W.TYPE_F32, 345, 32)]
    for nh, nkv, hd, ctx, kv, pos, seed in cases:
        q, kc, vc = _inputs(nh, nkv, hd, ctx, kv, seed)
        got, ref = _run_both(gpu, torch, q, kc, vc, kv, nh, nkv, hd, pos, ctx, mode)
        # both entry points run the same deterministic kernels (FAST included:
        # fixed summation orders), so any difference is workspace leaking
        # from the previous call: the comparison is bitwise in both modes
        assert bits_equal(got, ref), (mode, first_diff(got, ref))


def test_noalloc_rejects_oversized_workspace(gpu):
    import torch
    nh, hd, ctx = 64, 128, 32768          # workspace well above the 4 MiB array
    assert gpu.tos_attention_workspace_bytes(nh, ctx) > (4 << 20)
    d = torch.zeros(16, device="cuda")
    st = gpu.tos_attention_noalloc_dev(d.data_ptr(), d.data_ptr(), d.data_ptr(), d.data_ptr(), W.TYPE_F16, nh, nh,
                                       hd, 0, ctx, 0, torch.cuda.current_stream().cuda_stream)
    assert st == -2          # TOS_ENOMEM, nothing queued
