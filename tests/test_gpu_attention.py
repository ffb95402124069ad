"""Single-query decode attention (llm.c:683-714) on the GPU against the
oracle.  EXACT mode is bit-exact; FAST mode (split positions) is within a
normwise relative error of 1e-4."""
import numpy as np
import pytest

from conftest import assert_fast, attention_abs_scale, bits_equal, first_diff
from tensoros_b200 import workloads as W

pytestmark = pytest.mark.gpu
TOL = 1e-4   # FAST-mode bound: max|gpu - ref| / max|ref|


def make_case(oracle, n_heads, n_kv, hd, ctx, kv_type, seed=11, base=10000.0):
    """q roped at pos = ctx-1; cached k roped at its own position, then stored
    as fp16 (kv_type 1) or fp32; v ~ N(0,1)."""
    pos = ctx - 1
    q = oracle.rope_rows(W.normal_f32(n_heads * hd, seed, 1).reshape(1, -1), hd, [pos], base).ravel()
    k_raw = W.normal_f32(ctx * n_kv * hd, seed, 2).reshape(ctx, n_kv * hd)
    k = oracle.rope_rows(k_raw, hd, np.arange(ctx), base)
    if kv_type == W.TYPE_F16:
        kc = k.astype(np.float16).view(np.uint16)
        vc = W.normal_f16(ctx * n_kv * hd, seed, 3)
    else:
        kc = k.astype(np.float32)
        vc = W.normal_f32(ctx * n_kv * hd, seed, 3)
    return q, kc, vc, pos


def run_gpu(gpu, q, kc, vc, kv_type, n_heads, n_kv, hd, pos, max_ctx, mode):
    import torch
    dq = torch.from_numpy(q).cuda()
    dk = torch.from_numpy(np.ascontiguousarray(kc)).cuda()
    dv = torch.from_numpy(np.ascontiguousarray(vc)).cuda()
    out = torch.empty(n_heads * hd, device="cuda")
    wsb = gpu.tos_attention_workspace_bytes(n_heads, max_ctx)
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    st = gpu.tos_attention_dev(out.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), kv_type, n_heads,
                               n_kv, hd, pos, max_ctx, mode, ws.data_ptr(), wsb,
                               torch.cuda.current_stream().cuda_stream)
    assert st == 0
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("ctx", [512, 2048, 4096])
def test_attention_benchmark_config(gpu, oracle, ctx):
    nh, nkv, hd = 32, 32, 128
    q, kc, vc, pos = make_case(oracle, nh, nkv, hd, ctx, W.TYPE_F16)
    ref = oracle.attention(q, kc, vc, W.TYPE_F16, nh, nkv, hd, pos)
    got = run_gpu(gpu, q, kc, vc, W.TYPE_F16, nh, nkv, hd, pos, ctx, 0)
    assert bits_equal(got, ref), first_diff(got, ref)
    fast = run_gpu(gpu, q, kc, vc, W.TYPE_F16, nh, nkv, hd, pos, ctx, 1)
    assert_fast(fast, ref, TOL, ("attention", ctx),
                attention_abs_scale(q, kc, vc, W.TYPE_F16, nh, nkv, hd, pos))


@pytest.mark.parametrize("nh,nkv,hd,ctx,kv", [(8, 2, 64, 300, 0), (6, 6, 48, 272, 0), (4, 1, 128, 1, 1),
                                              (16, 4, 128, 777, 1)])
def test_attention_shapes(gpu, oracle, nh, nkv, hd, ctx, kv):
    """GQA groups, head_dim 48, a single position, fp32 and fp16 caches; the
    cache is allocated for more positions than are attended."""
    q, kc, vc, pos = make_case(oracle, nh, nkv, hd, ctx, kv, seed=ctx)
    ref = oracle.attention(q, kc, vc, kv, nh, nkv, hd, pos)
    got = run_gpu(gpu, q, kc, vc, kv, nh, nkv, hd, pos, ctx, 0)
    assert bits_equal(got, ref), first_diff(got, ref)
    fast = run_gpu(gpu, q, kc, vc, kv, nh, nkv, hd, pos, ctx, 1)
    assert_fast(fast, ref, TOL, ("attention", nh, nkv, hd, ctx, kv),
                attention_abs_scale(q, kc, vc, kv, nh, nkv, hd, pos))


def test_attention_prefix_of_cache(gpu, oracle):
    """pos < max_ctx - 1: only t <= pos is read (llm.c:692 loop bound)."""
    nh, nkv, hd, ctx = 4, 4, 64, 200
    q, kc, vc, _ = make_case(oracle, nh, nkv, hd, ctx, W.TYPE_F32, seed=5)
    pos = 57
    ref = oracle.attention(q, kc, vc, W.TYPE_F32, nh, nkv, hd, pos)
    got = run_gpu(gpu, q, kc, vc, W.TYPE_F32, nh, nkv, hd, pos, ctx, 0)
    assert bits_equal(got, ref)
