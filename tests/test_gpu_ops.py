"""GPU operators through the C-ABI drop-ins, bit-exact against the golden
vectors the reference produced (tests/golden/ops.npz)."""
import numpy as np
import pytest

from conftest import bits_equal, first_diff
from tensoros_b200 import ops
from tensoros_b200 import workloads as W

pytestmark = pytest.mark.gpu


def test_block_dots(gpu, golden):
    for t, name in [(W.TYPE_Q4_0, "q4_0"), (W.TYPE_Q8_0, "q8_0")]:
        blocks, x, ref = golden[f"blocks_{name}"], golden[f"blocks_{name}_x"], golden[f"blocks_{name}_out"]
        bs = W.BLOCK_BYTES[t]
        fn = ops.q4_0_dot32 if t == W.TYPE_Q4_0 else ops.q8_0_dot32
        got = np.array([fn(blocks[bs * i:bs * i + bs], x[32 * i:32 * i + 32]) for i in range(len(ref))], np.float32)
        assert bits_equal(got, ref), (name, first_diff(got, ref))


def test_block_dots_device_batch(gpu, golden):
    import torch
    for t, name in [(W.TYPE_Q4_0, "q4_0"), (W.TYPE_Q8_0, "q8_0")]:
        blocks, x, ref = golden[f"blocks_{name}"], golden[f"blocks_{name}_x"], golden[f"blocks_{name}_out"]
        db = torch.from_numpy(blocks).cuda()
        dx = torch.from_numpy(x).cuda()
        out = torch.empty(len(ref), dtype=torch.float32, device="cuda")
        st = gpu.tos_block_dots_dev(db.data_ptr(), t, dx.data_ptr(), len(ref), out.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream)
        assert st == 0
        torch.cuda.synchronize()
        assert bits_equal(out.cpu().numpy(), ref), name


@pytest.mark.parametrize("tag", ["q4_0", "q8_0", "q4_0_wide", "q8_0_wide"])
def test_gemv_golden(gpu, golden, tag):
    r, c, t = (int(v) for v in golden[f"gemv_{tag}_shape"])
    got = ops.gemv(golden[f"gemv_{tag}_w"], golden[f"gemv_{tag}_x"], r, c, t)
    ref = golden[f"gemv_{tag}_out"]
    assert bits_equal(got, ref), first_diff(got, ref)


def test_gemv_float_rows(gpu, golden):
    got = ops.gemv(golden["gemv_f32_w"], golden["gemv_f32_x"], 11, 100, W.TYPE_F32)
    assert bits_equal(got, golden["gemv_f32_out"])
    got = ops.gemv(golden["gemv_f16_w"], golden["gemv_f16_x"], 13, 102, W.TYPE_F16)
    assert bits_equal(got, golden["gemv_f16_out"])


@pytest.mark.parametrize("dim", [288, 290, 4096])
def test_rmsnorm(gpu, golden, dim):
    got = ops.rmsnorm(golden[f"rmsnorm_{dim}_x"], golden[f"rmsnorm_{dim}_w"], dim)
    assert bits_equal(got, golden[f"rmsnorm_{dim}_out"])


@pytest.mark.parametrize("hd", [48, 128])
def test_rope(gpu, golden, hd):
    v = golden[f"rope_{hd}_v"]
    for p, ref in zip(golden[f"rope_{hd}_pos"], golden[f"rope_{hd}_out"]):
        got = ops.rope(v, int(p), hd, 10000.0)
        assert bits_equal(got, ref), (int(p), first_diff(got, ref))


def test_softmax_silu(gpu, golden):
    for n in (1, 7, 1000):
        assert bits_equal(ops.softmax(golden[f"softmax_{n}_x"]), golden[f"softmax_{n}_out"]), n
    assert bits_equal(ops.silu(golden["silu_x"]), golden["silu_out"])


def test_dot_axpy_vadd_vmul(gpu, golden):
    for n in (48, 128, 131):
        assert bits_equal([ops.dot_f32(golden[f"dot_{n}_a"], golden[f"dot_{n}_b"])], golden[f"dot_{n}_out"]), n
    a, b = golden["vec_a"], golden["vec_b"]
    assert bits_equal(ops.axpy_f32(a, np.float32(0.3710938), b), golden["axpy_out"])
    assert bits_equal(ops.vadd_f32(a, b), golden["vadd_out"])
    assert bits_equal(ops.vmul_f32(a, b), golden["vmul_out"])


def test_argmax(gpu, golden):
    for i in range(6):
        assert ops.argmax(golden[f"argmax_{i}_x"]) == int(golden[f"argmax_{i}_out"][0]), i


def test_embed(gpu, golden):
    for t, dim, tag in [(W.TYPE_Q4_0, 4096, "q4_0"), (W.TYPE_Q8_0, 288, "q8_0"),
                        (W.TYPE_F32, 64, "f32"), (W.TYPE_F16, 64, "f16")]:
        for tok in range(5):
            got = ops.embed(golden[f"embed_{tag}_w"], t, dim, tok)
            assert bits_equal(got, golden[f"embed_{tag}_out"][tok]), (tag, tok)


def test_q4f(gpu, golden):
    assert bits_equal(ops.q4_gemv(golden["q4f_w"], golden["q4f_x"], 8, 64), golden["q4f_gemv_out"])
    qb, qx = golden["q4f_w"], golden["q4f_x"]
    got = [ops.q4_dot_block(qb[20 * i:20 * i + 20], qx[:32]) for i in range(4)]
    assert bits_equal(got, golden["q4f_block_out"])


def test_unsupported_type_gives_zeros(gpu):
    """llm_vec_dot returns 0 for unknown types (llm.c:285-287)."""
    w = np.ones(4 * 64, np.uint8)
    out = ops.gemv(w, np.ones(64, np.float32), 4, 64, 6)   # GGML_TYPE_Q5_0
    assert np.all(out == 0)
    out = ops.gemv(w, np.ones(64, np.float32), 4, 16, W.TYPE_Q4_0)   # in_dim < 32: no blocks
    assert np.all(out == 0)


def test_empty_and_invalid(gpu):
    assert len(ops.softmax(np.zeros(0, np.float32))) == 0
    with pytest.raises(ops.TosError):
        ops.rope(np.zeros(5, np.float32), 0, 5, 10000.0)   # odd head_dim
