"""ctypes declarations of the C-ABI in include/tensoros_nn_gpu.h and include/tos_synth.h.

The product is the shared library; this module only binds it.  Loading fails
loudly (ImportError) when the library has not been built: there is no Python
or CPU fallback for any operator.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

_LIB_DIR = Path(__file__).resolve().parent / "lib"
NN_PATH = _LIB_DIR / "libtensoros_nn.so"
SYNTH_PATH = _LIB_DIR / "libtos_synth.so"

vp = C.c_void_p
fp = C.POINTER(C.c_float)
ip = C.POINTER(C.c_int)
i32 = C.c_int
f32 = C.c_float
sz = C.c_size_t


class ModelDesc(C.Structure):
    """tos_model_desc_t"""
    _fields_ = [
        ("dim", i32), ("n_layers", i32), ("n_heads", i32), ("n_kv_heads", i32),
        ("ff_dim", i32), ("vocab_size", i32), ("max_seq", i32),
        ("rope_base", f32), ("norm_eps", f32),
        ("kv_type", i32), ("attn_mode", i32), ("wtype", i32), ("embd_type", i32), ("out_type", i32),
        ("token_embd", vp), ("output_weight", vp), ("output_norm", vp),
        ("attn_norm", C.POINTER(vp)), ("ffn_norm", C.POINTER(vp)),
        ("wq", C.POINTER(vp)), ("wk", C.POINTER(vp)), ("wv", C.POINTER(vp)), ("wo", C.POINTER(vp)),
        ("wgate", C.POINTER(vp)), ("wup", C.POINTER(vp)), ("wdown", C.POINTER(vp)),
        ("gemv_mode", i32), ("fused_step", i32),
    ]


class ShardPlan(C.Structure):
    """tos_shard_plan_t"""
    _fields_ = [(n, i32) for n in ("world", "rank", "head0", "n_heads", "kv_head0", "n_kv_heads", "q_row0",
                                   "n_q_rows", "kv_row0", "n_kv_rows", "row0", "n_rows", "ff0", "n_ff",
                                   "vocab0", "n_vocab")]


class TfDesc(C.Structure):
    """tos_tf_desc_t (the fp32 engine of runtime/nn/transformer.c)"""
    _fields_ = [(n, i32) for n in ("dim", "num_heads", "ff_dim", "num_layers", "vocab_size", "max_seq")] + \
               [(n, C.POINTER(vp)) for n in ("wq", "wk", "wv", "wo", "w1", "w2", "w3", "rms_att", "rms_ffn")] + \
               [("tok_embed", vp), ("rms_final", vp)]


class TensorDesc(C.Structure):
    """tos_tensor_desc_t (tensor_desc_t of kernel/core/kernel.h:30-40)"""
    _fields_ = [("ndim", C.c_uint32), ("shape", C.c_uint64 * 8), ("strides", C.c_uint64 * 8), ("dtype", C.c_int32),
                ("data_phys", C.c_uint64), ("data_virt", C.c_uint64), ("size_bytes", C.c_uint64),
                ("device_id", C.c_uint32), ("flags", C.c_uint32)]


# name -> (restype, argtypes)
NN_FUNCS = {
    "tos_status_string": (C.c_char_p, [i32]),
    "tos_last_status": (i32, []),
    "tos_init": (i32, [i32]),
    "tos_shutdown": (i32, []),
    "tos_device_count": (i32, []),
    "tos_synchronize": (i32, []),
    "tos_stream": (vp, []),
    "tos_weight_create": (i32, [C.POINTER(vp), vp, i32, i32, i32]),
    "tos_weight_create_dev": (i32, [C.POINTER(vp), vp, i32, i32, i32, vp]),
    "tos_weight_destroy": (None, [vp]),
    "tos_weight_device_bytes": (sz, [vp]),
    "tos_weight_cache_clear": (None, []),
    "tos_gemv_dev": (i32, [vp, vp, vp, vp]),
    "tos_gemv_norm_dev": (i32, [vp, vp, vp, f32, vp, vp]),
    "tos_gemv_mode_dev": (i32, [vp, vp, vp, f32, vp, i32, vp]),
    "tos_block_dots_dev": (i32, [vp, i32, vp, i32, vp, vp]),
    "tos_rmsnorm_dev": (i32, [vp, vp, vp, i32, i32, f32, vp]),
    "tos_rope_dev": (i32, [vp, i32, i32, i32, f32, vp]),
    "tos_softmax_dev": (i32, [vp, i32, vp]),
    "tos_silu_dev": (i32, [vp, i32, vp]),
    "tos_vadd_dev": (i32, [vp, vp, i32, vp]),
    "tos_vmul_dev": (i32, [vp, vp, i32, vp]),
    "tos_axpy_dev": (i32, [vp, f32, vp, i32, vp]),
    "tos_dot_dev": (i32, [vp, vp, i32, vp, vp]),
    "tos_embed_dev": (i32, [vp, vp, i32, i32, i32, vp]),
    "tos_argmax_dev": (i32, [vp, i32, vp, vp]),
    "tos_attention_workspace_bytes": (sz, [i32, i32]),
    "tos_attention_dev": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, vp, sz, vp]),
    "tos_attention_noalloc_dev": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, vp]),
    "tos_gemv": (None, [vp, vp, vp, i32, i32, i32]),
    "tos_vec_dot": (f32, [vp, vp, i32, i32]),
    "tos_q4_0_dot32": (f32, [vp, vp]),
    "tos_q8_0_dot32": (f32, [vp, vp]),
    "tos_embed": (None, [vp, vp, i32, i32, i32]),
    "tos_rmsnorm": (None, [vp, vp, vp, i32, i32]),
    "tos_rope": (None, [vp, i32, i32, f32]),
    "tos_softmax": (None, [vp, i32]),
    "tos_silu": (None, [vp, i32]),
    "tos_dot_f32": (f32, [vp, vp, i32]),
    "tos_axpy_f32": (None, [vp, f32, vp, i32]),
    "tos_vadd_f32": (None, [vp, vp, i32]),
    "tos_vmul_f32": (None, [vp, vp, i32]),
    "tos_argmax": (i32, [vp, i32]),
    "tos_q4_dot_block": (f32, [vp, vp]),
    "tos_q4_gemv": (None, [vp, vp, vp, i32, i32]),
    "tos_model_create": (i32, [C.POINTER(vp), C.POINTER(ModelDesc)]),
    "tos_model_destroy": (None, [vp]),
    "tos_model_reset": (i32, [vp]),
    "tos_model_forward_token": (i32, [vp, vp, i32, i32]),
    "tos_model_forward_argmax": (i32, [vp, i32, i32, ip]),
    "tos_model_generate_greedy": (i32, [vp, vp, i32, i32, vp]),
    "tos_model_decode": (i32, [vp, i32, i32, i32, vp]),
    "tos_model_prefill": (i32, [vp, vp, i32, i32, vp, ip]),
    "tos_model_decode_batch": (i32, [vp, vp, vp, vp, i32, vp, vp]),
    "tos_model_stream": (vp, [vp]),
    "tos_model_logits_dev": (vp, [vp]),
    "tos_model_device_bytes": (sz, [vp]),
    "tos_gguf_open": (i32, [C.POINTER(vp), vp, C.c_uint64]),
    "tos_gguf_open_file": (i32, [C.POINTER(vp), C.c_char_p]),
    "tos_gguf_close": (None, [vp]),
    "tos_gguf_version": (C.c_uint32, [vp]),
    "tos_gguf_n_tensors": (C.c_int64, [vp]),
    "tos_gguf_n_kv": (C.c_int64, [vp]),
    "tos_gguf_find_tensor": (C.c_int64, [vp, C.c_char_p]),
    "tos_gguf_tensor_info": (i32, [vp, C.c_int64, C.POINTER(C.c_char_p), ip, ip, C.POINTER(C.c_uint64),
                                   C.POINTER(vp), C.POINTER(C.c_uint64)]),
    "tos_gguf_get_u32": (i32, [vp, C.c_char_p, C.POINTER(C.c_uint32)]),
    "tos_gguf_get_f32": (i32, [vp, C.c_char_p, C.POINTER(C.c_float)]),
    "tos_gguf_get_str": (i32, [vp, C.c_char_p, C.POINTER(C.c_char_p), C.POINTER(C.c_uint64)]),
    "tos_gguf_model_desc": (i32, [vp, vp]),
    "tos_sample": (i32, [vp, i32, f32, C.c_uint32]),
    "tos_sample_dev": (i32, [vp, i32, f32, C.c_uint32, vp, vp]),
    "tos_model_fused": (i32, [vp]),
    "tos_shard_range": (i32, [i32, i32, i32, i32, ip, ip]),
    "tos_shard_plan": (i32, [C.POINTER(ModelDesc), i32, i32, C.POINTER(ShardPlan)]),
    "tos_nccl_unique_id": (i32, [vp, sz]),
    "tos_model_create_sharded": (i32, [C.POINTER(vp), C.POINTER(ModelDesc), i32, i32, vp]),
    "tos_argmax_sharded_dev": (i32, [vp, i32, i32, vp, vp]),
    "tos_gemm_workspace_bytes": (sz, [i32, i32, i32]),
    "tos_gemm_dev": (i32, [vp, vp, i32, vp, vp, sz, vp]),
    "tos_tf_rmsnorm": (None, [vp, vp, vp, i32]),
    "tos_tf_swiglu_ffn": (None, [vp, vp, vp, vp, vp, i32, i32]),
    "tos_tf_model_create": (i32, [C.POINTER(vp), C.POINTER(TfDesc)]),
    "tos_tf_model_destroy": (None, [vp]),
    "tos_tf_reset": (i32, [vp]),
    "tos_tf_cached_attention": (i32, [vp, vp, vp, vp, vp, i32, i32, i32]),
    "tos_tf_forward_token": (i32, [vp, vp, vp, i32]),
    "tos_tensor_select_backend": (i32, [i32, vp, C.c_uint32, C.c_uint32]),
    "tos_gpu_tensor_matmul": (i32, [C.c_uint32, vp, vp, vp]),
    "tos_gpu_tensor_attention": (i32, [C.c_uint32, vp, vp, vp, vp, f32]),
    "tos_gpu_tensor_softmax": (i32, [C.c_uint32, vp, vp, i32]),
    "tos_gpu_tensor_layernorm": (i32, [C.c_uint32, vp, vp, vp, vp, f32]),
    "tos_gpu_tensor_elementwise": (i32, [C.c_uint32, vp, vp, vp, i32]),
}

SYNTH_FUNCS = {
    "tos_synth_u64": (C.c_uint64, [C.c_uint64, C.c_uint64, C.c_uint64]),
    "tos_synth_f32_to_f16": (C.c_uint16, [f32]),
    "tos_synth_normal_f32": (None, [vp, sz, C.c_uint64, C.c_uint64, f32, f32, i32]),
    "tos_synth_normal_f16": (None, [vp, sz, C.c_uint64, C.c_uint64, f32, f32, i32]),
    "tos_synth_q4_0": (None, [vp, sz, C.c_uint64, C.c_uint64, f32, i32]),
    "tos_synth_q8_0": (None, [vp, sz, C.c_uint64, C.c_uint64, f32, i32]),
    "tos_synth_q4f": (None, [vp, sz, C.c_uint64, C.c_uint64, f32, i32]),
    "tos_synth_tokens": (None, [vp, sz, C.c_int32, C.c_uint64, C.c_uint64]),
}


def _bind(path: Path, funcs: dict) -> C.CDLL:
    if not path.exists():
        raise ImportError(f"{path.name} is not built (run tensoros_b200._build or __graft_entry__.build())")
    lib = C.CDLL(str(path))
    for name, (res, args) in funcs.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    return lib


_nn = None
_synth = None


def nn() -> C.CDLL:
    global _nn
    if _nn is None:
        _nn = _bind(NN_PATH, NN_FUNCS)
    return _nn


def synth() -> C.CDLL:
    global _synth
    if _synth is None:
        _synth = _bind(SYNTH_PATH, SYNTH_FUNCS)
    return _synth
