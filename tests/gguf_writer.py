"""Writes GGUF v3 files (the container runtime/nn/gguf.c parses) from a
workloads.SynthModel, for the loader tests: llama metadata keys, a string
array (as tokenizers carry), and the tensors under the names llm.c maps
(token_embd.weight, output_norm.weight, output.weight, blk.N.*)."""
import struct

import numpy as np

GT_U32, GT_F32, GT_STRING, GT_ARRAY = 4, 6, 8, 9


def _s(b: bytes) -> bytes:
    return struct.pack("<Q", len(b)) + b


def _kv(key, t, val):
    out = _s(key.encode()) + struct.pack("<I", t)
    if t == GT_U32:
        out += struct.pack("<I", val)
    elif t == GT_F32:
        out += struct.pack("<f", val)
    elif t == GT_STRING:
        out += _s(val.encode())
    elif t == GT_ARRAY:
        et, items = val
        out += struct.pack("<IQ", et, len(items))
        for it in items:
            out += _s(it.encode()) if et == GT_STRING else struct.pack("<I", it)
    return out


def gguf_bytes(synth, alignment=None, tied=False, extra_kv=(), norm_f16=False, version=3, override=None):
    """override: {tensor name: (dims, type, bytes)} replaces those tensors'
    infos and data (malformed-file tests)."""
    c = synth.cfg
    dim, ff, L = c["dim"], c["ff_dim"], c["n_layers"]
    hd = dim // c["n_heads"]
    qd, kvd = c["n_heads"] * hd, c["n_kv_heads"] * hd
    kvs = [("general.architecture", GT_STRING, "llama"), ("general.name", GT_STRING, c["name"]),
           ("llama.embedding_length", GT_U32, dim), ("llama.block_count", GT_U32, L),
           ("llama.attention.head_count", GT_U32, c["n_heads"]),
           ("llama.attention.head_count_kv", GT_U32, c["n_kv_heads"]),
           ("llama.feed_forward_length", GT_U32, ff), ("llama.context_length", GT_U32, c["max_seq"]),
           ("llama.rope.freq_base", GT_F32, c["rope_base"]),
           ("llama.attention.layer_norm_rms_epsilon", GT_F32, c["norm_eps"]),
           ("tokenizer.ggml.tokens", GT_ARRAY, (GT_STRING, ["<unk>", "<s>", "</s>", "a", "b"]))]
    if alignment:
        kvs.append(("general.alignment", GT_U32, alignment))
    kvs += list(extra_kv)
    wt = c["wtype"]
    norm_t = 1 if norm_f16 else 0

    def norm(a):
        return np.asarray(a, np.float16 if norm_f16 else np.float32).tobytes()

    tensors = [("token_embd.weight", [dim, c["vocab_size"]], c["embd_type"], bytes(synth.token_embd)),
               ("output_norm.weight", [dim], 0, np.asarray(synth.output_norm, np.float32).tobytes())]
    if not tied:
        tensors.append(("output.weight", [dim, c["vocab_size"]], c["out_type"], bytes(synth.output)))
    for l, ly in enumerate(synth.layers):
        tensors += [(f"blk.{l}.attn_norm.weight", [dim], norm_t, norm(ly["attn_norm"])),
                    (f"blk.{l}.attn_q.weight", [dim, qd], wt, bytes(ly["wq"])),
                    (f"blk.{l}.attn_k.weight", [dim, kvd], wt, bytes(ly["wk"])),
                    (f"blk.{l}.attn_v.weight", [dim, kvd], wt, bytes(ly["wv"])),
                    (f"blk.{l}.attn_output.weight", [qd, dim], wt, bytes(ly["wo"])),
                    (f"blk.{l}.ffn_norm.weight", [dim], norm_t, norm(ly["ffn_norm"])),
                    (f"blk.{l}.ffn_gate.weight", [dim, ff], wt, bytes(ly["wgate"])),
                    (f"blk.{l}.ffn_up.weight", [dim, ff], wt, bytes(ly["wup"])),
                    (f"blk.{l}.ffn_down.weight", [ff, dim], wt, bytes(ly["wdown"]))]
    if override:
        tensors = [(n, *override[n]) if n in override else (n, dm, t, b) for n, dm, t, b in tensors]
    align = alignment or 32
    head = struct.pack("<IIQQ", 0x46554747, version, len(tensors), len(kvs))
    head += b"".join(_kv(k, t, v) for k, t, v in kvs)
    infos, blobs, off = b"", [], 0
    for name, dims, t, blob in tensors:
        infos += _s(name.encode()) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        infos += struct.pack("<IQ", t, off)
        pad = (-len(blob)) % align
        blobs.append(blob + b"\0" * pad)
        off += len(blob) + pad
    meta = head + infos
    meta += b"\0" * ((-len(meta)) % align)
    return meta + b"".join(blobs)
