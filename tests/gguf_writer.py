"""A minimal GGUF writer for tests (the published GGUF v3 container layout:
magic, version, tensor and key-value counts, typed key-value pairs, tensor
infos with shapes innermost-first, padding to `general.alignment`, data).

`write_model` stores a synthetic model under the reference's WeightStore names
and GGUF shapes ([cols, rows], src/model_loader.rs:192-234) with the
`llama.*` metadata ModelMeta::from_gguf reads (:41-127)."""
import struct

import numpy as np

MAGIC = 0x46554747
T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 = range(13)
GGML_F32, GGML_F16, GGML_Q4_0 = 0, 1, 2
_FMT = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i", T_F32: "<f",
        T_BOOL: "<B", T_U64: "<Q", T_I64: "<q", T_F64: "<d"}


def _str(s):
    b = s.encode() if isinstance(s, str) else s
    return struct.pack("<Q", len(b)) + b


def _val(t, v):
    if t == T_STR:
        return _str(v)
    if t == T_ARR:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(_val(et, x) for x in items)
    return struct.pack(_FMT[t], v)


def header(kvs, tensors, version=3, magic=MAGIC):
    """kvs: [(key, type, value)]; tensors: [(name, shape, ggml_type, offset)]."""
    b = struct.pack("<IIQQ", magic, version, len(tensors), len(kvs))
    for k, t, v in kvs:
        b += _str(k) + struct.pack("<I", t) + _val(t, v)
    for name, shape, gt, off in tensors:
        b += _str(name) + struct.pack("<I", len(shape)) + b"".join(struct.pack("<Q", d) for d in shape)
        b += struct.pack("<IQ", gt, off)
    return b


def build(kvs, tensors, alignment=32, version=3):
    """tensors: [(name, shape, ggml_type, bytes)] -> file bytes, data offset."""
    infos, blob = [], b""
    for name, shape, gt, data in tensors:
        pad = (-len(blob)) % alignment
        blob += b"\0" * pad
        infos.append((name, shape, gt, len(blob)))
        blob += data
    h = header(kvs, infos, version)
    start = -(-len(h) // alignment) * alignment
    return h + b"\0" * (start - len(h)) + blob, start


def model_kvs(meta, n_ctx=2048, vocab_as_tokens=True):
    kv = [("general.architecture", T_STR, "llama"),
          ("llama.embedding_length", T_U32, meta["n_embd"]),
          ("llama.block_count", T_U32, meta["n_layer"]),
          ("llama.attention.head_count", T_U32, meta["n_head"]),
          ("llama.attention.head_count_kv", T_U32, meta["n_head_kv"]),
          ("llama.context_length", T_U32, n_ctx),
          ("llama.feed_forward_length", T_U32, meta["n_ff"]),
          ("llama.rope.freq_base", T_F32, meta["rope_freq_base"]),
          ("llama.attention.layer_norm_rms_epsilon", T_F32, meta["norm_eps"])]
    if vocab_as_tokens:
        kv.append(("tokenizer.ggml.tokens", T_ARR, (T_STR, [f"t{i}" for i in range(meta["n_vocab"])])))
    else:
        kv.append(("llama.vocab_size", T_U32, meta["n_vocab"]))
    return kv


def model_tensors(tensors):
    """{name: (velo dtype, array, rows, cols)} -> [(name, [cols, rows] or [cols], ggml type, bytes)]."""
    out = []
    for name, (dt, arr, rows, cols) in tensors.items():
        shape = [cols] if name.endswith("norm.weight") else [cols, rows]
        out.append((name, shape, {0: GGML_F32, 1: GGML_F16, 2: GGML_Q4_0}[dt],
                    np.ascontiguousarray(arr).tobytes()))
    return out


def write_model(path, meta, tensors, alignment=32, **kw):
    kvs = model_kvs(meta, **kw)
    if alignment != 32:
        kvs.append(("general.alignment", T_U32, alignment))
    data, start = build(kvs, model_tensors(tensors), alignment)
    with open(path, "wb") as f:
        f.write(data)
    return start
