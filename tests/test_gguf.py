"""GGUF loading on the host (velo_gguf_*, no GPU): the reference's own
container and loader tests re-expressed (src/gguf.rs tests, src/model_loader.rs
tests), and a synthetic model written as GGUF whose metadata and tensor bytes
come back unchanged, ready for velo_cuda_load_model."""
import struct

import numpy as np
import pytest

import gguf_writer as gw
import synthetic
import velo_cuda


def _open(tmp_path, data, name="m.gguf"):
    p = tmp_path / name
    p.write_bytes(data)
    return velo_cuda.Gguf(p)


def _err(tmp_path, data):
    with pytest.raises(velo_cuda.VeloError) as e:
        _open(tmp_path, data)
    return e.value


def test_parses_empty_v3_file(tmp_path):
    g = _open(tmp_path, gw.header([], []))
    assert (g.version, g.n_metadata, g.n_tensors) == (3, 0, 0)


@pytest.mark.parametrize("version", [1, 2, 3])
def test_accepts_versions_1_to_3(tmp_path, version):
    assert _open(tmp_path, gw.header([], [], version=version)).version == version


def test_rejects_bad_magic_and_versions(tmp_path):
    e = _err(tmp_path, gw.header([], [], magic=0x12345678))
    assert e.status == velo_cuda.ERR_GGUF and "bad magic" in e.message
    for v in (0, 4, 99):
        e = _err(tmp_path, gw.header([], [], version=v))
        assert e.status == velo_cuda.ERR_GGUF and f"unsupported GGUF version {v}" in e.message


def test_parses_all_metadata_types(tmp_path):
    kvs = [("v_u8", gw.T_U8, 42), ("v_i8", gw.T_I8, -42), ("v_u16", gw.T_U16, 42), ("v_i16", gw.T_I16, -42),
           ("v_u32", gw.T_U32, 42), ("v_i32", gw.T_I32, -42), ("v_f32", gw.T_F32, 4.2),
           ("v_bool", gw.T_BOOL, 1), ("v_str", gw.T_STR, "hello"), ("v_u64", gw.T_U64, 42),
           ("v_i64", gw.T_I64, -42), ("v_f64", gw.T_F64, 4.2),
           ("v_arr", gw.T_ARR, (gw.T_STR, ["hello", "world"]))]
    g = _open(tmp_path, gw.header(kvs, []))
    assert g.n_metadata == 13
    got = {k: g.metadata(k) for k, _, _ in kvs}
    assert got["v_u8"] == (0, 42) and got["v_i8"] == (1, -42) and got["v_u16"] == (2, 42)
    assert got["v_i16"] == (3, -42) and got["v_u32"] == (4, 42) and got["v_i32"] == (5, -42)
    assert got["v_f32"][0] == 6 and got["v_f32"][1] == pytest.approx(np.float32(4.2))
    assert got["v_bool"] == (7, True) and got["v_str"] == (8, "hello")
    assert got["v_u64"] == (10, 42) and got["v_i64"] == (11, -42) and got["v_f64"] == (12, 4.2)
    assert got["v_arr"] == (9, ["hello", "world"])
    with pytest.raises(velo_cuda.VeloError) as e:
        g.metadata("absent")
    assert e.value.status == velo_cuda.ERR_MISSING_META


def test_repeated_key_keeps_the_last_value(tmp_path):
    g = _open(tmp_path, gw.header([("k", gw.T_U32, 1), ("k", gw.T_U32, 2)], []))
    assert g.metadata("k") == (4, 2)


def test_rejects_bad_values(tmp_path):
    bad_utf8 = struct.pack("<IIQQ", gw.MAGIC, 3, 0, 1) + struct.pack("<Q", 2) + b"\xff\xff"
    e = _err(tmp_path, bad_utf8)
    assert e.status == velo_cuda.ERR_GGUF and "UTF-8" in e.message
    unknown = struct.pack("<IIQQ", gw.MAGIC, 3, 0, 1) + gw._str("k") + struct.pack("<I", 99)
    e = _err(tmp_path, unknown)
    assert e.status == velo_cuda.ERR_GGUF and "unknown ggml type 99" in e.message
    # arrays of arrays: the array element reader has no array case
    nested = struct.pack("<IIQQ", gw.MAGIC, 3, 0, 1) + gw._str("k") + struct.pack("<IIQ", 9, 9, 1)
    assert _err(tmp_path, nested).status == velo_cuda.ERR_GGUF


def test_rejects_too_many_dims_and_unknown_tensor_type(tmp_path):
    e = _err(tmp_path, gw.header([], [("t", [1, 1, 1, 1, 1], 0, 0)]))
    assert e.status == velo_cuda.ERR_GGUF and "too many dims" in e.message
    e = _err(tmp_path, gw.header([], [("t", [4], 999, 0)]))
    assert e.status == velo_cuda.ERR_GGUF and "unknown ggml type 999" in e.message


def test_truncated_input_is_an_io_error(tmp_path):
    full = gw.header([("k", gw.T_STR, "value")], [])
    for cut in (0, 3, 7, 20, len(full) - 1):
        assert _err(tmp_path, full[:cut]).status == velo_cuda.ERR_IO
    with pytest.raises(velo_cuda.VeloError) as e:
        velo_cuda.Gguf(tmp_path / "missing.gguf")
    assert e.value.status == velo_cuda.ERR_IO
    # tensor data shorter than the tensor infos say
    data, _ = gw.build([], [("t", [4], gw.GGML_F32, b"\0" * 16)])
    assert _err(tmp_path, data[:-1]).status == velo_cuda.ERR_IO


def test_tensor_reading_and_alignment(tmp_path):
    vals = np.array([1, 2, 3, 4], np.float32).tobytes()
    data, start = gw.build([("general.alignment", gw.T_U64, 64)], [("test_tensor", [4], gw.GGML_F32, vals)],
                           alignment=64)
    g = _open(tmp_path, data)
    assert g.data_offset == start and start % 64 == 0
    t = g.tensor("test_tensor")
    assert t["nbytes"] == 16 and t["data"] == vals and t["shape"] == [4]
    with pytest.raises(velo_cuda.VeloError) as e:
        g.tensor("nonexistent")
    assert e.value.status == velo_cuda.ERR_MISSING_TENSOR


def test_tensor_nbytes_by_type(tmp_path):
    tensors = [("q32", [32], gw.GGML_Q4_0, b"\1" * 18), ("q64", [64], gw.GGML_Q4_0, b"\2" * 36),
               ("f", [100], gw.GGML_F32, b"\3" * 400), ("q4k", [256, 2], 12, b"\4" * 288)]
    g = _open(tmp_path, gw.build([], tensors)[0])
    assert [g.tensor(n)["nbytes"] for n in ("q32", "q64", "f", "q4k")] == [18, 36, 400, 288]


def _llama3_8b_kvs(**drop):
    kv = [("general.architecture", gw.T_STR, "llama"), ("llama.embedding_length", gw.T_U32, 4096),
          ("llama.block_count", gw.T_U32, 32), ("llama.attention.head_count", gw.T_U32, 32),
          ("llama.attention.head_count_kv", gw.T_U32, 8), ("llama.context_length", gw.T_U32, 8192),
          ("llama.feed_forward_length", gw.T_U32, 14336), ("llama.rope.freq_base", gw.T_F32, 500000.0),
          ("tokenizer.ggml.tokens", gw.T_ARR, (gw.T_STR, [""] * 128256))]
    return [x for x in kv if x[0] not in drop.get("keys", ())]


def test_parses_llama3_8b_dimensions(tmp_path):
    m = _open(tmp_path, gw.header(_llama3_8b_kvs(), [])).model_meta()
    assert m["arch"] == "llama" and m["n_vocab"] == 128256 and m["n_embd"] == 4096
    assert (m["n_layer"], m["n_head"], m["n_head_kv"], m["n_ff"], m["head_dim"]) == (32, 32, 8, 14336, 128)
    assert m["rope_freq_base"] == 500000.0 and m["n_ctx"] == 8192


def test_model_meta_defaults_and_missing_keys(tmp_path):
    keys = ("llama.attention.head_count_kv", "llama.context_length", "llama.rope.freq_base",
            "general.architecture")
    m = _open(tmp_path, gw.header(_llama3_8b_kvs(keys=keys), [])).model_meta()
    assert m["n_head_kv"] == m["n_head"] == 32
    assert m["n_ctx"] == 4096 and m["rope_freq_base"] == 10000.0 and m["arch"] == "llama"
    assert m["norm_eps"] == pytest.approx(1e-5)
    # vocab from llama.vocab_size when there is no token list
    kvs = _llama3_8b_kvs(keys=("tokenizer.ggml.tokens",)) + [("llama.vocab_size", gw.T_U32, 32000)]
    assert _open(tmp_path, gw.header(kvs, [])).model_meta()["n_vocab"] == 32000
    for key, expect in (("tokenizer.ggml.tokens", "vocab_size"),
                        ("llama.embedding_length", "llama.embedding_length"),
                        ("llama.attention.head_count", "head_count"),
                        ("llama.feed_forward_length", "feed_forward_length")):
        g = _open(tmp_path, gw.header(_llama3_8b_kvs(keys=(key,)), []))
        with pytest.raises(velo_cuda.VeloError) as e:
            g.model_meta()
        assert e.value.status == velo_cuda.ERR_MISSING_META and expect in e.value.message


def test_infer_quantization(tmp_path):
    kvs = _llama3_8b_kvs()
    q4k = gw.build(kvs, [("blk.0.attn_q.weight", [256], 12, b"\0" * 144)])[0]
    assert _open(tmp_path, q4k).model_meta()["quantization"] == 1
    q40 = gw.build(kvs, [("token_embd.weight", [32], gw.GGML_Q4_0, b"\0" * 18)])[0]
    assert _open(tmp_path, q40).model_meta()["quantization"] == 0


SHAPE = dict(n_vocab=512, n_embd=256, n_layer=2, n_head=2, n_head_kv=1, n_ff=512)


def test_synthetic_model_round_trip(tmp_path):
    meta, tensors = synthetic.llama_q4_model(**SHAPE, seed=4)
    p = tmp_path / "model.gguf"
    gw.write_model(p, meta, tensors, alignment=64)
    with velo_cuda.Gguf(p) as g:
        m = g.model_meta()
        for k in ("n_vocab", "n_embd", "n_layer", "n_head", "n_head_kv", "n_ff", "head_dim"):
            assert m[k] == meta[k], k
        assert m["rope_freq_base"] == meta["rope_freq_base"]
        assert m["norm_eps"] == np.float32(meta["norm_eps"])
        g.validate()
        ws = g.weights()
        assert [w[0] for w in ws] == (["token_embd.weight"] +
                                      [f"layers.{l}.{n}.weight" for l in range(2) for n in synthetic.LAYER_TENSORS]
                                      + ["output_norm.weight", "output.weight"])
        for name, dt, rows, cols, data in ws:
            sdt, arr, srows, scols = tensors[name]
            assert (dt, rows, cols) == (sdt, srows, scols), name
            assert data == np.ascontiguousarray(arr).tobytes(), name


def test_validation_errors_in_reference_order(tmp_path):
    meta, tensors = synthetic.llama_q4_model(**SHAPE, seed=4)
    for drop, status, text in (("token_embd.weight", velo_cuda.ERR_MISSING_TENSOR, "token_embd.weight"),
                               ("layers.1.feed_forward.w2.weight", velo_cuda.ERR_MISSING_TENSOR, "w2"),
                               ("output.weight", velo_cuda.ERR_MISSING_TENSOR, "output.weight")):
        t = {k: v for k, v in tensors.items() if k != drop}
        p = tmp_path / "m.gguf"
        gw.write_model(p, meta, t)
        g = velo_cuda.Gguf(p)
        with pytest.raises(velo_cuda.VeloError) as e:
            g.validate()
        assert e.value.status == status and text in e.value.message
        g.close()
    # wrong shape of the first tensor checked
    t = dict(tensors)
    dt, arr, rows, cols = t["token_embd.weight"]
    t["token_embd.weight"] = (dt, arr, rows // 2, cols * 2)
    p = tmp_path / "s.gguf"
    gw.write_model(p, meta, t)
    with velo_cuda.Gguf(p) as g:
        with pytest.raises(velo_cuda.VeloError) as e:
            g.validate()
        assert e.value.status == velo_cuda.ERR_INVALID_SHAPE and "expected shape" in e.value.message


def test_weights_reject_types_the_kernels_do_not_take(tmp_path):
    meta, tensors = synthetic.llama_q4_model(**SHAPE, seed=4)
    kvs = gw.model_kvs(meta)
    ts = gw.model_tensors(tensors)
    ts = [(n, s, 8 if n == "layers.0.attention.wq.weight" else gt, d if n != "layers.0.attention.wq.weight"
           else b"\0" * (256 * 256 // 32 * 34)) for n, s, gt, d in ts]
    data, _ = gw.build(kvs, ts)
    g = _open(tmp_path, data)
    g.validate()  # shapes are right
    with pytest.raises(velo_cuda.VeloError) as e:
        g.weights()
    assert e.value.status == velo_cuda.ERR_INVALID_ARGUMENT and "wq" in e.value.message
