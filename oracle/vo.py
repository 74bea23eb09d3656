"""ctypes wrapper of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl
reference legs import this module, and only as the checker.  The product
library never loads it.

Every function is a thin view of oracle/velo_oracle.c, which restates the
reference's CPU path (src/llama_cpu.rs, src/quant.rs, src/sampling.rs,
src/speculative.rs, src/paged_attention.rs of developertogo/velo-core) and the
acceptance spec of the product.
"""
import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libvelo_oracle.so")
_lib = None

F32, F16, Q4_0 = 0, 1, 2
KV_F16, KV_I8 = 0, 1

_P = ctypes.c_void_p
_SZ = ctypes.c_size_t


def build():
    """Compile the oracle (make in oracle/)."""
    subprocess.check_call(["make", "-s", "-C", _HERE])


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        sig = {
            "vo_f16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
            "vo_f32_to_f16": (ctypes.c_uint16, [ctypes.c_float]),
            "vo_dequant_q4_0_row": (None, [_P, _P, _SZ]),
            "vo_dequant_row": (None, [ctypes.c_int, _P, _P, _SZ]),
            "vo_row_bytes": (_SZ, [ctypes.c_int, _SZ]),
            "vo_quantize_q4_0_row": (None, [_P, _SZ, _P]),
            "vo_rms_norm": (None, [_P, _P, _SZ, ctypes.c_float]),
            "vo_silu": (ctypes.c_float, [ctypes.c_float]),
            "vo_rope": (None, [_P, _P, _SZ, _SZ, _SZ, _SZ, ctypes.c_float]),
            "vo_softmax": (None, [_P, _SZ]),
            "vo_matvec_quant": (None, [_P, _P, ctypes.c_int, _P, _SZ, _SZ]),
            "vo_model_new": (_P, [_P, _P, _P]),
            "vo_model_free": (None, [_P]),
            "vo_model_kv_pos": (_SZ, [_P]),
            "vo_model_set_kv_pos": (None, [_P, _SZ]),
            "vo_forward_one": (ctypes.c_int, [_P, ctypes.c_uint32, _SZ, _P]),
            "vo_forward_sequence": (ctypes.c_int, [_P, _P, _SZ, _P]),
            "vo_verify_tree": (ctypes.c_int, [_P, _P, _P, _SZ, _SZ, _P]),
            "vo_commit_path": (ctypes.c_int, [_P, _P, _SZ, _SZ]),
            "vo_read_kv": (ctypes.c_int, [_P, ctypes.c_int, _SZ, _SZ, _P]),
            "vo_write_kv": (ctypes.c_int, [_P, ctypes.c_int, _SZ, _SZ, _SZ, _P]),
            "vo_set_threads": (None, [ctypes.c_int]),
            "vo_greedy": (ctypes.c_uint32, [_P, _SZ, _P, _P]),
            "vo_find_best_path": (_SZ, [_P, _P, _P, _SZ, _P, _P]),
            "vo_accept": (ctypes.c_int, [_P, _P, _P, _P, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_int, ctypes.c_float, _P, _P, ctypes.c_int]),
            "vo_spec_exp": (ctypes.c_float, [ctypes.c_float]),
            "vo_accept_tree": (ctypes.c_int, [_P, _P, _P, _P, _P, ctypes.c_int, ctypes.c_int,
                                              ctypes.c_int, ctypes.c_float, _P, _P, _P]),
            "vo_row_stats": (None, [_P, ctypes.c_int, ctypes.c_float, _P, _P]),
            "vo_pages_for_tokens": (_SZ, [_SZ, _SZ]),
            "vo_allocator_new": (_P, [_SZ, _SZ]),
            "vo_allocator_free": (None, [_P]),
            "vo_allocator_allocate": (ctypes.c_int, [_P, ctypes.c_uint64, _SZ, _P, _P, _P, _P]),
            "vo_allocator_release": (ctypes.c_int, [_P, ctypes.c_uint64]),
            "vo_allocator_free_pages": (_SZ, [_P]),
            "vo_tree_attention": (None, [_P, ctypes.c_int, _P, _P, _P, _P, _P, _SZ, _P, _P,
                                         _P, _SZ, _SZ, _SZ, _SZ, _SZ, _P]),
            "vo_quantize_kv_int8": (None, [_P, _SZ, _P, _P]),
            "vo_kv_commit": (ctypes.c_int, [ctypes.c_int, _P, _P, _P, _SZ, _SZ, _P, _P, _SZ,
                                            _SZ, _SZ, _SZ]),
            "vo_shard_strategy": (ctypes.c_int, [ctypes.c_char_p]),
            "vo_shard_weight": (ctypes.c_int, [ctypes.c_int, _P, _SZ, _SZ, ctypes.c_int,
                                               ctypes.c_int, ctypes.c_int, _P, _P, _P]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def c_arr(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def set_threads(n):
    """Split each matvec's rows over n threads (same bits; tests only)."""
    lib().vo_set_threads(int(n))


# ---------------------------------------------------------------- quant.rs
def f16_to_f32(bits):
    return lib().vo_f16_to_f32(int(bits))


def f32_to_f16(x):
    return lib().vo_f32_to_f16(float(x))


def dequant_row(dtype, data, n):
    data = c_arr(data, np.uint8)
    out = np.zeros(n, np.float32)
    lib().vo_dequant_row(dtype, ptr(data), ptr(out), n)
    return out


def quantize_q4_0(x):
    """[rows][cols] float32 -> [rows][cols/32*18] uint8 (interleaved q4_0)."""
    x = c_arr(x, np.float32)
    rows, cols = x.shape
    out = np.zeros((rows, cols // 32 * 18), np.uint8)
    L = lib()
    for r in range(rows):
        L.vo_quantize_q4_0_row(ptr(x[r]), cols, ptr(out[r]))
    return out


def dequant_matrix(dtype, data, rows, cols):
    data = c_arr(data, np.uint8).reshape(rows, -1)
    out = np.zeros((rows, cols), np.float32)
    L = lib()
    for r in range(rows):
        L.vo_dequant_row(dtype, ptr(data[r]), ptr(out[r]), cols)
    return out


# ----------------------------------------------------------- llama_cpu.rs
def rms_norm(x, w, eps):
    x = c_arr(x, np.float32).copy()
    w = c_arr(w, np.float32)
    lib().vo_rms_norm(ptr(x), ptr(w), x.size, eps)
    return x


def silu(x):
    return lib().vo_silu(float(x))


def rope(q, k, pos, n_heads, n_kv, head_dim, base):
    q = c_arr(q, np.float32).copy()
    k = c_arr(k, np.float32).copy()
    lib().vo_rope(ptr(q), ptr(k), pos, n_heads, n_kv, head_dim, base)
    return q, k


def softmax(x):
    x = c_arr(x, np.float32).copy()
    lib().vo_softmax(ptr(x), x.size)
    return x


def matvec_quant(data, dtype, x, rows, cols):
    data = c_arr(data, np.uint8)
    x = c_arr(x, np.float32)
    out = np.zeros(rows, np.float32)
    lib().vo_matvec_quant(ptr(out), ptr(data), dtype, ptr(x), rows, cols)
    return out


class Meta(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in
                ("n_vocab", "n_embd", "n_layer", "n_head", "n_head_kv", "n_ff",
                 "head_dim", "n_ctx")] + [("rope_freq_base", ctypes.c_float),
                                          ("norm_eps", ctypes.c_float)]


class Model:
    """LlamaCpuModel (llama_cpu.rs:168-419) over raw tensor bytes.

    tensors: list in the oracle order (token_embd, output_norm, output|None,
    then per layer attention_norm, wq, wk, wv, wo, ffn_norm, w1, w2, w3) of
    (dtype, numpy uint8/float32 array)."""

    def __init__(self, meta: dict, tensors):
        self._keep = []
        ptrs = (ctypes.c_void_p * len(tensors))()
        dts = (ctypes.c_int * len(tensors))()
        for i, t in enumerate(tensors):
            if t is None:
                ptrs[i] = None
                dts[i] = F32
                continue
            dt, arr = t
            arr = np.ascontiguousarray(arr)
            self._keep.append(arr)
            ptrs[i] = arr.ctypes.data
            dts[i] = dt
        self.meta = meta
        m = Meta(**meta)
        self._h = lib().vo_model_new(ctypes.byref(m), ptrs, dts)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().vo_model_free(self._h)
            self._h = None

    @property
    def pos(self):
        return lib().vo_model_kv_pos(self._h)

    @pos.setter
    def pos(self, p):
        lib().vo_model_set_kv_pos(self._h, p)

    def forward_one(self, token, pos):
        out = np.zeros(self.meta["n_vocab"], np.float32)
        rc = lib().vo_forward_one(self._h, token, pos, ptr(out))
        if rc:
            raise ValueError("forward_one failed")
        return out

    def forward_sequence(self, tokens):
        t = c_arr(tokens, np.uint32)
        out = np.zeros(self.meta["n_vocab"], np.float32)
        rc = lib().vo_forward_sequence(self._h, ptr(t), t.size, ptr(out))
        if rc:
            raise ValueError("forward_sequence failed")
        return out

    def verify_tree(self, tokens, parents, n_cached):
        t = c_arr(tokens, np.uint32)
        p = c_arr(parents, np.int32)
        out = np.zeros((t.size, self.meta["n_vocab"]), np.float32)
        rc = lib().vo_verify_tree(self._h, ptr(t), ptr(p), t.size, n_cached, ptr(out))
        if rc:
            raise ValueError("verify_tree failed")
        return out

    def commit_path(self, path, n_cached):
        p = c_arr(path, np.int32)
        rc = lib().vo_commit_path(self._h, ptr(p), p.size, n_cached)
        if rc:
            raise ValueError("commit_path failed")

    def write_kv(self, which, layer, pos0, rows):
        """Place cached K (which 0) or V (1) rows [n][n_kv * head_dim] of
        `layer` at positions pos0.. (test setup in place of a prefill)."""
        r = c_arr(rows, np.float32)
        kvs = self.meta["n_head_kv"] * self.meta["head_dim"]
        n = r.size // kvs
        rc = lib().vo_write_kv(self._h, which, layer, pos0, n, ptr(r))
        if rc:
            raise ValueError("write_kv failed")

    def read_kv(self, which, layer, n):
        kvs = self.meta["n_head_kv"] * self.meta["head_dim"]
        out = np.zeros((n, kvs), np.float32)
        rc = lib().vo_read_kv(self._h, which, layer, n, ptr(out))
        if rc:
            raise ValueError("read_kv failed")
        return out


# ------------------------------------------------------------ sampling.rs
def greedy(logits, mask=None):
    lg = c_arr(logits, np.float32)
    mk = None if mask is None else c_arr(mask, np.uint8)
    conf = ctypes.c_float()
    tok = lib().vo_greedy(ptr(lg), lg.size, ptr(mk), ctypes.byref(conf))
    return tok, conf.value


# --------------------------------------------------------- speculative.rs
def find_best_path(parents, tokens, expected):
    p = c_arr(parents, np.int32)
    t = c_arr(tokens, np.uint32)
    e = c_arr(expected, np.uint32)
    out = np.zeros(max(1, p.size), np.int32)
    bonus = ctypes.c_uint32()
    n = lib().vo_find_best_path(ptr(p), ptr(t), ptr(e), p.size, ptr(out), ctypes.byref(bonus))
    return out[:n].tolist(), bonus.value


def accept(tgt, drf, tok, u, temperature, n_threads=0):
    """Acceptance spec.  tgt [B][k+1][V], drf [B][k][V] (None if greedy)."""
    tgt = c_arr(tgt, np.float32)
    B, k1, V = tgt.shape
    k = k1 - 1
    drf = None if drf is None else c_arr(drf, np.float32)
    tok = c_arr(tok, np.uint32).reshape(B, k)
    u = np.zeros((B, k + 1), np.float32) if u is None else c_arr(u, np.float32).reshape(B, k + 1)
    acc = np.zeros(B, np.int32)
    bonus = np.zeros(B, np.uint32)
    rc = lib().vo_accept(ptr(tgt), ptr(drf), ptr(tok), ptr(u), B, k, V, temperature,
                         ptr(acc), ptr(bonus), n_threads)
    if rc:
        raise ValueError("vo_accept: invalid arguments")
    return acc, bonus


def accept_tree(tgt, drf, tok, parents, u, temperature):
    """Tree rejection sampling spec.  tgt [B][N][V], drf [B][N-1][V],
    tok / parents [B][N], u [B][N].  Returns (path [B][N] -1 padded,
    path_len [B], bonus [B])."""
    tgt = c_arr(tgt, np.float32)
    B, N, V = tgt.shape
    drf = c_arr(drf, np.float32).reshape(B, N - 1, V)
    tok = c_arr(tok, np.uint32).reshape(B, N)
    par = c_arr(parents, np.int32).reshape(B, N)
    u = c_arr(u, np.float32).reshape(B, N)
    path = np.zeros((B, N), np.int32)
    plen = np.zeros(B, np.int32)
    bonus = np.zeros(B, np.uint32)
    rc = lib().vo_accept_tree(ptr(tgt), ptr(drf), ptr(tok), ptr(par), ptr(u), B, N, V,
                              float(temperature), ptr(path), ptr(plen), ptr(bonus))
    if rc:
        raise ValueError("vo_accept_tree: invalid arguments")
    return path, plen, bonus


def spec_exp(y):
    return lib().vo_spec_exp(float(y))


def row_stats(row, inv_t):
    row = c_arr(row, np.float32)
    M, Z = ctypes.c_float(), ctypes.c_float()
    lib().vo_row_stats(ptr(row), row.size, inv_t, ctypes.byref(M), ctypes.byref(Z))
    return M.value, Z.value


# ------------------------------------------------------ paged_attention.rs
def pages_for_tokens(tokens, block_size):
    return lib().vo_pages_for_tokens(tokens, block_size)


class OutOfPages(Exception):
    def __init__(self, requested, available):
        super().__init__(f"requested {requested} pages but only {available} are available")
        self.requested = requested
        self.available = available


class Allocator:
    """PagedAttentionBlockManager (paged_attention.rs:92-211)."""

    def __init__(self, block_size, total_pages):
        self._h = lib().vo_allocator_new(block_size, total_pages)
        if not self._h:
            raise ValueError("block size must be greater than zero")
        self.total = total_pages

    def __del__(self):
        if getattr(self, "_h", None):
            lib().vo_allocator_free(self._h)

    def allocate(self, handle, token_len):
        pages = np.zeros(max(1, self.total), np.uint32)
        n, req, av = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
        rc = lib().vo_allocator_allocate(self._h, handle, token_len, ptr(pages),
                                         ctypes.byref(n), ctypes.byref(req), ctypes.byref(av))
        if rc:
            raise OutOfPages(req.value, av.value)
        return pages[:n.value].tolist()

    def release(self, handle):
        if lib().vo_allocator_release(self._h, handle):
            raise KeyError(handle)

    def free_pages(self):
        return lib().vo_allocator_free_pages(self._h)


# ------------------------------------------------------- tree attention
def tree_attention(q, kv_dtype, k_pool, v_pool, k_scale, v_scale, page_table, n_cached,
                   k_nodes, v_nodes, parents, n_head, n_kv, hd, page_size):
    q = c_arr(q, np.float32)
    n_nodes = q.shape[0]
    out = np.zeros((n_nodes, n_head, hd), np.float32)
    pt = c_arr(page_table, np.uint32)
    kn = c_arr(k_nodes, np.uint16)
    vn = c_arr(v_nodes, np.uint16)
    par = c_arr(parents, np.int32)
    ks = None if k_scale is None else c_arr(k_scale, np.uint16)
    vs = None if v_scale is None else c_arr(v_scale, np.uint16)
    kp = np.ascontiguousarray(k_pool)
    vp = np.ascontiguousarray(v_pool)
    lib().vo_tree_attention(ptr(q), kv_dtype, ptr(kp), ptr(vp), ptr(ks), ptr(vs), ptr(pt),
                            n_cached, ptr(kn), ptr(vn), ptr(par), n_nodes, n_head, n_kv, hd,
                            page_size, ptr(out))
    return out


def quantize_kv_int8(x):
    x = c_arr(x, np.float32)
    q = np.zeros(x.size, np.int8)
    s = ctypes.c_uint16()
    lib().vo_quantize_kv_int8(ptr(x), x.size, ptr(q), ctypes.byref(s))
    return q, s.value


def kv_commit(kv_dtype, pool, scale, page_table, n_bound, n_cached, node_kv, path,
              n_kv, hd, page_size):
    """In-place on pool / scale (numpy arrays).  Returns the status code."""
    pt = c_arr(page_table, np.uint32)
    nk = c_arr(node_kv, np.uint16)
    p = c_arr(path, np.int32)
    return lib().vo_kv_commit(kv_dtype, ptr(pool), ptr(scale), ptr(pt), n_bound, n_cached,
                              ptr(nk), ptr(p), p.size, n_kv, hd, page_size)


# ------------------------------------------------------------ sharding.rs
def shard_strategy(name):
    return lib().vo_shard_strategy(name.encode())


def shard_weight(dtype, data, rows, cols, strategy, tp, rank):
    """sharding.rs:28-110.  Returns (bytes, rows, cols) or raises ValueError."""
    d = np.ascontiguousarray(data).view(np.uint8).reshape(-1)  # raw bytes of any dtype
    out = np.zeros(d.size, np.uint8)
    r, c = ctypes.c_size_t(), ctypes.c_size_t()
    rc = lib().vo_shard_weight(dtype, ptr(d), rows, cols, strategy, tp, rank, ptr(out),
                               ctypes.byref(r), ctypes.byref(c))
    if rc:
        raise ValueError("shard_weight: not divisible")
    return out[:r.value * row_bytes(dtype, c.value)], r.value, c.value


def row_bytes(dtype, cols):
    return lib().vo_row_bytes(dtype, cols)
