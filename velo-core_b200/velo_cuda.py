"""Python view of the velo_cuda C ABI (include/velo_cuda.h), through ctypes.

This is the host-side harness the tests and bench.py use; it calls the same
extern "C" entry points a Rust backend binds.  There is
no fallback: if libvelo_cuda.so is missing, importing fails loudly.

Errors mirror the reference: every non-zero status raises VeloError whose
`status` is the velo_status code (SpeculativeError / PageManagerError
analogues) and whose message is velo_cuda_last_error().
"""
import ctypes
import os
import re

import numpy as np

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libvelo_cuda.so")
HEADER = os.path.join(os.path.dirname(_PKG), "include", "velo_cuda.h")

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_EMPTY_DRAFT_WINDOW = 2
ERR_DRAFT_TOO_MANY = 3
ERR_TARGET_WRONG_LENGTH = 4
ERR_OUT_OF_PAGES = 5
ERR_UNKNOWN_HANDLE = 6
ERR_INVALID_BLOCK_SIZE = 7
ERR_CUDA = 8
ERR_NO_DEVICE = 9
ERR_TIMEOUT = 10
ERR_OUT_OF_MEMORY = 11
ERR_NCCL = 12
ERR_DEVICE_FLAG = 13
ERR_IO = 14
ERR_GGUF = 15
ERR_MISSING_META = 16
ERR_MISSING_TENSOR = 17
ERR_INVALID_SHAPE = 18

KV_F16, KV_INT8, KV_F32 = 0, 1, 2  # KV_F32: the fp32 path of the model

_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_SZ = ctypes.c_size_t
_U32P = ctypes.POINTER(ctypes.c_uint32)
_SZP = ctypes.POINTER(ctypes.c_size_t)
# velo_session.h model callbacks
DRAFT_FN = ctypes.CFUNCTYPE(ctypes.c_int32, ctypes.c_void_p, _U32P, ctypes.c_size_t, ctypes.c_size_t, _U32P,
                            ctypes.c_size_t, _SZP)
VERIFY_FN = ctypes.CFUNCTYPE(ctypes.c_int32, ctypes.c_void_p, _U32P, ctypes.c_size_t, _U32P, ctypes.c_size_t,
                             _U32P, ctypes.c_size_t, _SZP)


_U32PP = ctypes.POINTER(_U32P)
DRAFT_BATCH_FN = ctypes.CFUNCTYPE(ctypes.c_int32, ctypes.c_void_p, ctypes.c_size_t, _U32P, _U32PP, _SZP, _SZP,
                                  _U32P, ctypes.c_size_t, _SZP)
VERIFY_BATCH_FN = ctypes.CFUNCTYPE(ctypes.c_int32, ctypes.c_void_p, ctypes.c_size_t, _U32P, _U32PP, _SZP, _U32PP,
                                   _SZP, _U32P, ctypes.c_size_t, _SZP)


class SpecStats(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in
                ("draft_calls", "target_calls", "drafted_tokens", "accepted_tokens", "rejected_tokens")]
_lib = None


class VeloError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f"velo_cuda status {status}: {message}")
        self.status = status
        self.message = message


class Config(ctypes.Structure):
    _fields_ = [("struct_size", ctypes.c_uint32), ("page_size", ctypes.c_uint32),
                ("kv_dtype", ctypes.c_uint32), ("max_slots", ctypes.c_uint32),
                ("total_pages", ctypes.c_uint32), ("max_pages_per_slot", ctypes.c_uint32)]


_SIGS = {
    "velo_cuda_abi_version": (_I32, []),
    "velo_cuda_last_error": (ctypes.c_char_p, []),
    "velo_cuda_create": (_I32, [_P, _I32, _I32, _I32, _P, ctypes.POINTER(_P)]),
    "velo_cuda_destroy": (None, [_P]),
    "velo_cuda_set_stream": (_I32, [_P, _P]),
    "velo_cuda_sync": (_I32, [_P, ctypes.c_int64]),
    "velo_cuda_accept": (_I32, [_P, _P, _P, _P, _P, _I32, _I32, _I32, ctypes.c_float, _P, _P]),
    "velo_cuda_accept_device": (_I32, [_P, _P, _P, _P, _P, _I32, _I32, _I32, ctypes.c_float,
                                       _P, _P]),
    "velo_cuda_accept_static": (_I32, [_P, _P, _P, _P, _I32, _I32, _I32, ctypes.c_float, _P, _P,
                                       _P]),
    "velo_cuda_accept_static_error": (_I32, [_P, _P]),
    "velo_cuda_accept_tree": (_I32, [_P, _P, _P, _P, _P, _P, _I32, _I32, _I32, ctypes.c_float, _P, _P,
                                     _P]),
    "velo_cuda_accept_tree_device": (_I32, [_P, _P, _P, _P, _P, _P, _I32, _I32, _I32, ctypes.c_float,
                                            _P, _P, _P]),
    "velo_cuda_q4_0_repacked_bytes": (ctypes.c_size_t, [_I32, _I32]),
    "velo_cuda_q4_0_repack": (_I32, [_P, _P, _P, _I32, _I32, _P]),
    "velo_cuda_gemm_q4_0": (_I32, [_P, _P, _P, _I32, _I32, _I32, _P, _I32, _I32]),
    "velo_cuda_tree_attention": (_I32, [_P, _P, _P, _P, _P, _P, _I32, _P, _I32, _P, _P, _P, _P,
                                        _I32, _I32, _I32, _I32, _I32, _I32, _P, _I32]),
    "velo_cuda_load_model": (_I32, [_P, _P, _P, _I32]),
    "velo_cuda_bind_slot": (_I32, [_P, ctypes.c_uint32, _P, ctypes.c_size_t]),
    "velo_cuda_write_kv": (_I32, [_P, ctypes.c_uint32, _I32, _I32, _I32, _P, _P]),
    "velo_cuda_read_kv": (_I32, [_P, ctypes.c_uint32, _I32, _I32, _I32, _P, _P, _P, _P]),
    "velo_cuda_verify_step": (_I32, [_P, _P, _P]),
    "velo_cuda_nccl_unique_id": (_I32, [_P]),
    "velo_cuda_profile": (_I32, [_P, _I32]),
    "velo_cuda_profile_read": (_I32, [_P, ctypes.POINTER(ctypes.c_double), _I32, ctypes.POINTER(_I32)]),
    "velo_cuda_tp_sum_path": (_I32, [_P, ctypes.POINTER(_I32)]),
    "velo_cuda_tp_wait_selftest": (_I32, [_I32, ctypes.POINTER(_I32)]),
    "velo_cuda_shard_strategy": (_I32, [ctypes.c_char_p]),
    "velo_cuda_shard_weight": (_I32, [_P, _I32, _I32, _I32, _P, ctypes.c_size_t,
                                      ctypes.POINTER(ctypes.c_uint64),
                                      ctypes.POINTER(ctypes.c_uint64)]),
    "velo_cuda_slot_allocate": (_I32, [_P, ctypes.c_uint32, _SZ, _P, _SZ, ctypes.POINTER(_SZ)]),
    "velo_cuda_slot_release": (_I32, [_P, ctypes.c_uint32]),
    "velo_cuda_free_pages": (_I32, [_P, ctypes.POINTER(_SZ)]),
    "velo_page_allocator_create": (_I32, [_SZ, _SZ, ctypes.POINTER(_P)]),
    "velo_page_allocator_destroy": (None, [_P]),
    "velo_page_allocator_allocate": (_I32, [_P, ctypes.c_uint64, _SZ, _P, _SZ, ctypes.POINTER(_SZ),
                                            ctypes.POINTER(_SZ), ctypes.POINTER(_SZ)]),
    "velo_page_allocator_release": (_I32, [_P, ctypes.c_uint64]),
    "velo_page_allocator_mapped_pages": (_I32, [_P, ctypes.c_uint64, _P, _SZ, ctypes.POINTER(_SZ)]),
    "velo_page_allocator_free_pages": (_SZ, [_P]),
    "velo_page_allocator_pages_for_tokens": (_SZ, [_P, _SZ]),
    "velo_gguf_open": (_I32, [ctypes.c_char_p, ctypes.POINTER(_P)]),
    "velo_gguf_close": (None, [_P]),
    "velo_gguf_version": (ctypes.c_uint32, [_P]),
    "velo_gguf_n_tensors": (ctypes.c_uint64, [_P]),
    "velo_gguf_n_metadata": (ctypes.c_uint64, [_P]),
    "velo_gguf_data_offset": (ctypes.c_uint64, [_P]),
    "velo_gguf_metadata": (_I32, [_P, ctypes.c_char_p, _P]),
    "velo_gguf_metadata_elem": (_I32, [_P, ctypes.c_char_p, ctypes.c_uint64, _P]),
    "velo_gguf_tensor_info": (_I32, [_P, ctypes.c_char_p, _P]),
    "velo_gguf_read_model_meta": (_I32, [_P, _P]),
    "velo_gguf_validate": (_I32, [_P]),
    "velo_gguf_weights": (_I32, [_P, _P, _I32, ctypes.POINTER(_I32)]),
    "velo_cuda_load_gguf": (_I32, [_P, ctypes.c_char_p]),
    "velo_spec_session_create": (_I32, [ctypes.c_uint32, ctypes.c_uint32, _P, _SZ, ctypes.POINTER(_P)]),
    "velo_spec_session_destroy": (None, [_P]),
    "velo_spec_session_draft": (_I32, [_P, DRAFT_FN, _P, VERIFY_FN, _P, _SZ, _P, _SZ, _SZP]),
    "velo_spec_session_commit": (_I32, [_P, _P, _SZ, _P, _SZ, _P, _SZ, _SZP]),
    "velo_spec_session_take_rejected": (_I32, [_P, _U32P]),
    "velo_spec_session_has_pending_rejection": (_I32, [_P]),
    "velo_spec_session_context": (_SZ, [_P, _P, _SZ]),
    "velo_spec_session_window": (ctypes.c_uint32, [_P]),
    "velo_spec_session_stats": (None, [_P, ctypes.POINTER(SpecStats)]),
    "velo_spec_session_record_draft_call": (None, [_P]),
    "velo_spec_session_record_target_call": (None, [_P]),
    "velo_spec_generate_batch": (_I32, [ctypes.c_uint32, ctypes.c_uint32, _SZ, DRAFT_BATCH_FN, _P,
                                        VERIFY_BATCH_FN, _P, _SZ, _P, _P, _P, _P, _P, _P]),
    "velo_spec_generate": (_I32, [ctypes.c_uint32, ctypes.c_uint32, DRAFT_FN, _P, VERIFY_FN, _P, _P, _SZ, _SZ,
                                  _P, _SZ, _SZP, ctypes.POINTER(SpecStats)]),
}

DT_F32, DT_F16, DT_Q4_0 = 0, 1, 2


class ModelDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in
                ("struct_size", "n_vocab", "n_embd", "n_layer", "n_head", "n_head_kv", "n_ff",
                 "head_dim")] + [("rope_freq_base", ctypes.c_float), ("norm_eps", ctypes.c_float)]


class WeightDesc(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("dtype", ctypes.c_int32), ("flags", ctypes.c_uint32),
                ("data", ctypes.c_void_p), ("rows", ctypes.c_uint64), ("cols", ctypes.c_uint64)]


WEIGHT_DEVICE, WEIGHT_SHARD = 1, 2


class VerifyBatch(ctypes.Structure):
    _fields_ = [("struct_size", ctypes.c_uint32), ("B", ctypes.c_int32), ("n_nodes", ctypes.c_int32),
                ("slots", _P), ("ctx_len", _P), ("tokens", _P), ("parents", _P),
                ("temperature", ctypes.c_float), ("draft_logits", _P), ("uniforms", _P),
                ("commit", ctypes.c_int32)]


class VerifyResult(ctypes.Structure):
    _fields_ = [("accepted_len", _P), ("accepted_nodes", _P), ("bonus_token", _P), ("logits", _P),
                ("expected", _P)]

EPI_STORE_F32, EPI_STORE_F16, EPI_ADD_F32, EPI_SWIGLU, EPI_STORE_BF16 = 0, 1, 2, 3, 4

# velo_phase: the step phases velo_cuda_profile times
PHASES = ("other", "gemm_qkv", "attention", "gemm_o", "gemm_ffn_up", "gemm_ffn_down", "allreduce",
          "lm_head", "accept_commit")


def lib():
    """Load libvelo_cuda.so (built in-tree by velo-core_b200/build.py)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is not built; run __graft_entry__.build()")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def header_functions():
    """Names of the functions include/*.h declare."""
    inc = os.path.dirname(HEADER)
    src = "".join(open(os.path.join(inc, f)).read() for f in sorted(os.listdir(inc)) if f.endswith(".h"))
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(velo_(?:cuda|page_allocator|gguf|spec)_\w+)\s*\(", src)))


def last_error():
    return lib().velo_cuda_last_error().decode()


def check(status):
    if status != OK:
        raise VeloError(status, last_error())
    return status


def _ptr(a):
    """Host numpy array or device torch tensor -> void*."""
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        return a.ctypes.data_as(_P)
    return ctypes.c_void_p(a.data_ptr())  # torch tensor


class Context:
    """One velo_cuda_ctx: a device, a stream and the device buffers."""

    def __init__(self, device=0, page_size=16, kv_dtype=KV_F16, max_slots=1, total_pages=0,
                 max_pages_per_slot=0, tp_rank=0, tp_size=1, nccl_id=None):
        cfg = Config(ctypes.sizeof(Config), page_size, kv_dtype, max_slots, total_pages,
                     max_pages_per_slot)
        self.kv_dtype = kv_dtype
        h = _P()
        nid = None if nccl_id is None else ctypes.c_char_p(bytes(nccl_id))
        check(lib().velo_cuda_create(ctypes.byref(cfg), device, tp_rank, tp_size, nid,
                                     ctypes.byref(h)))
        self._h = h
        self.device = device

    def close(self):
        if getattr(self, "_h", None):
            lib().velo_cuda_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    @property
    def handle(self):
        return self._h

    def set_stream(self, stream_ptr):
        check(lib().velo_cuda_set_stream(self._h, _P(stream_ptr) if stream_ptr else None))

    def sync(self, timeout_ns=-1):
        check(lib().velo_cuda_sync(self._h, timeout_ns))

    # ------------------------------------------------------------ acceptance
    def accept(self, target_logits, draft_logits, draft_tokens, uniforms, temperature):
        """Host-buffer acceptance.  Returns (accepted_len[B] i32, bonus[B] u32)."""
        t = np.ascontiguousarray(target_logits, np.float32)
        B, k1, V = t.shape
        k = k1 - 1
        d = None if draft_logits is None else np.ascontiguousarray(draft_logits, np.float32)
        tok = np.ascontiguousarray(draft_tokens, np.uint32).reshape(B, k)
        u = None if uniforms is None else np.ascontiguousarray(uniforms, np.float32)
        acc = np.zeros(B, np.int32)
        bonus = np.zeros(B, np.uint32)
        check(lib().velo_cuda_accept(self._h, _ptr(t), _ptr(d), _ptr(tok), _ptr(u), B, k, V,
                                     float(temperature), _ptr(acc), _ptr(bonus)))
        return acc, bonus

    def accept_device(self, target_logits, draft_logits, draft_tokens, uniforms, temperature,
                      accepted_len, bonus_token):
        """Device-buffer acceptance on torch CUDA tensors (asynchronous)."""
        B, k1, V = target_logits.shape
        check(lib().velo_cuda_accept_device(
            self._h, _ptr(target_logits), _ptr(draft_logits), _ptr(draft_tokens),
            _ptr(uniforms), B, k1 - 1, V, float(temperature), _ptr(accepted_len),
            _ptr(bonus_token)))

    # ------------------------------------------------------------ q4_0 GEMM
    def accept_tree(self, target_logits, draft_logits, tokens, parents, uniforms, temperature):
        """Tree rejection sampling, host buffers: target [B][N][V], draft
        [B][N-1][V], tokens / parents / uniforms [B][N].  Returns (path [B][N],
        path_len [B], bonus [B])."""
        tgt = np.ascontiguousarray(target_logits, np.float32)
        B, N, V = tgt.shape
        drf = np.ascontiguousarray(draft_logits, np.float32)
        tok = np.ascontiguousarray(tokens, np.uint32).reshape(B, N)
        par = np.ascontiguousarray(parents, np.int32).reshape(B, N)
        u = np.ascontiguousarray(uniforms, np.float32).reshape(B, N)
        path = np.zeros((B, N), np.int32)
        plen = np.zeros(B, np.int32)
        bonus = np.zeros(B, np.uint32)
        check(lib().velo_cuda_accept_tree(self._h, _ptr(tgt), _ptr(drf), _ptr(tok), _ptr(par), _ptr(u), B,
                                          N, V, float(temperature), _ptr(path), _ptr(plen), _ptr(bonus)))
        return path, plen, bonus

    def accept_tree_device(self, target_logits, draft_logits, tokens, parents, uniforms, temperature,
                           path, path_len, bonus):
        """Device-buffer form (torch CUDA tensors), asynchronous."""
        B, N, V = target_logits.shape
        check(lib().velo_cuda_accept_tree_device(
            self._h, _ptr(target_logits), _ptr(draft_logits), _ptr(tokens), _ptr(parents), _ptr(uniforms),
            B, N, V, float(temperature), _ptr(path), _ptr(path_len), _ptr(bonus)))

    def q4_0_repack(self, src, N, K, out, src_b=None):
        """Repack q4_0 rows (device uint8 [N][K/32*18], or two halves for a
        SwiGLU pair) into `out` (device, q4_0_repacked_bytes(N, K) bytes)."""
        check(lib().velo_cuda_q4_0_repack(self._h, _ptr(src), _ptr(src_b), N, K, _ptr(out)))

    def gemm_q4_0(self, w, x, M, N, K, y, ldy, mode):
        """y (+)= x[M][K] (f16) * W^T on the tensor cores; asynchronous."""
        check(lib().velo_cuda_gemm_q4_0(self._h, _ptr(w), _ptr(x), M, N, K, _ptr(y), ldy, mode))


    # ------------------------------------------------------------ attention
    def tree_attention(self, q, k_pool, v_pool, k_scale, v_scale, page_table, ctx_len, node_k,
                       node_v, parents, n_kv, kv_dtype, out):
        """Tree-masked paged attention on torch CUDA tensors (asynchronous).
        q [B][N][Hq][128] f16; pools [P][n_kv][16][128]; out f32 or f16."""
        B, N, Hq, hd = q.shape
        out_f16 = 1 if out.dtype.itemsize == 2 else 0
        check(lib().velo_cuda_tree_attention(
            self._h, _ptr(q), _ptr(k_pool), _ptr(v_pool), _ptr(k_scale), _ptr(v_scale),
            k_pool.shape[0], _ptr(page_table), page_table.shape[1], _ptr(ctx_len), _ptr(node_k),
            _ptr(node_v), _ptr(parents), B, N, Hq, n_kv, hd, kv_dtype, _ptr(out), out_f16))


    # ------------------------------------------------------------ model + verify
    def load_model(self, meta, tensors, shards=False):
        """meta: dict of velo_model_desc fields; tensors: {name: (dtype, array, rows, cols)}
        in the reference's WeightStore layout.  An array is a host ndarray or a
        CUDA torch tensor on the context's device (VELO_WEIGHT_DEVICE);
        shards=True: the tensors are already this rank's shards."""
        d = ModelDesc(ctypes.sizeof(ModelDesc), *(int(meta[k]) for k in
                      ("n_vocab", "n_embd", "n_layer", "n_head", "n_head_kv", "n_ff", "head_dim")),
                      float(meta["rope_freq_base"]), float(meta["norm_eps"]))
        keep, ws = [], (WeightDesc * len(tensors))()
        for i, (name, (dt, arr, rows, cols)) in enumerate(tensors.items()):
            flags = WEIGHT_SHARD if shards else 0
            if hasattr(arr, "data_ptr") and getattr(arr, "is_cuda", False):
                a = arr.contiguous()
                ptr, flags = a.data_ptr(), flags | WEIGHT_DEVICE
            else:
                a = np.ascontiguousarray(arr)
                ptr = a.ctypes.data
            nm = name.encode()
            keep += [a, nm]
            ws[i] = WeightDesc(nm, dt, flags, ptr, rows, cols)
        check(lib().velo_cuda_load_model(self._h, ctypes.byref(d), ws, len(tensors)))

    def load_gguf(self, path):
        """load_gguf + upload (velo_cuda_load_gguf)."""
        check(lib().velo_cuda_load_gguf(self._h, os.fsencode(path)))

    def bind_slot(self, slot, pages):
        p = np.ascontiguousarray(pages, np.uint32)
        check(lib().velo_cuda_bind_slot(self._h, slot, _ptr(p), p.size))

    def slot_allocate(self, slot, token_len):
        """Pages for `token_len` tokens from the context's allocator, bound to
        `slot`; returns their ids."""
        need = -(-int(token_len) // 16)
        pages = np.zeros(max(need, 1), np.uint32)
        n = _SZ()
        check(lib().velo_cuda_slot_allocate(self._h, slot, token_len, _ptr(pages), pages.size,
                                            ctypes.byref(n)))
        return pages[:n.value].copy()

    def slot_release(self, slot):
        check(lib().velo_cuda_slot_release(self._h, slot))

    def free_pages(self):
        n = _SZ()
        check(lib().velo_cuda_free_pages(self._h, ctypes.byref(n)))
        return n.value

    def write_kv(self, slot, layer, pos0, k, v):
        """k, v [n][n_kv][head_dim]: f32 for an f32 pool, else f16."""
        dt = np.float32 if self.kv_dtype == KV_F32 else np.float16
        k = np.ascontiguousarray(k, dt)
        v = np.ascontiguousarray(v, dt)
        check(lib().velo_cuda_write_kv(self._h, slot, layer, pos0, k.shape[0], _ptr(k), _ptr(v)))

    def read_kv(self, slot, layer, pos0, n, n_kv, int8=False, head_dim=128):
        dt = np.int8 if int8 else np.float32 if self.kv_dtype == KV_F32 else np.float16
        k = np.zeros((n, n_kv, head_dim), dt)
        v = np.zeros((n, n_kv, head_dim), dt)
        ks = np.zeros((n, n_kv), np.uint16)
        vs = np.zeros((n, n_kv), np.uint16)
        check(lib().velo_cuda_read_kv(self._h, slot, layer, pos0, n, _ptr(k), _ptr(v), _ptr(ks),
                                      _ptr(vs)))
        return (k, v, ks, vs) if int8 else (k, v)

    def profile(self, enable=True):
        """Start (or stop) timing the phases of the following verify steps."""
        check(lib().velo_cuda_profile(self._h, 1 if enable else 0))

    def profile_read(self):
        """({phase name: total device ms}, profiled steps) since profile()."""
        ms = (ctypes.c_double * len(PHASES))()
        steps = _I32(0)
        check(lib().velo_cuda_profile_read(self._h, ms, len(PHASES), ctypes.byref(steps)))
        return {n: float(ms[i]) for i, n in enumerate(PHASES)}, int(steps.value)

    def tp_sum_path(self):
        """'none', 'nccl', 'peer', 'fused' or 'ce': how the tensor-parallel
        partial sums run."""
        v = _I32(0)
        check(lib().velo_cuda_tp_sum_path(self._h, ctypes.byref(v)))
        return ("none", "nccl", "peer", "fused", "ce")[v.value]

    def verify_step(self, slots, ctx_len, tokens, parents, temperature=0.0, draft_logits=None,
                    uniforms=None, commit=True, want_logits=False, n_vocab=None):
        """One verify step (host buffers).  commit: True (the accepted path),
        False, or "all" (every node of a chain: prefill / draft decode).
        Returns dict(accepted_len, accepted_nodes, bonus, logits)."""
        tok = np.ascontiguousarray(tokens, np.uint32)
        B, N = tok.shape
        par = np.ascontiguousarray(parents, np.int32).reshape(B, N)
        sl = np.ascontiguousarray(slots, np.uint32)
        cl = np.ascontiguousarray(ctx_len, np.int32)
        dl = None if draft_logits is None else np.ascontiguousarray(draft_logits, np.float32)
        un = None if uniforms is None else np.ascontiguousarray(uniforms, np.float32)
        acc = np.zeros(B, np.int32)
        nodes = np.zeros((B, N), np.int32)
        bonus = np.zeros(B, np.uint32)
        logits = np.zeros((B, N, n_vocab), np.float32) if want_logits else None
        cm = 2 if commit == "all" else (1 if commit else 0)
        bt = VerifyBatch(ctypes.sizeof(VerifyBatch), B, N, _ptr(sl), _ptr(cl), _ptr(tok), _ptr(par),
                         float(temperature), _ptr(dl), _ptr(un), cm)
        expected = np.zeros((B, N), np.uint32)
        rs = VerifyResult(_ptr(acc), _ptr(nodes), _ptr(bonus), _ptr(logits), _ptr(expected))
        check(lib().velo_cuda_verify_step(self._h, ctypes.byref(bt), ctypes.byref(rs)))
        return {"accepted_len": acc, "accepted_nodes": nodes, "bonus": bonus, "logits": logits,
                "expected": expected}


def prefill(ctx, slot, tokens, pos0=0, chunk=64, n_vocab=None):
    """Fill `slot`'s pages with the K/V of `tokens` at positions pos0.. by
    chained verify steps that commit every node (chunks of <= 64 tokens).
    Returns the greedy next token after the last one."""
    toks = np.asarray(tokens, np.uint32)
    nxt = None
    for c0 in range(0, len(toks), chunk):
        part = toks[c0:c0 + chunk]
        par = np.arange(-1, len(part) - 1, dtype=np.int32)
        r = ctx.verify_step([slot], [pos0 + c0], part[None], par[None], commit="all",
                            n_vocab=n_vocab)
        nxt = int(r["bonus"][0])
    return nxt


class GgufValue(ctypes.Structure):
    _fields_ = [("type", _I32), ("array_type", _I32), ("u", ctypes.c_uint64), ("i", ctypes.c_int64),
                ("f", ctypes.c_double), ("s", ctypes.POINTER(ctypes.c_char)), ("s_len", ctypes.c_uint64),
                ("array_len", ctypes.c_uint64)]


class GgufTensor(ctypes.Structure):
    _fields_ = [("ggml_type", _I32), ("n_dims", ctypes.c_uint32), ("shape", ctypes.c_uint64 * 4),
                ("offset", ctypes.c_uint64), ("nbytes", ctypes.c_uint64), ("data", _P)]


class GgufModelMeta(ctypes.Structure):
    _fields_ = [("struct_size", ctypes.c_uint32), ("desc", ModelDesc), ("n_ctx", ctypes.c_uint32),
                ("quantization", _I32), ("arch", ctypes.c_char * 64)]


class Gguf:
    """A GGUF file, parsed on the host with its tensor data mapped
    (GgufFile + ModelMeta + WeightStore, src/gguf.rs, src/model_loader.rs)."""

    def __init__(self, path):
        self._h = None
        h = _P()
        check(lib().velo_gguf_open(os.fsencode(path), ctypes.byref(h)))
        self._h = h

    def close(self):
        if self._h:
            lib().velo_gguf_close(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    @property
    def version(self):
        return lib().velo_gguf_version(self._h)

    @property
    def n_tensors(self):
        return lib().velo_gguf_n_tensors(self._h)

    @property
    def n_metadata(self):
        return lib().velo_gguf_n_metadata(self._h)

    @property
    def data_offset(self):
        return lib().velo_gguf_data_offset(self._h)

    @staticmethod
    def _value(v, fetch_elem):
        t = v.type
        if t in (0, 2, 4, 10):
            return ("u", v.u)
        if t == 7:
            return ("bool", bool(v.u))
        if t in (1, 3, 5, 11):
            return ("i", v.i)
        if t in (6, 12):
            return ("f", v.f)
        if t == 8:
            return ("str", ctypes.string_at(v.s, v.s_len).decode())
        return ("array", [fetch_elem(k) for k in range(v.array_len)])

    def metadata(self, key):
        """(type id, python value); VeloError ERR_MISSING_META when absent."""
        v = GgufValue()
        k = key.encode()
        check(lib().velo_gguf_metadata(self._h, k, ctypes.byref(v)))

        def elem(i):
            e = GgufValue()
            check(lib().velo_gguf_metadata_elem(self._h, k, i, ctypes.byref(e)))
            return self._value(e, None)[1]
        return v.type, self._value(v, elem)[1]

    def tensor(self, name):
        """dict(ggml_type, shape, offset, nbytes, data=bytes)."""
        t = GgufTensor()
        check(lib().velo_gguf_tensor_info(self._h, name.encode(), ctypes.byref(t)))
        data = ctypes.string_at(t.data, t.nbytes) if t.data else b""
        return {"ggml_type": t.ggml_type, "shape": [t.shape[d] for d in range(t.n_dims)],
                "offset": t.offset, "nbytes": t.nbytes, "data": data}

    def model_meta(self):
        m = GgufModelMeta()
        m.struct_size = ctypes.sizeof(GgufModelMeta)
        check(lib().velo_gguf_read_model_meta(self._h, ctypes.byref(m)))
        d = m.desc
        return {"arch": m.arch.decode(), "n_vocab": d.n_vocab, "n_embd": d.n_embd, "n_layer": d.n_layer,
                "n_head": d.n_head, "n_head_kv": d.n_head_kv, "n_ff": d.n_ff, "head_dim": d.head_dim,
                "rope_freq_base": d.rope_freq_base, "norm_eps": d.norm_eps, "n_ctx": m.n_ctx,
                "quantization": m.quantization}

    def validate(self):
        check(lib().velo_gguf_validate(self._h))

    def weights(self):
        """[(name, dtype, rows, cols, bytes)] as velo_cuda_load_model takes them."""
        n = _I32()
        check(lib().velo_gguf_weights(self._h, None, 0, ctypes.byref(n)))
        ws = (WeightDesc * n.value)()
        check(lib().velo_gguf_weights(self._h, ws, n.value, ctypes.byref(n)))
        out = []
        for w in ws:
            nb = q4_0_row_bytes(w.cols) * w.rows if w.dtype == 2 else w.rows * w.cols * (4 if w.dtype == 0 else 2)
            out.append((w.name.decode(), w.dtype, w.rows, w.cols, ctypes.string_at(w.data, nb)))
        return out


def q4_0_row_bytes(cols):
    return cols // 32 * 18


class OutOfPages(VeloError):
    """PageManagerError::OutOfPages { requested, available }."""

    def __init__(self, requested, available, message):
        super().__init__(ERR_OUT_OF_PAGES, message)
        self.requested = requested
        self.available = available


class PageAllocator:
    """The KV page allocator without a context or GPU
    (PagedAttentionBlockManager, src/paged_attention.rs:92-211)."""

    def __init__(self, block_size, total_pages):
        self._h = None
        h = _P()
        check(lib().velo_page_allocator_create(block_size, total_pages, ctypes.byref(h)))
        self._h = h

    def close(self):
        if self._h:
            lib().velo_page_allocator_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def pages_for_tokens(self, token_len):
        return lib().velo_page_allocator_pages_for_tokens(self._h, token_len)

    def allocate(self, handle, token_len):
        need = self.pages_for_tokens(token_len)
        pages = np.zeros(max(need, 1), np.uint32)
        n, rq, av = _SZ(), _SZ(), _SZ()
        st = lib().velo_page_allocator_allocate(self._h, handle, token_len, _ptr(pages), pages.size,
                                                ctypes.byref(n), ctypes.byref(rq), ctypes.byref(av))
        if st == ERR_OUT_OF_PAGES:
            raise OutOfPages(rq.value, av.value, last_error())
        check(st)
        return pages[:n.value].copy()

    def release(self, handle):
        check(lib().velo_page_allocator_release(self._h, handle))

    def mapped_pages(self, handle):
        """The handle's pages, or None (mapped_pages returning None)."""
        n = _SZ()
        if lib().velo_page_allocator_mapped_pages(self._h, handle, None, 0, ctypes.byref(n)) == \
                ERR_UNKNOWN_HANDLE:
            return None
        pages = np.zeros(max(n.value, 1), np.uint32)
        check(lib().velo_page_allocator_mapped_pages(self._h, handle, _ptr(pages), pages.size,
                                                     ctypes.byref(n)))
        return pages[:n.value].copy()

    def free_pages(self):
        return lib().velo_page_allocator_free_pages(self._h)


def nccl_unique_id():
    """128-byte NCCL unique id for a tensor-parallel group (rank 0 makes it)."""
    buf = (ctypes.c_char * 128)()
    check(lib().velo_cuda_nccl_unique_id(buf))
    return bytes(buf)


def tp_wait_selftest(device=0):
    """velo_cuda_tp_wait_selftest: the error code the peer-sum kernel records
    when its partner rank never arrives (0x7101), after its bounded waits."""
    code = _I32(0)
    check(lib().velo_cuda_tp_wait_selftest(device, ctypes.byref(code)))
    return int(code.value)


def shard_strategy(name):
    return int(lib().velo_cuda_shard_strategy(name.encode()))


def shard_weight(name, dtype, data, rows, cols, strategy, tp, rank):
    """velo_cuda_shard_weight on a host tensor: returns (bytes, rows, cols)."""
    a = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
    w = WeightDesc(name.encode(), dtype, 0, a.ctypes.data, rows, cols)
    out = np.zeros(a.size, np.uint8)
    r, c = ctypes.c_uint64(), ctypes.c_uint64()
    check(lib().velo_cuda_shard_weight(ctypes.byref(w), strategy, tp, rank, _ptr(out), out.size,
                                       ctypes.byref(r), ctypes.byref(c)))
    rb = cols * 4 if dtype == DT_F32 else cols * 2 if dtype == DT_F16 else cols // 32 * 18
    n = r.value * (rb if strategy != 2 else rb // tp)
    return out[:n], r.value, c.value


def q4_0_repacked_bytes(N, K):
    return int(lib().velo_cuda_q4_0_repacked_bytes(N, K))


def accept_static(target_logits, draft_logits, draft_tokens, uniforms, temperature,
                  accepted_len, bonus_token, stream_ptr=None):
    """velo_cuda_accept_static on torch CUDA tensors: no context and no device
    allocation; asynchronous on `stream_ptr` (None: the default stream)."""
    B, k1, V = target_logits.shape
    check(lib().velo_cuda_accept_static(
        _ptr(target_logits), _ptr(draft_logits), _ptr(draft_tokens), _ptr(uniforms), B, k1 - 1,
        V, float(temperature), _ptr(accepted_len), _ptr(bonus_token),
        _P(stream_ptr) if stream_ptr else None))


def accept_static_error(flag_out, stream_ptr=None):
    """velo_cuda_accept_static_error: the last static call's input check into
    flag_out (a one-element int32 CUDA tensor), asynchronously on stream_ptr."""
    check(lib().velo_cuda_accept_static_error(_ptr(flag_out), _P(stream_ptr) if stream_ptr else None))
