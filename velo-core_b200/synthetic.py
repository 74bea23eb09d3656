"""Seeded synthetic inputs for the verify-step workloads.

No public dataset is involved: every config is defined by shapes and value
distributions, generated here from numpy's Philox bit generator with seed 0
(one independent stream per tensor, `stream` below), so that the CUDA path and
the CPU oracle consume the same bytes.
"""
import numpy as np


def rng(seed=0, stream=0):
    """Philox counter-based generator; `stream` selects an independent key."""
    return np.random.Generator(np.random.Philox(key=seed * 1000003 + stream))


def softmax64(x, axis=-1):
    x = x.astype(np.float64)
    x = x - x.max(axis=axis, keepdims=True)
    e = np.exp(x)
    return e / e.sum(axis=axis, keepdims=True)


def acceptance_inputs(B=64, k=8, V=32000, temperature=0.8, seed=0, target_sigma=2.0,
                      draft_sigma=0.5):
    """Acceptance microbench.

    target logits ~ N(0, target_sigma^2)            [B][k+1][V] f32
    draft logits  = target rows 0..k-1 + N(0, draft_sigma^2)   [B][k][V] f32
    draft tokens  sampled from q = softmax(draft/T) (stream seed+1)
    uniforms      U(0,1): one per draft position + one residual draw [B][k+1]
    """
    tgt = rng(seed, 0).normal(0.0, target_sigma, (B, k + 1, V)).astype(np.float32)
    drf = (tgt[:, :k] + rng(seed, 1).normal(0.0, draft_sigma, (B, k, V))).astype(np.float32)
    g = rng(seed + 1, 2)
    tok = np.zeros((B, k), np.uint32)
    T = temperature if temperature > 0 else 1.0
    for b in range(B):
        q = softmax64(drf[b] / T)
        c = np.cumsum(q, axis=-1)
        uu = g.random(k)
        tok[b] = np.minimum((c < uu[:, None]).sum(-1), V - 1)
    u = rng(seed, 3).random((B, k + 1)).astype(np.float32)
    return tgt, drf, tok, u


def quantize_q4_0(x):
    """[rows][cols] float32 -> [rows][cols/32*18] uint8 q4_0 in velo-core's
    interleaved order (src/quant.rs:50-64: byte i of a block holds element 2i
    in the low nibble and 2i+1 in the high nibble).  Per 32-block: m = the
    element of largest magnitude, d = m / -8 (f32, stored as f16),
    q = clamp(trunc(x * (1/d) + 8.5), 0, 15) in f32 arithmetic."""
    x = np.ascontiguousarray(x, np.float32)
    rows, cols = x.shape
    assert cols % 32 == 0
    xb = x.reshape(rows, cols // 32, 32)
    idx = np.abs(xb).argmax(axis=-1)
    m = np.take_along_axis(xb, idx[..., None], axis=-1)[..., 0]
    d = (m / np.float32(-8.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    qf = (xb * inv[..., None]).astype(np.float32) + np.float32(8.5)
    q = np.clip(np.trunc(qf), 0, 15).astype(np.uint8)
    out = np.zeros((rows, cols // 32, 18), np.uint8)
    out[..., 0:2] = d.astype(np.float16).view(np.uint8).reshape(rows, cols // 32, 2)
    out[..., 2:] = q[..., 0::2] | (q[..., 1::2] << 4)
    return out.reshape(rows, cols // 32 * 18)


def dequant_q4_0_f16(data, rows, cols):
    """The f16 weights the tensor-core GEMM multiplies: f16(d * (q - 8)),
    one rounding of the exact product."""
    blk = np.ascontiguousarray(data, np.uint8).reshape(rows, cols // 32, 18)
    d = blk[..., 0:2].copy().view(np.float16)[..., 0].astype(np.float32)
    q = np.empty((rows, cols // 32, 32), np.float32)
    q[..., 0::2] = (blk[..., 2:] & 15).astype(np.float32) - 8
    q[..., 1::2] = (blk[..., 2:] >> 4).astype(np.float32) - 8
    return (d[..., None] * q).astype(np.float16).reshape(rows, cols)


def random_q4_0(rows, cols, seed=0, stream=10, sigma=0.02):
    """q4_0 bytes [rows][cols/32*18] drawn directly in the quantised domain:
    uniform random nibbles (q - 8 has standard deviation ~4.6) and per-block
    f16 scales d = sigma / 4.6 * U(0.5, 1.5), so weights have standard
    deviation ~sigma.  Generating the bytes takes a fraction of the time of
    drawing and quantising normals at the 70B shapes."""
    assert cols % 32 == 0
    g = rng(seed, stream)
    nb = cols // 32
    out = np.frombuffer(g.bytes(rows * nb * 18), np.uint8).reshape(rows, nb, 18).copy()
    d = (sigma / 4.6 * g.uniform(0.5, 1.5, (rows, nb))).astype(np.float16)
    out[..., 0:2] = d.view(np.uint8).reshape(rows, nb, 2)
    return out.reshape(rows, nb * 18)


def dequant_q4_0_f32(data, rows, cols):
    """f32 weights of q4_0 bytes as the reference dequantises them
    (src/quant.rs:50-73: f16 scale widened to f32, times q - 8; the product is
    exact in f32)."""
    blk = np.ascontiguousarray(data, np.uint8).reshape(rows, cols // 32, 18)
    d = blk[..., 0:2].copy().view(np.float16)[..., 0].astype(np.float32)
    q = np.empty((rows, cols // 32, 32), np.float32)
    q[..., 0::2] = (blk[..., 2:] & 15).astype(np.float32) - 8
    q[..., 1::2] = (blk[..., 2:] >> 4).astype(np.float32) - 8
    return (d[..., None] * q).reshape(rows, cols)


def llama_random_q4_model(n_vocab, n_embd, n_layer, n_head, n_head_kv, n_ff, seed=0, sigma=0.02,
                          norm_sigma=0.1, rope_freq_base=10000.0):
    """A Llama model of the given shape with q4_0 matrices and embedding from
    random_q4_0 (fast at the 7B / 70B layer shapes) and f32 norm weights
    1 + N(0, norm_sigma^2); head_dim 128.  Same return as llama_model."""
    hd = 128
    meta = dict(n_vocab=n_vocab, n_embd=n_embd, n_layer=n_layer, n_head=n_head,
                n_head_kv=n_head_kv, n_ff=n_ff, head_dim=hd, rope_freq_base=rope_freq_base,
                norm_eps=1e-5)
    g = rng(seed, 51)
    st = [100]

    def mat(rows, cols):
        st[0] += 1
        return (2, random_q4_0(rows, cols, seed, st[0], sigma), rows, cols)

    def norm():
        return (0, (1.0 + g.normal(0, norm_sigma, n_embd)).astype(np.float32), 1, n_embd)

    t = {"token_embd.weight": mat(n_vocab, n_embd), "output_norm.weight": norm(),
         "output.weight": mat(n_vocab, n_embd)}
    for l in range(n_layer):
        p = f"layers.{l}."
        t[p + "attention_norm.weight"] = norm()
        t[p + "attention.wq.weight"] = mat(n_head * hd, n_embd)
        t[p + "attention.wk.weight"] = mat(n_head_kv * hd, n_embd)
        t[p + "attention.wv.weight"] = mat(n_head_kv * hd, n_embd)
        t[p + "attention.wo.weight"] = mat(n_embd, n_head * hd)
        t[p + "ffn_norm.weight"] = norm()
        t[p + "feed_forward.w1.weight"] = mat(n_ff, n_embd)
        t[p + "feed_forward.w2.weight"] = mat(n_embd, n_ff)
        t[p + "feed_forward.w3.weight"] = mat(n_ff, n_embd)
    return meta, t


def q4_0_weights(rows, cols, sigma=0.02, seed=0, stream=10):
    """Random-init weight N(0, sigma^2), quantised to q4_0."""
    w = rng(seed, stream).normal(0.0, sigma, (rows, cols)).astype(np.float32)
    return quantize_q4_0(w)


def quantize_kv_int8(x):
    """Per-row int8 quantisation of K/V rows [..., head_dim] (the reference's
    kv_update_int8 rule, src/kernels.metal:783-801, with an fp16 scale):
    scale = max|x| / 127, q = trunc(x * (127 / max|x|)), in f32 arithmetic.
    Returns (int8 values, f16 scales [...])."""
    x = np.ascontiguousarray(x, np.float32)
    mx = np.abs(x).max(axis=-1)
    sc = (mx / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(mx > 0, np.float32(127.0) / mx, np.float32(0.0)).astype(np.float32)
    q = np.trunc((x * inv[..., None]).astype(np.float32)).astype(np.int8)
    return q, sc.astype(np.float16)


def random_tree(n_nodes, max_depth, g):
    """Parents of a random draft tree: node 0 is the root (-1); node n picks a
    parent uniformly among earlier nodes of depth < max_depth."""
    parents = np.full(n_nodes, -1, np.int32)
    depth = np.zeros(n_nodes, np.int32)
    for n in range(1, n_nodes):
        cand = np.nonzero(depth[:n] < max_depth - 1)[0]
        p = int(cand[g.integers(0, len(cand))])
        parents[n] = p
        depth[n] = depth[p] + 1
    return parents


def tree_attention_inputs(B, n_nodes, n_head, n_kv, ctx_lens, kv_dtype=0, seed=0, max_depth=6,
                          head_dim=128, page=16, spare_pages=3):
    """Paged tree-attention inputs (BASELINE config 4 distributions): K/V and
    queries ~ N(0,1); pages of all sequences are a random permutation of the
    pool; int8 pools hold trunc-quantised values with f16 per-token scales.
    Returns a dict of numpy arrays in the layouts of velo_cuda_tree_attention."""
    ctx_lens = np.asarray(ctx_lens, np.int32)
    npages = [(int(c) + page - 1) // page for c in ctx_lens]
    max_pages = max(1, max(npages))
    total = sum(npages) + spare_pages
    perm = rng(seed, 30).permutation(total).astype(np.uint32)
    page_table = np.zeros((B, max_pages), np.uint32)
    off = 0
    for b in range(B):
        page_table[b, :npages[b]] = perm[off:off + npages[b]]
        off += npages[b]
    kv = rng(seed, 31).normal(0, 1, (2, total, n_kv, page, head_dim)).astype(np.float32)
    out = {"page_table": page_table, "ctx_len": ctx_lens, "kv_dtype": kv_dtype}
    if kv_dtype == 0:
        out["k_pool"] = kv[0].astype(np.float16)
        out["v_pool"] = kv[1].astype(np.float16)
        out["k_scale"] = out["v_scale"] = None
    else:
        out["k_pool"], out["k_scale"] = quantize_kv_int8(kv[0])
        out["v_pool"], out["v_scale"] = quantize_kv_int8(kv[1])
    out["q"] = rng(seed, 32).normal(0, 1, (B, n_nodes, n_head, head_dim)).astype(np.float16)
    out["node_k"] = rng(seed, 33).normal(0, 1, (B, n_nodes, n_kv, head_dim)).astype(np.float16)
    out["node_v"] = rng(seed, 34).normal(0, 1, (B, n_nodes, n_kv, head_dim)).astype(np.float16)
    g = rng(seed, 35)
    out["parents"] = np.stack([random_tree(n_nodes, max_depth, g) for _ in range(B)])
    return out


LAYER_TENSORS = ("attention_norm", "attention.wq", "attention.wk", "attention.wv", "attention.wo",
                 "ffn_norm", "feed_forward.w1", "feed_forward.w2", "feed_forward.w3")


def llama_model(n_vocab, n_embd, n_layer, n_head, n_head_kv, n_ff, seed=0, sigma=0.02,
                tied=False, dtype=2, head_dim=128, norm_sigma=0.1):
    """Random-init Llama weights in the reference's WeightStore layout
    (src/model_loader.rs:216-232; matrices [out][in]): matrices and embedding
    from N(0, sigma^2) as q4_0 (dtype 2) or f32 (dtype 0), f32 norm weights
    1 + N(0, norm_sigma^2).  Returns (meta, {name: (dtype, array, rows, cols)})."""
    hd = head_dim
    meta = dict(n_vocab=n_vocab, n_embd=n_embd, n_layer=n_layer, n_head=n_head,
                n_head_kv=n_head_kv, n_ff=n_ff, head_dim=hd, rope_freq_base=10000.0,
                norm_eps=1e-5)
    g = rng(seed, 50)

    def mat(rows, cols):
        w = g.normal(0, sigma, (rows, cols)).astype(np.float32)
        return (2, quantize_q4_0(w), rows, cols) if dtype == 2 else (0, w, rows, cols)

    def norm():
        w = np.ones(n_embd, np.float32)
        if norm_sigma:
            w = (1.0 + g.normal(0, norm_sigma, n_embd)).astype(np.float32)
        return (0, w, 1, n_embd)

    t = {"token_embd.weight": mat(n_vocab, n_embd), "output_norm.weight": norm()}
    if not tied:
        t["output.weight"] = mat(n_vocab, n_embd)
    for l in range(n_layer):
        p = f"layers.{l}."
        t[p + "attention_norm.weight"] = norm()
        t[p + "attention.wq.weight"] = mat(n_head * hd, n_embd)
        t[p + "attention.wk.weight"] = mat(n_head_kv * hd, n_embd)
        t[p + "attention.wv.weight"] = mat(n_head_kv * hd, n_embd)
        t[p + "attention.wo.weight"] = mat(n_embd, n_head * hd)
        t[p + "ffn_norm.weight"] = norm()
        t[p + "feed_forward.w1.weight"] = mat(n_ff, n_embd)
        t[p + "feed_forward.w2.weight"] = mat(n_embd, n_ff)
        t[p + "feed_forward.w3.weight"] = mat(n_ff, n_embd)
    return meta, t


def llama_q4_model(n_vocab, n_embd, n_layer, n_head, n_head_kv, n_ff, seed=0, sigma=0.02,
                   tied=False):
    """q4_0 weights, head_dim 128 (the tensor-core path)."""
    return llama_model(n_vocab, n_embd, n_layer, n_head, n_head_kv, n_ff, seed, sigma, tied)


def c1_pair(seed=0):
    """The CPU-runnable tiny fp32 Llama pair: target 2 layers, hidden 256,
    4 heads x 64, SwiGLU FFN 688, vocab 4096, RMSNorm eps 1e-5, RoPE theta 1e4;
    draft 1 layer of the same dims.  Weights N(0, 0.02^2) f32, norm weights 1,
    both from `seed` (so the draft shares the target's embedding, LM head and
    first layer).  Returns (target_meta, target_tensors, draft_meta, draft_tensors)."""
    kw = dict(n_vocab=4096, n_embd=256, n_head=4, n_head_kv=4, n_ff=688, sigma=0.02, dtype=0,
              head_dim=64, norm_sigma=0.0, seed=seed)
    tm, tw = llama_model(n_layer=2, **kw)
    dm, dw = llama_model(n_layer=1, **kw)
    return tm, tw, dm, dw


def oracle_tensor_list(meta, tensors):
    """The same tensors in the CPU oracle's order (token_embd, output_norm,
    output|None, then per layer attention_norm, wq, wk, wv, wo, ffn_norm, w1,
    w2, w3) as (dtype, array)."""
    out = [tensors["token_embd.weight"][:2], tensors["output_norm.weight"][:2],
           tensors["output.weight"][:2] if "output.weight" in tensors else None]
    for l in range(meta["n_layer"]):
        for nm in LAYER_TENSORS:
            out.append(tensors[f"layers.{l}.{nm}.weight"][:2])
    return out
