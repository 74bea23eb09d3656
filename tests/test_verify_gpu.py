"""The full verify step (velo_cuda_verify_step) against the CPU oracle of the
reference's forward (oracle vo_verify_tree: llama_cpu.rs forward_one with the
tree contract, q4_0 weights dequantised as quant.rs).

- logits of every draft-tree node within 2e-2 max-abs (the q4_0/f16 bar);
- accept decisions, accepted paths and bonus tokens bit-exact against the
  oracle's GreedySampler + find_best_path (or the rejection-sampling rule)
  applied to the same (GPU) logits;
- the committed K/V of the accepted path land at positions ctx_len.. of the
  slot's pages (compared with the oracle's committed cache, f16 tolerance)."""
import numpy as np
import pytest

import synthetic
import velo_cuda
import vo

pytestmark = pytest.mark.gpu

TOL_LOGITS = 2e-2


def _setup(meta, tensors, prompt, slot, pages_total=96, max_slots=3, max_pages=40, seed=0):
    ora = vo.Model(dict(meta, n_ctx=1024), synthetic.oracle_tensor_list(meta, tensors))
    ora.forward_sequence(prompt)
    ctx = velo_cuda.Context(device=0, total_pages=pages_total, max_slots=max_slots,
                            max_pages_per_slot=max_pages)
    ctx.load_model(meta, tensors)
    pages = synthetic.rng(seed, 60).permutation(pages_total)[:max_pages].astype(np.uint32)
    ctx.bind_slot(slot, pages)
    P = len(prompt)
    Hkv = meta["n_head_kv"]
    for l in range(meta["n_layer"]):
        K = ora.read_kv(0, l, P).reshape(P, Hkv, 128).astype(np.float16)
        V = ora.read_kv(1, l, P).reshape(P, Hkv, 128).astype(np.float16)
        for p0 in range(0, P, 64):
            ctx.write_kv(slot, l, p0, K[p0:p0 + 64], V[p0:p0 + 64])
    return ora, ctx


def _grow_tree(ora, P, parents, V, g, p_follow=0.7):
    """Node tokens: with probability p_follow a child takes the target's argmax
    after its parent (so some drafts are accepted), else a random token."""
    N = len(parents)
    tokens = g.integers(0, V, N).astype(np.uint32)
    for n in range(1, N):
        if g.random() < p_follow:
            lg = ora.verify_tree(tokens[:n], parents[:n], P)
            tokens[n] = vo.greedy(lg[parents[n]])[0]
    return tokens


@pytest.mark.parametrize("shape", [
    dict(n_vocab=512, n_embd=256, n_layer=2, n_head=2, n_head_kv=1, n_ff=512),
    dict(n_vocab=1000, n_embd=512, n_layer=3, n_head=4, n_head_kv=2, n_ff=1408)])
def test_verify_tree_logits_decisions_commit(shape):
    meta, tensors = synthetic.llama_q4_model(**shape, seed=1)
    g = synthetic.rng(2, 61)
    P = 70
    prompt = g.integers(0, meta["n_vocab"], P).astype(np.uint32)
    ora, ctx = _setup(meta, tensors, prompt, slot=1)
    try:
        N = 12
        parents = synthetic.random_tree(N, 5, g)
        tokens = _grow_tree(ora, P, parents, meta["n_vocab"], g)
        ref = ora.verify_tree(tokens, parents, P)
        res = ctx.verify_step([1], [P], tokens[None], parents[None], commit=True,
                              want_logits=True, n_vocab=meta["n_vocab"])
        got = res["logits"][0]
        assert np.abs(got - ref).max() <= TOL_LOGITS, np.abs(got - ref).max()
        # decisions on the same logits: bit-exact
        expected = np.array([vo.greedy(got[n])[0] for n in range(N)], np.uint32)
        path, bonus = vo.find_best_path(parents, tokens, expected)
        n_path = len(path)
        assert res["accepted_len"][0] == n_path - 1
        assert list(res["accepted_nodes"][0][:n_path]) == list(path)
        assert all(res["accepted_nodes"][0][n_path:] == -1)
        assert res["bonus"][0] == bonus
        # commit: the path's K/V now sit at positions P .. P + n_path - 1
        ora.commit_path(path, P)
        Hkv = meta["n_head_kv"]
        for l in range(meta["n_layer"]):
            k, v = ctx.read_kv(1, l, P, n_path, Hkv)
            rk = ora.read_kv(0, l, P + n_path)[P:].reshape(n_path, Hkv, 128)
            rv = ora.read_kv(1, l, P + n_path)[P:].reshape(n_path, Hkv, 128)
            assert np.abs(k.astype(np.float32) - rk).max() <= 2e-2
            assert np.abs(v.astype(np.float32) - rv).max() <= 2e-2
        # the cache written before the step is untouched
        k, _ = ctx.read_kv(1, 0, 0, 8, Hkv)
        assert np.array_equal(k, ora.read_kv(0, 0, 8).reshape(8, Hkv, 128).astype(np.float16))
    finally:
        ctx.close()


def test_verify_batch_of_sequences_and_sampling_chain():
    shape = dict(n_vocab=512, n_embd=256, n_layer=2, n_head=2, n_head_kv=2, n_ff=512)
    meta, tensors = synthetic.llama_q4_model(**shape, seed=3)
    g = synthetic.rng(4, 62)
    V = meta["n_vocab"]
    ctx = velo_cuda.Context(device=0, total_pages=64, max_slots=4, max_pages_per_slot=16)
    try:
        ctx.load_model(meta, tensors)
        ctx.bind_slot(0, np.arange(0, 16))
        ctx.bind_slot(2, np.arange(16, 32))
        ctx.bind_slot(3, np.arange(32, 48))
        # empty caches: ctx_len 0, a chain of k = 5 drafts each
        B, N = 3, 6
        tokens = g.integers(0, V, (B, N)).astype(np.uint32)
        parents = np.tile(np.arange(-1, N - 1, dtype=np.int32), (B, 1))
        res = ctx.verify_step([0, 2, 3], [0, 0, 0], tokens, parents, commit=False,
                              want_logits=True, n_vocab=V)
        for b in range(B):
            ora = vo.Model(dict(meta, n_ctx=256), synthetic.oracle_tensor_list(meta, tensors))
            ref = ora.verify_tree(tokens[b], parents[b], 0)
            assert np.abs(res["logits"][b] - ref).max() <= TOL_LOGITS
        # sampling on chains: same decisions as the acceptance spec on the same logits
        lg = res["logits"]
        drf = (lg[:, :N - 1] + g.normal(0, 0.5, (B, N - 1, V))).astype(np.float32)
        u = g.random((B, N)).astype(np.float32)
        res2 = ctx.verify_step([0, 2, 3], [0, 0, 0], tokens, parents, temperature=0.9,
                               draft_logits=drf, uniforms=u, commit=True, n_vocab=V)
        ra, rb = vo.accept(lg, drf, tokens[:, 1:], u, 0.9)
        assert np.array_equal(res2["accepted_len"], ra)
        assert np.array_equal(res2["bonus"], rb)
    finally:
        ctx.close()


def test_verify_errors_mirror_reference():
    shape = dict(n_vocab=512, n_embd=256, n_layer=1, n_head=2, n_head_kv=1, n_ff=512)
    meta, tensors = synthetic.llama_q4_model(**shape, seed=5)
    ctx = velo_cuda.Context(device=0, total_pages=8, max_slots=1, max_pages_per_slot=2)
    try:
        ctx.load_model(meta, tensors)
        with pytest.raises(velo_cuda.VeloError) as e:
            ctx.bind_slot(0, np.arange(3))  # row holds 2 pages
        assert e.value.status == velo_cuda.ERR_OUT_OF_PAGES
        ctx.bind_slot(0, [5, 6])
        tok = np.zeros((1, 4), np.uint32)
        par = np.array([[-1, 0, 1, 2]], np.int32)
        with pytest.raises(velo_cuda.VeloError) as e:  # position 31 + 3 > 32 tokens
            ctx.verify_step([0], [31], tok, par, commit=True, n_vocab=512)
        assert e.value.status == velo_cuda.ERR_OUT_OF_PAGES
        with pytest.raises(velo_cuda.VeloError) as e:
            ctx.verify_step([0], [0], np.zeros((1, 0), np.uint32), np.zeros((1, 0), np.int32))
        assert e.value.status == velo_cuda.ERR_EMPTY_DRAFT_WINDOW
    finally:
        ctx.close()


@pytest.mark.parametrize("int8", [False, True])
def test_write_kv_matches_oracle_commit_bit_exact(int8):
    """KV write / commit through the page table (kv_update_int8 semantics for
    INT8) equals the oracle's vo_kv_commit byte for byte."""
    shape = dict(n_vocab=512, n_embd=256, n_layer=2, n_head=2, n_head_kv=2, n_ff=512)
    meta, tensors = synthetic.llama_q4_model(**shape, seed=6)
    ctx = velo_cuda.Context(device=0, total_pages=16, max_slots=2, max_pages_per_slot=8,
                            kv_dtype=velo_cuda.KV_INT8 if int8 else velo_cuda.KV_F16)
    try:
        ctx.load_model(meta, tensors)
        pages = np.array([9, 3, 12, 0, 7, 1, 14, 5], np.uint32)
        ctx.bind_slot(1, pages)
        g = synthetic.rng(7, 63)
        n, pos0, Hkv = 40, 13, 2
        k = g.normal(0, 1, (n, Hkv, 128)).astype(np.float16)
        v = g.normal(0, 1, (n, Hkv, 128)).astype(np.float16)
        ctx.write_kv(1, 1, pos0, k, v)
        got = ctx.read_kv(1, 1, pos0, n, Hkv, int8=int8)
        # oracle: commit the same rows through the same page table into its pool
        kvd = vo.KV_I8 if int8 else vo.KV_F16
        dt = np.int8 if int8 else np.uint16
        for which, src in ((0, k), (1, v)):
            pool = np.zeros((16, Hkv, 16, 128), dt)
            scale = np.zeros((16, Hkv, 16), np.uint16)
            rc = vo.kv_commit(kvd, pool, scale, pages, 8, pos0, src.view(np.uint16),
                              np.arange(n, dtype=np.int32), Hkv, 128, 16)
            assert rc == 0
            for i in range(n):
                p = pos0 + i
                pg, sl = pages[p // 16], p % 16
                ref = pool[pg, :, sl]
                out = got[which][i]
                assert np.array_equal(out.view(dt), ref), (which, i)
                if int8:
                    assert np.array_equal(got[2 + which][i], scale[pg, :, sl])
    finally:
        ctx.close()


def test_prefill_and_decode_through_the_step_match_oracle():
    """Prefill by chained steps that commit every node (chunks of 64) and greedy
    decoding one token per step (the draft model's loop) reproduce the oracle's
    forward_sequence / forward_one: same next tokens, cache within f16 rounding."""
    shape = dict(n_vocab=512, n_embd=256, n_layer=2, n_head=2, n_head_kv=1, n_ff=512)
    meta, tensors = synthetic.llama_q4_model(**shape, seed=31)
    g = synthetic.rng(32, 90)
    P = 150
    prompt = g.integers(0, meta["n_vocab"], P).astype(np.uint32)
    ora = vo.Model(dict(meta, n_ctx=512), synthetic.oracle_tensor_list(meta, tensors))
    lg = ora.forward_sequence(prompt)
    ctx = velo_cuda.Context(device=0, total_pages=32, max_slots=1, max_pages_per_slot=16)
    try:
        ctx.load_model(meta, tensors)
        ctx.bind_slot(0, np.arange(16)[::-1].copy())
        nxt = velo_cuda.prefill(ctx, 0, prompt, n_vocab=meta["n_vocab"])
        k, _ = ctx.read_kv(0, 1, 0, P, 1)
        assert np.abs(k.astype(np.float32) - ora.read_kv(0, 1, P).reshape(P, 1, 128)).max() <= 2e-2
        # greedy decode 8 tokens: GPU step on its own last token vs oracle forward_one
        ref_tok = vo.greedy(lg)[0]
        pos = P
        agree = 0
        for _ in range(8):
            r = ctx.verify_step([0], [pos], np.array([[nxt]], np.uint32), np.array([[-1]], np.int32),
                                commit="all", want_logits=True, n_vocab=meta["n_vocab"])
            ref = ora.forward_one(int(nxt), pos)
            assert np.abs(r["logits"][0, 0] - ref).max() <= 2e-2
            agree += int(nxt == ref_tok)
            ref_tok = vo.greedy(ref)[0]
            nxt = int(r["bonus"][0])
            assert nxt == vo.greedy(r["logits"][0, 0])[0]
            pos += 1
        assert agree >= 1
    finally:
        ctx.close()


def test_device_tensors_load_like_host():
    """Weights handed over as device tensors (VELO_WEIGHT_DEVICE, here also
    flagged as this rank's shards) give the same repacked model as host
    tensors: identical logits and decisions."""
    import torch
    meta, tensors = synthetic.llama_q4_model(512, 256, 2, 2, 1, 512, seed=5)
    dev = {k: (dt, torch.from_numpy(np.ascontiguousarray(a)).cuda(), r, c)
           for k, (dt, a, r, c) in tensors.items()}
    tokens = np.array([[7, 300, 41, 9]], np.uint32)
    parents = np.array([[-1, 0, 1, 1]], np.int32)
    out = []
    for src, shards in ((tensors, False), (dev, True)):
        with velo_cuda.Context(device=0, total_pages=8, max_slots=1, max_pages_per_slot=8) as ctx:
            ctx.load_model(meta, src, shards=shards)
            ctx.bind_slot(0, np.arange(8))
            velo_cuda.prefill(ctx, 0, [3, 1, 4, 1, 5, 9, 2, 6], n_vocab=512)
            out.append(ctx.verify_step([0], [8], tokens, parents, commit=False, want_logits=True,
                                       n_vocab=512))
    assert np.array_equal(out[0]["logits"], out[1]["logits"])
    assert np.array_equal(out[0]["accepted_len"], out[1]["accepted_len"])
    assert np.array_equal(out[0]["bonus"], out[1]["bonus"])


def test_slot_allocator_binds_pages():
    """velo_cuda_slot_allocate takes FIFO pages from the context's pool and
    binds them: two slots filled with the same prompt through allocated pages
    hold the same cache and predict the same token; release returns the pages
    (src/paged_attention.rs:155-198)."""
    shape = dict(n_vocab=512, n_embd=256, n_layer=2, n_head=2, n_head_kv=2, n_ff=512)
    meta, tensors = synthetic.llama_q4_model(**shape, seed=8)
    g = synthetic.rng(9, 62)
    prompt = g.integers(0, meta["n_vocab"], 40).astype(np.uint32)
    ctx = velo_cuda.Context(device=0, total_pages=8, max_slots=2, max_pages_per_slot=4)
    try:
        ctx.load_model(meta, tensors)
        assert ctx.free_pages() == 8
        assert list(ctx.slot_allocate(0, 40)) == [0, 1, 2]
        assert list(ctx.slot_allocate(1, 40)) == [3, 4, 5]
        assert ctx.free_pages() == 2
        t0 = velo_cuda.prefill(ctx, 0, prompt, n_vocab=meta["n_vocab"])
        t1 = velo_cuda.prefill(ctx, 1, prompt, n_vocab=meta["n_vocab"])
        assert t0 == t1
        for l in range(meta["n_layer"]):
            k0, v0 = ctx.read_kv(0, l, 0, 40, 2)
            k1, v1 = ctx.read_kv(1, l, 0, 40, 2)
            assert np.array_equal(k0, k1) and np.array_equal(v0, v1)
        ctx.slot_release(0)
        assert ctx.free_pages() == 5
        with pytest.raises(velo_cuda.VeloError) as e:
            ctx.slot_release(0)
        assert e.value.status == velo_cuda.ERR_UNKNOWN_HANDLE
        with pytest.raises(velo_cuda.VeloError) as e:
            ctx.slot_allocate(0, 4 * 16 + 1)  # five pages: more than a page-table row
        assert e.value.status == velo_cuda.ERR_OUT_OF_PAGES
        assert ctx.free_pages() == 5
        assert list(ctx.slot_allocate(0, 64)) == [6, 7, 0, 1]
        assert ctx.free_pages() == 1
    finally:
        ctx.close()


def test_load_gguf_matches_load_model(tmp_path):
    """velo_cuda_load_gguf (load_gguf, src/model_loader.rs:291-309, then the
    upload) gives the step the same model as velo_cuda_load_model on the same
    tensors: identical logits."""
    import gguf_writer
    shape = dict(n_vocab=512, n_embd=256, n_layer=2, n_head=2, n_head_kv=1, n_ff=512)
    meta, tensors = synthetic.llama_q4_model(**shape, seed=12)
    path = tmp_path / "model.gguf"
    gguf_writer.write_model(path, meta, tensors)
    g = synthetic.rng(13, 62)
    tokens = g.integers(0, meta["n_vocab"], (1, 8)).astype(np.uint32)
    parents = np.arange(-1, 7, dtype=np.int32)[None]
    out = []
    for via_file in (False, True):
        ctx = velo_cuda.Context(device=0, total_pages=4, max_slots=1, max_pages_per_slot=4)
        try:
            if via_file:
                ctx.load_gguf(path)
            else:
                ctx.load_model(meta, tensors)
            ctx.bind_slot(0, [0, 1, 2, 3])
            out.append(ctx.verify_step([0], [0], tokens, parents, commit=False, want_logits=True,
                                       n_vocab=meta["n_vocab"])["logits"])
        finally:
            ctx.close()
    assert np.array_equal(out[0], out[1])
