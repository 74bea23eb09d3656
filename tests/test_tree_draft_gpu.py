"""Tree drafts on the device (TreeDraftModel::draft_tree, backend.rs:255-294,
with TopKSampler) and whole-tree verification (TargetModel::verify_tree,
speculative.rs:217-242) against the CPU oracle on the tiny fp32 pair: the same
trees, the same expected token after every node, the same best path and bonus,
and the same contexts over several draft / verify / commit rounds."""
import numpy as np
import pytest

import synthetic
import velo_cuda
import vo
from speculative import CudaTreeDraft, SpeculativeTree, rooted_tree, top_k, verify_tree_on_device

pytestmark = pytest.mark.gpu


class OracleTreeDraft:
    """draft_tree over the oracle model (forward_one per node), same sampler."""

    def __init__(self, model):
        self.m, self.tokens = model, []

    def _decode(self, token):
        lg = self.m.forward_one(int(token), len(self.tokens))
        self.tokens.append(int(token))
        return lg

    def draft_tree(self, context, max_tokens, width):
        common = 0
        for a, b in zip(self.tokens, context[:-1]):
            if a != b:
                break
            common += 1
        self.tokens = self.tokens[:common]
        for i in range(common, len(context) - 1):
            self._decode(context[i])
        top = top_k(self._decode(context[-1]), width)
        tree = SpeculativeTree(top[0].token)
        for pred in top[1:]:
            tree.add_child(0, pred.token)
        curr = 0
        for _ in range(1, max_tokens):
            curr = tree.add_child(curr, top_k(self._decode(tree.tokens[curr]), 1)[0].token)
        return tree


def _ctx():
    return velo_cuda.Context(device=0, kv_dtype=velo_cuda.KV_F32, total_pages=16, max_slots=1,
                             max_pages_per_slot=16)


def test_tree_draft_verify_rounds_match_oracle():
    tm, tw, dm, dw = synthetic.c1_pair()
    V = tm["n_vocab"]
    context = [int(t) for t in synthetic.rng(0, 93).integers(0, V, 40)]
    ora_t = vo.Model(dict(tm, n_ctx=512), synthetic.oracle_tensor_list(tm, tw))
    ora_d = OracleTreeDraft(vo.Model(dict(dm, n_ctx=512), synthetic.oracle_tensor_list(dm, dw)))
    ora_t.forward_sequence(np.array(context[:-1], np.uint32))
    ref_ctx = list(context)
    with _ctx() as tctx, _ctx() as dctx:
        tctx.load_model(tm, tw)
        dctx.load_model(dm, dw)
        tctx.bind_slot(0, np.arange(16))
        dctx.bind_slot(0, np.arange(16))
        velo_cuda.prefill(tctx, 0, context[:-1], n_vocab=V)
        draft = CudaTreeDraft(dctx, 0, V)
        for _ in range(6):
            tree = draft.draft_tree(context, 4, 3)
            rtree = ora_d.draft_tree(ref_ctx, 4, 3)
            assert tree.tokens == rtree.tokens and tree.parents == rtree.parents
            rt, res, r = verify_tree_on_device(tctx, 0, V, context, tree, commit=True)
            # oracle: logits of every node of the rooted tree, greedy, best path
            ort = rooted_tree(ref_ctx, rtree)
            par = np.array([-1] + ort.parents[1:], np.int32)
            lg = ora_t.verify_tree(np.array(ort.tokens, np.uint32), par, len(ref_ctx) - 1)
            exp = [vo.greedy(lg[i])[0] for i in range(len(ort.tokens))]
            assert res.expected == exp
            path, bonus = rt.find_best_path(res.expected)
            nodes = [int(i) for i in r["accepted_nodes"][0] if i >= 0]
            assert [rt.tokens[i] for i in nodes] == path and int(r["bonus"][0]) == bonus
            rpath = vo.find_best_path(par, np.array(ort.tokens, np.uint32), np.array(exp, np.uint32))[0]
            ora_t.commit_path(list(rpath), len(ref_ctx) - 1)
            context = context + path[1:] + [bonus]
            ref_ctx = ref_ctx + path[1:] + [bonus]
            assert context == ref_ctx
