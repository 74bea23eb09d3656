"""The speculative-decoding session over the B200 verify step.

A host-side restatement of velo-core's session loop (src/speculative.rs):
SpeculativeDecoder (:255-361), SpeculativeSession::draft / commit (:400-519),
adjust_window (:529-537), SpeculativeStats and SpeculativeError (:280-305),
driving device models through the TargetModel / DraftModel shape
(:133-254):

- CudaTarget.verify runs one velo_cuda_verify_step over a chain whose root is
  the last context token (the trait contract: step i holds the target's token
  for drafted[i]) and commits the accepted path's K/V into the slot's pages;
- CudaDraft.draft decodes greedily one token per step through the same call
  (commit of every node), rewinding its cache to the prefix it shares with the
  session's context, so rejected drafts are rolled back by length.

The session logic itself is plain Python; every model call is the C ABI.
"""
import ctypes
import re
from dataclasses import dataclass, field

import numpy as np

import velo_cuda


class SpeculativeError(Exception):
    """SpeculativeError (speculative.rs:294-305)."""


class EmptyDraftWindow(SpeculativeError):
    def __str__(self):
        return "draft window must be greater than zero"


class DraftReturnedTooMany(SpeculativeError):
    def __init__(self, requested, returned):
        super().__init__(requested, returned)
        self.requested, self.returned = requested, returned

    def __str__(self):
        return f"draft model returned {self.returned} tokens, requested at most {self.requested}"


class TargetReturnedWrongLength(SpeculativeError):
    def __init__(self, drafted, returned):
        super().__init__(drafted, returned)
        self.drafted, self.returned = drafted, returned

    def __str__(self):
        return (f"target model returned {self.returned} verification steps "
                f"for {self.drafted} drafted tokens")


@dataclass
class SpeculativeStats:
    draft_calls: int = 0
    target_calls: int = 0
    drafted_tokens: int = 0
    accepted_tokens: int = 0
    rejected_tokens: int = 0


@dataclass
class SpeculativeOutput:
    tokens: list
    stats: SpeculativeStats


@dataclass
class NextTokenPrediction:
    token: int
    confidence: float = 1.0


@dataclass
class VerifyStep:
    expected: int


class SpeculativeTree:
    """SpeculativeTree / TreeNode (speculative.rs:47-96): drafted tokens with
    parent links; node 0 is the root (parent None)."""

    def __init__(self, token):
        self.tokens, self.parents = [int(token)], [None]

    def add_child(self, parent_idx, token):
        self.tokens.append(int(token))
        self.parents.append(int(parent_idx))
        return len(self.tokens) - 1

    def get_path(self, idx):
        path = []
        while idx is not None:
            path.append(self.tokens[idx])
            idx = self.parents[idx]
        return path[::-1]

    def find_best_path(self, expected):
        """find_best_path (speculative.rs:97-129): valid[0]; valid[n] =
        valid[parent] and token[n] == expected[parent]; the deepest valid node
        wins (ties to the later index); returns (path tokens, expected[best])."""
        n = len(self.tokens)
        valid, depth = [False] * n, [0] * n
        valid[0], depth[0] = True, 1
        best = 0
        for i in range(1, n):
            p = self.parents[i]
            if valid[p] and self.tokens[i] == expected[p]:
                valid[i], depth[i] = True, depth[p] + 1
            if valid[i] and depth[i] >= depth[best]:
                best = i
        return self.get_path(best), expected[best]


@dataclass
class TreeVerifyResult:
    expected: list


def top_k(logits, k):
    """TopKSampler::sample_top_k (sampling.rs:105-131): the k largest logits
    by a stable descending sort (equal logits keep ascending token order).
    TopKSampler::sample (sampling.rs:76-100) is its first entry.  Finite
    logits only (the reference's NaN placement depends on its sort)."""
    x = np.asarray(logits, np.float32)
    order = np.argsort(-x, kind="stable")[:k]
    return [NextTokenPrediction(int(i), float(x[i])) for i in order]


class SpeculativeDecoder:
    """SpeculativeDecoder::new / with_max_window / generate / begin."""

    def __init__(self, draft_window, max_window=None):
        if draft_window == 0 or (max_window is not None and max_window < draft_window):
            raise EmptyDraftWindow()
        self.draft_window = draft_window
        self.max_window = draft_window * 2 if max_window is None else max_window

    def begin(self, prompt):
        return SpeculativeSession(self.draft_window, self.max_window, list(prompt))

    def generate(self, draft_model, target_model, prompt, max_new_tokens):
        session = self.begin(prompt)
        generated = []
        while len(generated) < max_new_tokens:
            remaining = max_new_tokens - len(generated)
            drafted = session.draft(draft_model, target_model, remaining)
            if not drafted and not session.has_pending_rejection():
                break
            generated.extend(drafted)
            if not session.has_pending_rejection():
                continue
            token = session.take_rejected_token()
            if token is not None:
                generated.append(token)
        return SpeculativeOutput(generated, session.stats)


@dataclass
class SpeculativeSession:
    draft_window: int
    max_window: int
    prompt: list
    context: list = field(default=None)
    stats: SpeculativeStats = field(default_factory=SpeculativeStats)
    rejected_token: object = None

    def __post_init__(self):
        if self.context is None:
            self.context = list(self.prompt)

    def has_pending_rejection(self):
        return self.rejected_token is not None

    def take_rejected_token(self):
        t, self.rejected_token = self.rejected_token, None
        return t

    def current_window(self):
        return self.draft_window

    def record_draft_call(self):
        self.stats.draft_calls += 1

    def record_target_call(self):
        self.stats.target_calls += 1

    def draft(self, draft_model, target_model, max_new_tokens):
        """SpeculativeSession::draft (speculative.rs:400-471)."""
        requested = min(max_new_tokens, self.draft_window)
        predictions = draft_model.draft(self.context, requested)
        self.stats.draft_calls += 1
        if len(predictions) > requested:
            raise DraftReturnedTooMany(requested, len(predictions))
        if not predictions:
            return []
        drafted = [p.token for p in predictions]
        self.stats.drafted_tokens += len(drafted)
        verified = target_model.verify(self.context, drafted)
        self.stats.target_calls += 1
        if len(verified) != len(drafted):
            raise TargetReturnedWrongLength(len(drafted), len(verified))
        return self._accept(drafted, verified)

    def commit(self, drafted, verified):
        """SpeculativeSession::commit (speculative.rs:473-519)."""
        if len(verified) != len(drafted):
            raise TargetReturnedWrongLength(len(drafted), len(verified))
        self.stats.drafted_tokens += len(drafted)
        return self._accept([p.token for p in drafted], verified)

    def _accept(self, drafted, verified):
        accepted_this_round, rejected = 0, None
        for index, (tok, step) in enumerate(zip(drafted, verified)):
            if tok == step.expected:
                accepted_this_round += 1
                continue
            rejected = (index, step.expected)
            break
        accepted = list(drafted[:accepted_this_round])
        if accepted:
            self.context.extend(accepted)
            self.stats.accepted_tokens += accepted_this_round
        if rejected is not None:
            self.context.append(rejected[1])
            self.rejected_token = rejected[1]
            self.stats.rejected_tokens += len(drafted) - rejected[0]
        else:
            self.rejected_token = None
        self._adjust_window(accepted_this_round, len(drafted))
        return accepted

    def _adjust_window(self, accepted_count, drafted_count):
        """adjust_window (speculative.rs:529-537)."""
        if accepted_count == drafted_count:
            if self.draft_window < self.max_window:
                self.draft_window += 1
        else:
            self.draft_window = max(accepted_count + 1, 1)


# ---------------------------------------------------------------- device models
def sample_token(logits, temperature, u):
    """Inverse-CDF draw from softmax(logits / T) with the uniform u (the draft
    model's sampler at T > 0; float64 on the host)."""
    z = np.asarray(logits, np.float64) / temperature
    p = np.exp(z - z.max())
    c = np.cumsum(p)
    return min(int(np.searchsorted(c, u * c[-1], side="right")), len(c) - 1)


class CudaTarget:
    """TargetModel over velo_cuda_verify_step for one sequence (`slot`).

    The slot's pages hold the K/V of context[:-1]; verify() runs the chain
    [context[-1]] + drafted and commits the accepted path, so the invariant
    holds for the session's next context.  Rows past the first mismatch are
    not needed by the session and repeat the target's token there.

    temperature > 0: rejection sampling against the draft's distributions
    (`draft.last_logits`) with uniforms from `rng`; the residual / bonus draw
    stands at the first rejected position."""

    def __init__(self, ctx, slot, n_vocab, temperature=0.0, draft=None, rng=None):
        self.ctx, self.slot, self.n_vocab, self.T = ctx, slot, n_vocab, temperature
        self.draft, self.rng = draft, rng
        self.cached = 0  # tokens of the context whose K/V are in the pages

    def prefill(self, context):
        n = len(context) - 1
        if n > self.cached:
            velo_cuda.prefill(self.ctx, self.slot, context[self.cached:n], pos0=self.cached,
                              n_vocab=self.n_vocab)
            self.cached = n

    def verify(self, context, drafted):
        self.prefill(context)
        pos = len(context) - 1
        nodes = np.array([context[-1]] + list(drafted), np.uint32)
        parents = np.arange(-1, len(nodes) - 1, dtype=np.int32)
        kw = {}
        if self.T > 0 and drafted:
            kw = dict(temperature=self.T, draft_logits=self.draft.last_logits[None, :len(drafted)],
                      uniforms=self.rng.random((1, len(nodes))).astype(np.float32))
        r = self.ctx.verify_step([self.slot], [pos], nodes[None], parents[None], commit=True,
                                 n_vocab=self.n_vocab, **kw)
        acc, bonus = int(r["accepted_len"][0]), int(r["bonus"][0])
        self.cached = pos + acc + 1
        return ([VerifyStep(t) for t in drafted[:acc]] +
                [VerifyStep(bonus)] * (len(drafted) - acc))


class CudaDraft:
    """DraftModel: decoding on the device, one verify step per token (commit
    of every node), cache rewound to the prefix it shares with the session's
    context.  Greedy at temperature 0, else each token drawn from the step's
    logits (sample_token) and the logits kept in `last_logits` for the
    target's rejection sampling."""

    def __init__(self, ctx, slot, n_vocab, temperature=0.0, rng=None):
        self.ctx, self.slot, self.n_vocab, self.T, self.rng = ctx, slot, n_vocab, temperature, rng
        self.tokens = []  # tokens whose K/V are in the draft's pages
        self.last_logits = None

    def prefill(self, context):
        """Rewind to the prefix shared with context[:-1], then fill the rest."""
        common = 0
        for a, b in zip(self.tokens, context[:-1]):
            if a != b:
                break
            common += 1
        self.tokens = self.tokens[:common]
        if len(context) - 1 > common:
            velo_cuda.prefill(self.ctx, self.slot, context[common:-1], pos0=common,
                              n_vocab=self.n_vocab)
            self.tokens = list(context[:-1])

    def draft(self, context, max_tokens):
        if max_tokens <= 0:
            return []
        self.prefill(context)
        out, last, logits = [], context[-1], []
        for _ in range(max_tokens):
            pos = len(self.tokens)
            r = self.ctx.verify_step([self.slot], [pos], np.array([[last]], np.uint32),
                                     np.array([[-1]], np.int32), commit="all",
                                     want_logits=self.T > 0, n_vocab=self.n_vocab)
            self.tokens.append(last)
            if self.T > 0:
                lg = r["logits"][0, 0]
                logits.append(lg)
                last = sample_token(lg, self.T, self.rng.random())
            else:
                last = int(r["bonus"][0])
            out.append(NextTokenPrediction(last))
        if self.T > 0:
            self.last_logits = np.stack(logits)
        return out


class CudaTreeDraft(CudaDraft):
    """TreeDraftModel::draft_tree (backend.rs:255-294) on the device: the
    draft's top-`width` tokens after the context form the root and its
    children, then the primary branch is extended greedily (TopKSampler) to
    max_tokens nodes, one decode step per node."""

    def _decode(self, token):
        pos = len(self.tokens)
        r = self.ctx.verify_step([self.slot], [pos], np.array([[token]], np.uint32),
                                 np.array([[-1]], np.int32), commit="all", want_logits=True,
                                 n_vocab=self.n_vocab)
        self.tokens.append(int(token))
        return r["logits"][0, 0]

    def draft_tree(self, context, max_tokens, width):
        self.prefill(context)
        top = top_k(self._decode(context[-1]), width)
        if not top:
            raise SpeculativeError("Draft model returned no tokens")
        tree = SpeculativeTree(top[0].token)
        for pred in top[1:]:
            tree.add_child(0, pred.token)
        curr = 0
        for _ in range(1, max_tokens):
            nxt = top_k(self._decode(tree.tokens[curr]), 1)[0].token
            curr = tree.add_child(curr, nxt)
        return tree


def rooted_tree(context, tree):
    """The tree the device verifies: the last context token as root, the draft
    tree under it (its root a child of node 0).  find_best_path over this tree
    checks the first drafted token as well (the trait contract), where the
    reference's draft_tree root would be taken unchecked."""
    t = SpeculativeTree(context[-1])
    for tok, p in zip(tree.tokens, tree.parents):
        t.add_child(0 if p is None else p + 1, tok)
    return t


def verify_tree_on_device(ctx, slot, n_vocab, context, tree, commit=True):
    """TargetModel::verify_tree (speculative.rs:217-242) over the whole tree in
    one verify step.  Returns (the rooted tree, TreeVerifyResult with the
    target's token after each of its nodes, the step's result); with commit
    the accepted path's K/V are written at len(context) - 1 onwards."""
    rt = rooted_tree(context, tree)
    nodes = np.array(rt.tokens, np.uint32)
    parents = np.array([-1] + rt.parents[1:], np.int32)
    r = ctx.verify_step([slot], [len(context) - 1], nodes[None], parents[None], commit=commit,
                        n_vocab=n_vocab)
    return rt, TreeVerifyResult([int(e) for e in r["expected"][0]]), r


# ---------------------------------------------------------------- batched engine
class SlotsExhausted(SpeculativeError):
    """SlotPool has no free slot for a request (the engine's acquire failure)."""

    def __init__(self, requested, available):
        super().__init__(requested, available)
        self.requested, self.available = requested, available

    def __str__(self):
        return f"no free slot: {self.requested} requests, {self.available} slots"


def _draft_batch(model, reqs):
    """DraftModel::draft_batch; the trait's default drafts one request at a
    time (speculative.rs:133-254).  reqs: [(request id, context, max tokens)]."""
    if hasattr(model, "draft_batch"):
        return model.draft_batch(reqs)
    return [model.draft(c, m) for _, c, m in reqs]


def _verify_batch(model, reqs):
    """TargetModel::verify_batch, default one request at a time.
    reqs: [(request id, context, drafted tokens)]."""
    if hasattr(model, "verify_batch"):
        return model.verify_batch(reqs)
    return [model.verify(c, d) for _, c, d in reqs]


class SpeculativeEngine:
    """VeloEngine::generate_batch (engine.rs:233-420) over the verify step.

    Each round, every request still short of max_new_tokens drafts
    min(remaining, draft_window) tokens (the decoder's fixed window, as the
    engine's loop uses it), ONE verify_batch call covers all of them (on the
    device: one velo_cuda_verify_step for all slots), then each session
    commits its own result and emits the target's token at a rejection.
    Requests are numbered 0..n-1 and bound to slots 0..n-1; more requests
    than `max_slots` is an error, as when the engine's SlotPool runs dry.
    A round in which no request makes progress (a draft model returning
    nothing) ends the loop instead of repeating forever."""

    def __init__(self, draft_window, max_window=None, max_slots=None):
        self.decoder = SpeculativeDecoder(draft_window, max_window)
        self.max_slots = max_slots

    def generate_batch(self, draft_model, target_model, requests):
        """requests: [(prompt, max_new_tokens)] -> [SpeculativeOutput]."""
        if self.max_slots is not None and len(requests) > self.max_slots:
            raise SlotsExhausted(len(requests), self.max_slots)
        sessions = [self.decoder.begin(p) for p, _ in requests]
        limits = [int(m) for _, m in requests]
        generated = [[] for _ in requests]
        for model in (draft_model, target_model):
            if hasattr(model, "bind_slot"):
                for i in range(len(requests)):
                    model.bind_slot(i)
        while True:
            active = [i for i in range(len(requests)) if len(generated[i]) < limits[i]]
            if not active:
                break
            window = self.decoder.draft_window
            drafts = _draft_batch(draft_model, [(i, sessions[i].context,
                                                 min(limits[i] - len(generated[i]), window))
                                                for i in active])
            for i in active:
                sessions[i].record_draft_call()
            verified = _verify_batch(target_model, [(i, sessions[i].context, [p.token for p in d])
                                                    for i, d in zip(active, drafts)])
            for i in active:
                sessions[i].record_target_call()
            progressed = False
            for i, d, v in zip(active, drafts, verified):
                accepted = sessions[i].commit(d, v)
                generated[i].extend(accepted)
                progressed |= bool(accepted)
                if sessions[i].has_pending_rejection():
                    token = sessions[i].take_rejected_token()
                    if token is not None:
                        generated[i].append(token)
                        progressed = True
            if not progressed:
                break
        return [SpeculativeOutput(generated[i], sessions[i].stats) for i in range(len(requests))]


class CudaBatchTarget:
    """TargetModel::verify_batch on the device: the chains of all requests
    with the same draft length run as ONE velo_cuda_verify_step (B requests,
    N = k + 1 nodes each, every sequence at its own context length), each
    committing its accepted path into its own slot (`slots[request id]`).
    Per slot the pages hold the K/V of context[:-1], as for CudaTarget."""

    def __init__(self, ctx, slots, n_vocab):
        self.ctx, self.slots, self.n_vocab = ctx, list(slots), n_vocab
        self.cached = {}

    def _prefill(self, rid, context):
        have, n = self.cached.get(rid, 0), len(context) - 1
        if n > have:
            velo_cuda.prefill(self.ctx, self.slots[rid], context[have:n], pos0=have, n_vocab=self.n_vocab)
            self.cached[rid] = n

    def verify_batch(self, reqs):
        out = [None] * len(reqs)
        groups = {}
        for j, (rid, context, drafted) in enumerate(reqs):
            self._prefill(rid, context)
            groups.setdefault(len(drafted), []).append(j)
        for k, members in groups.items():
            # k == 0 still runs: the root's K/V is committed, as CudaTarget does
            tokens = np.array([[reqs[j][1][-1]] + list(reqs[j][2]) for j in members], np.uint32)
            parents = np.tile(np.arange(-1, k, dtype=np.int32), (len(members), 1))
            pos = [len(reqs[j][1]) - 1 for j in members]
            r = self.ctx.verify_step([self.slots[reqs[j][0]] for j in members], pos, tokens, parents,
                                     commit=True, n_vocab=self.n_vocab)
            for b, j in enumerate(members):
                rid, _, drafted = reqs[j]
                acc, bonus = int(r["accepted_len"][b]), int(r["bonus"][b])
                self.cached[rid] = pos[b] + acc + 1
                out[j] = [VerifyStep(t) for t in drafted[:acc]] + [VerifyStep(bonus)] * (k - acc)
        return out


class CudaBatchDraft:
    """DraftModel::draft_batch on the device, greedy: each slot's cache is
    rewound to the prefix it shares with its context (as CudaDraft), then
    every draft position is ONE velo_cuda_verify_step over all requests that
    still need a token (B requests, one node each, commit of every node)."""

    def __init__(self, ctx, slots, n_vocab):
        self.ctx, self.slots, self.n_vocab = ctx, list(slots), n_vocab
        self.tokens = {}

    def _prefill(self, rid, context):
        have = self.tokens.get(rid, [])
        common = 0
        for a, b in zip(have, context[:-1]):
            if a != b:
                break
            common += 1
        self.tokens[rid] = list(have[:common])
        if len(context) - 1 > common:
            velo_cuda.prefill(self.ctx, self.slots[rid], context[common:-1], pos0=common,
                              n_vocab=self.n_vocab)
            self.tokens[rid] = [int(t) for t in context[:-1]]

    def draft_batch(self, reqs):
        out = [[] for _ in reqs]
        last = []
        for rid, context, _ in reqs:
            self._prefill(rid, context)
            last.append(int(context[-1]))
        while True:
            live = [j for j, (_, _, m) in enumerate(reqs) if len(out[j]) < m]
            if not live:
                break
            rids = [reqs[j][0] for j in live]
            r = self.ctx.verify_step([self.slots[rid] for rid in rids],
                                     [len(self.tokens[rid]) for rid in rids],
                                     np.array([[last[j]] for j in live], np.uint32),
                                     np.full((len(live), 1), -1, np.int32), commit="all",
                                     n_vocab=self.n_vocab)
            for b, j in enumerate(live):
                self.tokens[rids[b]].append(last[j])
                last[j] = int(r["bonus"][b])
                out[j].append(NextTokenPrediction(last[j]))
        return out


# ---------------------------------------------------------------- native session
def _native_error(status, errors):
    """The SpeculativeError (or the model's own exception) for a status of the
    native session (include/velo_session.h)."""
    if errors:
        return errors[0]
    msg = velo_cuda.last_error()
    if status == velo_cuda.ERR_EMPTY_DRAFT_WINDOW:
        return EmptyDraftWindow()
    if status == velo_cuda.ERR_DRAFT_TOO_MANY:
        m = re.search(r"returned (\d+) tokens, requested at most (\d+)", msg)
        return DraftReturnedTooMany(int(m.group(2)), int(m.group(1)))
    if status == velo_cuda.ERR_TARGET_WRONG_LENGTH:
        m = re.search(r"returned (\d+) verification steps for (\d+) drafted", msg)
        return TargetReturnedWrongLength(int(m.group(2)), int(m.group(1)))
    return velo_cuda.VeloError(status, msg)


def _callbacks(draft_model, target_model, errors):
    """ctypes callbacks over Python DraftModel / TargetModel objects; an
    exception is kept in `errors` and reported as a model failure."""

    @velo_cuda.DRAFT_FN
    def draft_fn(_user, ctx, n, max_tokens, out, cap, n_out):
        try:
            preds = draft_model.draft([ctx[i] for i in range(n)], max_tokens)
            for i, p in enumerate(preds[:cap]):
                out[i] = int(p.token)
            n_out[0] = len(preds)
            return 0
        except Exception as e:  # noqa: BLE001 -- handed back to the caller
            errors.append(e)
            return velo_cuda.ERR_INVALID_ARGUMENT

    @velo_cuda.VERIFY_FN
    def verify_fn(_user, ctx, n, drafted, k, out, cap, n_out):
        try:
            steps = target_model.verify([ctx[i] for i in range(n)], [drafted[i] for i in range(k)])
            for i, st in enumerate(steps[:cap]):
                out[i] = int(st.expected)
            n_out[0] = len(steps)
            return 0
        except Exception as e:  # noqa: BLE001
            errors.append(e)
            return velo_cuda.ERR_INVALID_ARGUMENT

    return draft_fn, verify_fn


def _stats(s):
    return SpeculativeStats(s.draft_calls, s.target_calls, s.drafted_tokens, s.accepted_tokens,
                            s.rejected_tokens)


def native_generate(draft_window, draft_model, target_model, prompt, max_new_tokens, max_window=None):
    """SpeculativeDecoder::generate through the native loop (velo_spec_generate)."""
    errors = []
    dfn, vfn = _callbacks(draft_model, target_model, errors)
    p = np.ascontiguousarray(prompt, np.uint32)
    out = np.zeros(max(int(max_new_tokens), 1), np.uint32)
    n = ctypes.c_size_t()
    st = velo_cuda.SpecStats()
    rc = velo_cuda.lib().velo_spec_generate(draft_window, max_window or 0, dfn, None, vfn, None,
                                            p.ctypes.data_as(ctypes.c_void_p), p.size, max_new_tokens,
                                            out.ctypes.data_as(ctypes.c_void_p), out.size, ctypes.byref(n),
                                            ctypes.byref(st))
    if rc:
        raise _native_error(rc, errors)
    return SpeculativeOutput([int(t) for t in out[:n.value]], _stats(st))


class NativeSession:
    """SpeculativeSession over the native session (velo_spec_session_*)."""

    def __init__(self, draft_window, prompt, max_window=None):
        self._h = None
        p = np.ascontiguousarray(prompt, np.uint32)
        h = ctypes.c_void_p()
        rc = velo_cuda.lib().velo_spec_session_create(draft_window, max_window or 0,
                                                      p.ctypes.data_as(ctypes.c_void_p), p.size, ctypes.byref(h))
        if rc:
            raise _native_error(rc, [])
        self._h = h

    def __del__(self):
        if getattr(self, "_h", None):
            velo_cuda.lib().velo_spec_session_destroy(self._h)
            self._h = None

    def _accepted(self, call, cap):
        out = np.zeros(max(cap, 1), np.uint32)
        n = ctypes.c_size_t()
        rc = call(out.ctypes.data_as(ctypes.c_void_p), out.size, ctypes.byref(n))
        return rc, [int(t) for t in out[:n.value]] if not rc else []

    def draft(self, draft_model, target_model, max_new_tokens):
        errors = []
        dfn, vfn = _callbacks(draft_model, target_model, errors)
        rc, acc = self._accepted(lambda o, c, n: velo_cuda.lib().velo_spec_session_draft(
            self._h, dfn, None, vfn, None, max_new_tokens, o, c, n), max_new_tokens)
        if rc:
            raise _native_error(rc, errors)
        return acc

    def commit(self, drafted, verified):
        d = np.ascontiguousarray([p.token for p in drafted], np.uint32)
        v = np.ascontiguousarray([s.expected for s in verified], np.uint32)
        rc, acc = self._accepted(lambda o, c, n: velo_cuda.lib().velo_spec_session_commit(
            self._h, d.ctypes.data_as(ctypes.c_void_p), d.size, v.ctypes.data_as(ctypes.c_void_p), v.size,
            o, c, n), len(drafted))
        if rc:
            raise _native_error(rc, [])
        return acc

    def has_pending_rejection(self):
        return bool(velo_cuda.lib().velo_spec_session_has_pending_rejection(self._h))

    def take_rejected_token(self):
        t = ctypes.c_uint32()
        return int(t.value) if velo_cuda.lib().velo_spec_session_take_rejected(self._h, ctypes.byref(t)) else None

    @property
    def context(self):
        n = velo_cuda.lib().velo_spec_session_context(self._h, None, 0)
        out = np.zeros(max(n, 1), np.uint32)
        velo_cuda.lib().velo_spec_session_context(self._h, out.ctypes.data_as(ctypes.c_void_p), n)
        return [int(t) for t in out[:n]]

    @property
    def draft_window(self):
        return velo_cuda.lib().velo_spec_session_window(self._h)

    @property
    def stats(self):
        s = velo_cuda.SpecStats()
        velo_cuda.lib().velo_spec_session_stats(self._h, ctypes.byref(s))
        return _stats(s)

    def record_draft_call(self):
        velo_cuda.lib().velo_spec_session_record_draft_call(self._h)

    def record_target_call(self):
        velo_cuda.lib().velo_spec_session_record_target_call(self._h)


def native_generate_batch(draft_window, draft_model, target_model, requests, max_window=None, max_slots=None):
    """SpeculativeEngine.generate_batch through the native engine loop
    (velo_spec_generate_batch); the models' draft_batch / verify_batch (or
    their one-request methods) are the callbacks."""
    errors = []

    @velo_cuda.DRAFT_BATCH_FN
    def draft_fn(_user, n, ids, ctxs, nctx, want, out, stride, n_out):
        try:
            reqs = [(ids[j], [ctxs[j][i] for i in range(nctx[j])], want[j]) for j in range(n)]
            for j, preds in enumerate(_draft_batch(draft_model, reqs)):
                for i, p in enumerate(preds[:stride]):
                    out[j * stride + i] = int(p.token)
                n_out[j] = len(preds)
            return 0
        except Exception as e:  # noqa: BLE001
            errors.append(e)
            return velo_cuda.ERR_INVALID_ARGUMENT

    @velo_cuda.VERIFY_BATCH_FN
    def verify_fn(_user, n, ids, ctxs, nctx, drafted, nd, out, stride, n_out):
        try:
            reqs = [(ids[j], [ctxs[j][i] for i in range(nctx[j])], [drafted[j][i] for i in range(nd[j])])
                    for j in range(n)]
            for j, steps in enumerate(_verify_batch(target_model, reqs)):
                for i, st in enumerate(steps[:stride]):
                    out[j * stride + i] = int(st.expected)
                n_out[j] = len(steps)
            return 0
        except Exception as e:  # noqa: BLE001
            errors.append(e)
            return velo_cuda.ERR_INVALID_ARGUMENT

    n = len(requests)
    prompts = [np.ascontiguousarray(p, np.uint32) for p, _ in requests]
    limits = np.array([int(m) for _, m in requests], np.uintp)
    outs = [np.zeros(max(int(m), 1), np.uint32) for _, m in requests]
    pp = (ctypes.c_void_p * max(n, 1))(*[p.ctypes.data for p in prompts])
    op = (ctypes.c_void_p * max(n, 1))(*[o.ctypes.data for o in outs])
    npr = np.array([p.size for p in prompts], np.uintp)
    n_out = np.zeros(max(n, 1), np.uintp)
    stats = (velo_cuda.SpecStats * max(n, 1))()
    rc = velo_cuda.lib().velo_spec_generate_batch(
        draft_window, max_window or 0, max_slots or 0, draft_fn, None, verify_fn, None, n, pp,
        npr.ctypes.data_as(ctypes.c_void_p), limits.ctypes.data_as(ctypes.c_void_p), op,
        n_out.ctypes.data_as(ctypes.c_void_p), stats)
    if rc:
        if rc == velo_cuda.ERR_INVALID_ARGUMENT and "no free slot" in velo_cuda.last_error() and not errors:
            raise SlotsExhausted(n, max_slots)
        raise _native_error(rc, errors)
    return [SpeculativeOutput([int(t) for t in outs[i][:n_out[i]]], _stats(stats[i])) for i in range(n)]
