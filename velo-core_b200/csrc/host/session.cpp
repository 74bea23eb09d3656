// session.cpp -- the speculative-decoding session loop (include/velo_session.h),
// following src/speculative.rs: SpeculativeDecoder::new / with_max_window /
// generate / begin (:310-370), SpeculativeSession::draft (:400-471), commit
// (:473-519) and adjust_window (:529-537).  Models are callbacks; this file
// holds the window and accept rules and the statistics.
#include <algorithm>
#include <vector>

#include "runtime/context.h"
#include "velo_session.h"

struct velo_spec_session {
    size_t window = 0, max_window = 0;
    std::vector<uint32_t> context;
    velo_spec_stats stats{};
    bool pending = false;
    uint32_t rejected = 0;
};

using velo::fail;

namespace {

// The accept rule: the longest prefix of drafted whose tokens equal the
// target's, then the target's token at the first mismatch.
void accept(velo_spec_session* s, const uint32_t* drafted, size_t n, const uint32_t* expected,
            std::vector<uint32_t>* accepted) {
    size_t acc = 0;
    while (acc < n && drafted[acc] == expected[acc]) ++acc;
    accepted->assign(drafted, drafted + acc);
    s->context.insert(s->context.end(), drafted, drafted + acc);
    s->stats.accepted_tokens += acc;
    if (acc < n) {
        s->context.push_back(expected[acc]);
        s->pending = true;
        s->rejected = expected[acc];
        s->stats.rejected_tokens += n - acc;
    } else {
        s->pending = false;
    }
    // adjust_window: grow by one after a fully accepted round (up to the
    // maximum), else shrink to one past the accepted count
    if (acc == n) {
        if (s->window < s->max_window) ++s->window;
    } else {
        s->window = std::max<size_t>(acc + 1, 1);
    }
}

int32_t copy_out(const std::vector<uint32_t>& v, uint32_t* out, size_t cap, size_t* n) {
    if (n) *n = v.size();
    if (v.size() > cap || (!out && !v.empty()))
        return fail(VELO_ERR_INVALID_ARGUMENT, "output holds %zu tokens, %zu accepted", cap, v.size());
    std::copy(v.begin(), v.end(), out);
    return VELO_OK;
}

// One draft + verify round; accepted tokens in *accepted.
int32_t draft_round(velo_spec_session* s, velo_draft_fn draft, void* du, velo_verify_fn verify, void* vu,
                    size_t max_new_tokens, std::vector<uint32_t>* accepted) {
    accepted->clear();
    const size_t requested = std::min(max_new_tokens, s->window);
    std::vector<uint32_t> drafted(requested);
    size_t n = 0;
    int32_t st = draft(du, s->context.data(), s->context.size(), requested, drafted.data(), requested, &n);
    s->stats.draft_calls += 1;
    if (st) return fail(st, "draft model failed (status %d)", st);
    if (n > requested)
        return fail(VELO_ERR_DRAFT_TOO_MANY, "draft model returned %zu tokens, requested at most %zu", n, requested);
    if (n == 0) return VELO_OK;
    drafted.resize(n);
    s->stats.drafted_tokens += n;
    std::vector<uint32_t> expected(n);
    size_t m = 0;
    st = verify(vu, s->context.data(), s->context.size(), drafted.data(), n, expected.data(), n, &m);
    s->stats.target_calls += 1;
    if (st) return fail(st, "target model failed (status %d)", st);
    if (m != n)
        return fail(VELO_ERR_TARGET_WRONG_LENGTH,
                    "target model returned %zu verification steps for %zu drafted tokens", m, n);
    accept(s, drafted.data(), n, expected.data(), accepted);
    return VELO_OK;
}

}  // namespace

extern "C" {

int32_t velo_spec_session_create(uint32_t draft_window, uint32_t max_window, const uint32_t* prompt,
                                 size_t n_prompt, velo_spec_session** out) {
    velo::clear_last_error();
    if (!out) return fail(VELO_ERR_INVALID_ARGUMENT, "out is NULL");
    *out = nullptr;
    const size_t mw = max_window ? max_window : (size_t)draft_window * 2;
    if (draft_window == 0 || mw < draft_window)
        return fail(VELO_ERR_EMPTY_DRAFT_WINDOW, "draft window must be greater than zero");
    if (n_prompt && !prompt) return fail(VELO_ERR_INVALID_ARGUMENT, "prompt is NULL");
    velo_spec_session* s = new velo_spec_session();
    s->window = draft_window;
    s->max_window = mw;
    s->context.assign(prompt, prompt + n_prompt);
    *out = s;
    return VELO_OK;
}

void velo_spec_session_destroy(velo_spec_session* s) { delete s; }

int32_t velo_spec_session_draft(velo_spec_session* s, velo_draft_fn draft, void* draft_user, velo_verify_fn verify,
                                void* verify_user, size_t max_new_tokens, uint32_t* accepted, size_t cap,
                                size_t* n_accepted) {
    velo::clear_last_error();
    if (!s || !draft || !verify) return fail(VELO_ERR_INVALID_ARGUMENT, "NULL argument");
    std::vector<uint32_t> acc;
    const int32_t st = draft_round(s, draft, draft_user, verify, verify_user, max_new_tokens, &acc);
    if (st) return st;
    return copy_out(acc, accepted, cap, n_accepted);
}

int32_t velo_spec_session_commit(velo_spec_session* s, const uint32_t* drafted, size_t n_drafted,
                                 const uint32_t* verified, size_t n_verified, uint32_t* accepted, size_t cap,
                                 size_t* n_accepted) {
    velo::clear_last_error();
    if (!s) return fail(VELO_ERR_INVALID_ARGUMENT, "session is NULL");
    if (n_verified != n_drafted)
        return fail(VELO_ERR_TARGET_WRONG_LENGTH,
                    "target model returned %zu verification steps for %zu drafted tokens", n_verified, n_drafted);
    if (n_drafted && (!drafted || !verified)) return fail(VELO_ERR_INVALID_ARGUMENT, "NULL tokens");
    s->stats.drafted_tokens += n_drafted;
    std::vector<uint32_t> acc;
    accept(s, drafted, n_drafted, verified, &acc);
    return copy_out(acc, accepted, cap, n_accepted);
}

int32_t velo_spec_session_take_rejected(velo_spec_session* s, uint32_t* token) {
    if (!s || !s->pending) return 0;
    s->pending = false;
    if (token) *token = s->rejected;
    return 1;
}

int32_t velo_spec_session_has_pending_rejection(const velo_spec_session* s) { return s && s->pending ? 1 : 0; }

size_t velo_spec_session_context(const velo_spec_session* s, uint32_t* out, size_t cap) {
    if (!s) return 0;
    if (out) std::copy_n(s->context.begin(), std::min(cap, s->context.size()), out);
    return s->context.size();
}

uint32_t velo_spec_session_window(const velo_spec_session* s) { return s ? (uint32_t)s->window : 0; }

void velo_spec_session_stats(const velo_spec_session* s, velo_spec_stats* out) {
    if (s && out) *out = s->stats;
}

void velo_spec_session_record_draft_call(velo_spec_session* s) {
    if (s) s->stats.draft_calls += 1;
}

void velo_spec_session_record_target_call(velo_spec_session* s) {
    if (s) s->stats.target_calls += 1;
}

int32_t velo_spec_generate(uint32_t draft_window, uint32_t max_window, velo_draft_fn draft, void* draft_user,
                           velo_verify_fn verify, void* verify_user, const uint32_t* prompt, size_t n_prompt,
                           size_t max_new_tokens, uint32_t* out, size_t cap, size_t* n_out, velo_spec_stats* stats) {
    velo::clear_last_error();
    if (!draft || !verify || !n_out) return fail(VELO_ERR_INVALID_ARGUMENT, "NULL argument");
    if (cap < max_new_tokens || (max_new_tokens && !out))
        return fail(VELO_ERR_INVALID_ARGUMENT, "output holds %zu tokens, %zu may be generated", cap, max_new_tokens);
    velo_spec_session* s = nullptr;
    int32_t st = velo_spec_session_create(draft_window, max_window, prompt, n_prompt, &s);
    if (st) return st;
    std::vector<uint32_t> generated, acc;
    while (generated.size() < max_new_tokens) {
        st = draft_round(s, draft, draft_user, verify, verify_user, max_new_tokens - generated.size(), &acc);
        if (st) break;
        if (acc.empty() && !s->pending) break;
        generated.insert(generated.end(), acc.begin(), acc.end());
        if (!s->pending) continue;
        s->pending = false;
        generated.push_back(s->rejected);
    }
    if (stats) *stats = s->stats;
    delete s;
    if (st) return st;
    *n_out = generated.size();
    std::copy(generated.begin(), generated.end(), out);
    return VELO_OK;
}

int32_t velo_spec_generate_batch(uint32_t draft_window, uint32_t max_window, size_t max_slots,
                                 velo_draft_batch_fn draft, void* draft_user, velo_verify_batch_fn verify,
                                 void* verify_user, size_t n, const uint32_t* const* prompts, const size_t* n_prompt,
                                 const size_t* max_new_tokens, uint32_t* const* out, size_t* n_out,
                                 velo_spec_stats* stats) {
    velo::clear_last_error();
    if (!draft || !verify || (n && (!prompts || !n_prompt || !max_new_tokens || !out || !n_out)))
        return fail(VELO_ERR_INVALID_ARGUMENT, "NULL argument");
    if (max_slots && n > max_slots)
        return fail(VELO_ERR_INVALID_ARGUMENT, "no free slot: %zu requests, %zu slots", n, max_slots);
    std::vector<velo_spec_session*> sess(n, nullptr);
    auto cleanup = [&](int32_t st) {
        for (size_t i = 0; i < n; ++i) {
            if (stats && sess[i]) stats[i] = sess[i]->stats;
            delete sess[i];
        }
        return st;
    };
    for (size_t i = 0; i < n; ++i) {
        const int32_t st = velo_spec_session_create(draft_window, max_window, prompts[i], n_prompt[i], &sess[i]);
        if (st) return cleanup(st);
    }
    std::vector<std::vector<uint32_t>> gen(n);
    const size_t window = draft_window;  // the engine drafts with the decoder's window
    for (;;) {
        std::vector<uint32_t> ids;
        for (size_t i = 0; i < n; ++i)
            if (gen[i].size() < max_new_tokens[i]) ids.push_back((uint32_t)i);
        if (ids.empty()) break;
        const size_t a = ids.size();
        std::vector<const uint32_t*> ctx(a);
        std::vector<size_t> nctx(a), want(a), nd(a, 0);
        for (size_t j = 0; j < a; ++j) {
            velo_spec_session* s = sess[ids[j]];
            ctx[j] = s->context.data();
            nctx[j] = s->context.size();
            want[j] = std::min(max_new_tokens[ids[j]] - gen[ids[j]].size(), window);
        }
        std::vector<uint32_t> drafted(a * window);
        int32_t st = draft(draft_user, a, ids.data(), ctx.data(), nctx.data(), want.data(), drafted.data(), window,
                           nd.data());
        if (st) return cleanup(fail(st, "draft model failed (status %d)", st));
        for (size_t j = 0; j < a; ++j) {
            sess[ids[j]]->stats.draft_calls += 1;
            if (nd[j] > want[j])
                return cleanup(fail(VELO_ERR_DRAFT_TOO_MANY, "draft model returned %zu tokens, requested at most %zu",
                                    nd[j], want[j]));
        }
        std::vector<const uint32_t*> dp(a);
        for (size_t j = 0; j < a; ++j) dp[j] = drafted.data() + j * window;
        std::vector<uint32_t> expected(a * window);
        std::vector<size_t> nv(a, 0);
        st = verify(verify_user, a, ids.data(), ctx.data(), nctx.data(), dp.data(), nd.data(), expected.data(), window,
                    nv.data());
        if (st) return cleanup(fail(st, "target model failed (status %d)", st));
        // one target call for every active request, before any per-request
        // check can end the round (engine.rs records them the same way)
        for (size_t j = 0; j < a; ++j) sess[ids[j]]->stats.target_calls += 1;
        bool progressed = false;
        std::vector<uint32_t> acc;
        for (size_t j = 0; j < a; ++j) {
            velo_spec_session* s = sess[ids[j]];
            if (nv[j] != nd[j])
                return cleanup(fail(VELO_ERR_TARGET_WRONG_LENGTH,
                                    "target model returned %zu verification steps for %zu drafted tokens", nv[j],
                                    nd[j]));
            s->stats.drafted_tokens += nd[j];
            accept(s, dp[j], nd[j], expected.data() + j * window, &acc);
            auto& g = gen[ids[j]];
            g.insert(g.end(), acc.begin(), acc.end());
            progressed |= !acc.empty();
            if (s->pending) {
                s->pending = false;
                g.push_back(s->rejected);
                progressed = true;
            }
        }
        if (!progressed) break;
    }
    for (size_t i = 0; i < n; ++i) {
        n_out[i] = gen[i].size();
        std::copy(gen[i].begin(), gen[i].end(), out[i]);
    }
    return cleanup(VELO_OK);
}

}  // extern "C"
