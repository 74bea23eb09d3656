/*
 * velo_session.h -- the speculative-decoding session loop in native code.
 *
 * Replaces SpeculativeDecoder / SpeculativeSession (src/speculative.rs:
 * 255-537) for a host that is not Rust: the same window rule, accept rule,
 * statistics and errors (SpeculativeError, :294-305 -> velo_status codes 2-4),
 * with the draft and target models supplied as callbacks.  A callback that
 * returns non-zero aborts the call with that status (SpeculativeError::Model).
 * Host only; the models decide where they run (the velo_cuda verify step for
 * the B200 path).
 */
#ifndef VELO_SESSION_H
#define VELO_SESSION_H

#include "velo_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* SpeculativeStats (speculative.rs:285-291) */
typedef struct velo_spec_stats {
    uint64_t draft_calls, target_calls, drafted_tokens, accepted_tokens, rejected_tokens;
} velo_spec_stats;

/* DraftModel::draft: up to max_tokens predicted tokens after `context`,
 * written to out (room for out_cap), their count to *n_out.  A count above
 * max_tokens is DraftReturnedTooMany. */
typedef int32_t (*velo_draft_fn)(void *user, const uint32_t *context, size_t n_context, size_t max_tokens,
                                 uint32_t *out, size_t out_cap, size_t *n_out);

/* TargetModel::verify: for each i the target's token after context +
 * drafted[:i] (VerifyStep::expected), written to out (room for out_cap), the
 * count to *n_out.  A count other than n_drafted is TargetReturnedWrongLength. */
typedef int32_t (*velo_verify_fn)(void *user, const uint32_t *context, size_t n_context, const uint32_t *drafted,
                                  size_t n_drafted, uint32_t *out, size_t out_cap, size_t *n_out);

typedef struct velo_spec_session velo_spec_session;

/* SpeculativeDecoder::new / with_max_window + begin: VELO_ERR_EMPTY_DRAFT_WINDOW
 * when draft_window is 0 or max_window < draft_window (max_window 0 = twice
 * the draft window). */
VELO_API int32_t velo_spec_session_create(uint32_t draft_window, uint32_t max_window, const uint32_t *prompt,
                                          size_t n_prompt, velo_spec_session **out);
VELO_API void velo_spec_session_destroy(velo_spec_session *s);

/* SpeculativeSession::draft (:400-471): one draft + verify round of at most
 * min(max_new_tokens, window) tokens; the accepted tokens go to `accepted`
 * (room for cap).  A rejection leaves the target's token pending. */
VELO_API int32_t velo_spec_session_draft(velo_spec_session *s, velo_draft_fn draft, void *draft_user,
                                         velo_verify_fn verify, void *verify_user, size_t max_new_tokens,
                                         uint32_t *accepted, size_t cap, size_t *n_accepted);

/* SpeculativeSession::commit (:473-519): apply an externally run round. */
VELO_API int32_t velo_spec_session_commit(velo_spec_session *s, const uint32_t *drafted, size_t n_drafted,
                                          const uint32_t *verified, size_t n_verified, uint32_t *accepted,
                                          size_t cap, size_t *n_accepted);

/* take_rejected_token: 1 and the token when one is pending, else 0. */
VELO_API int32_t velo_spec_session_take_rejected(velo_spec_session *s, uint32_t *token);
VELO_API int32_t velo_spec_session_has_pending_rejection(const velo_spec_session *s);
/* The session's context (prompt + committed tokens): its length; the first
 * min(length, cap) tokens are copied to out (may be NULL). */
VELO_API size_t velo_spec_session_context(const velo_spec_session *s, uint32_t *out, size_t cap);
VELO_API uint32_t velo_spec_session_window(const velo_spec_session *s);
VELO_API void velo_spec_session_stats(const velo_spec_session *s, velo_spec_stats *out);
VELO_API void velo_spec_session_record_draft_call(velo_spec_session *s);
VELO_API void velo_spec_session_record_target_call(velo_spec_session *s);

/* SpeculativeDecoder::generate (:325-361): rounds until max_new_tokens are
 * out or the draft model stops; out needs room for max_new_tokens. */
VELO_API int32_t velo_spec_generate(uint32_t draft_window, uint32_t max_window, velo_draft_fn draft,
                                    void *draft_user, velo_verify_fn verify, void *verify_user,
                                    const uint32_t *prompt, size_t n_prompt, size_t max_new_tokens, uint32_t *out,
                                    size_t cap, size_t *n_out, velo_spec_stats *stats);

/* DraftModel::draft_batch for n requests: request i has id ids[i], context
 * contexts[i] (n_context[i] tokens) and may take up to max_tokens[i] tokens,
 * written at out + i * out_stride (out_stride >= every max_tokens[i]) with
 * the count in n_out[i]. */
typedef int32_t (*velo_draft_batch_fn)(void *user, size_t n, const uint32_t *ids, const uint32_t *const *contexts,
                                       const size_t *n_context, const size_t *max_tokens, uint32_t *out,
                                       size_t out_stride, size_t *n_out);
/* TargetModel::verify_batch for n requests: expected tokens of request i at
 * out + i * out_stride, count in n_out[i]. */
typedef int32_t (*velo_verify_batch_fn)(void *user, size_t n, const uint32_t *ids, const uint32_t *const *contexts,
                                        const size_t *n_context, const uint32_t *const *drafted,
                                        const size_t *n_drafted, uint32_t *out, size_t out_stride, size_t *n_out);

/* VeloEngine::generate_batch (src/engine.rs:233-420): every round, each
 * request short of max_new_tokens[i] drafts min(remaining, draft_window)
 * tokens (the decoder's fixed window), one verify_batch call covers all of
 * them, each session commits and emits the target's token at a rejection.
 * Request i has id i (its slot); more than max_slots requests (0: no limit)
 * is VELO_ERR_INVALID_ARGUMENT, as the engine's SlotPool running dry.  A
 * round without progress ends the loop.  A draft count above max_tokens[i]
 * is DraftReturnedTooMany here (the reference engine would verify the
 * surplus).  out[i] needs room for max_new_tokens[i]; stats (or NULL) is [n]. */
VELO_API int32_t velo_spec_generate_batch(uint32_t draft_window, uint32_t max_window, size_t max_slots,
                                          velo_draft_batch_fn draft, void *draft_user, velo_verify_batch_fn verify,
                                          void *verify_user, size_t n, const uint32_t *const *prompts,
                                          const size_t *n_prompt, const size_t *max_new_tokens,
                                          uint32_t *const *out, size_t *n_out, velo_spec_stats *stats);

#ifdef __cplusplus
}
#endif

#endif /* VELO_SESSION_H */
