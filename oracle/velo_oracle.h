/*
 * velo_oracle.h -- CPU oracle for the speculative-decoding verify step.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links, loads or
 * calls this code.  Only tests/, __graft_entry__.smoke() and the cpu_baseline
 * / --impl reference legs of bench.py use it, and only as the checker.
 *
 * It restates, in plain C, the CPU path of developertogo/velo-core:
 *   - src/quant.rs        f16 decode, interleaved q4_0 dequant, dequant_row
 *   - src/llama_cpu.rs    rms_norm, matvec_quant, silu, rope, softmax,
 *                         forward_one, forward_sequence
 *   - src/sampling.rs     GreedySampler (last maximal index wins, NaN skipped)
 *   - src/speculative.rs  SpeculativeTree::find_best_path, commit prefix rule
 *   - src/paged_attention.rs  pages_for_tokens, FIFO page allocator
 *   - src/kernels.metal   paged_attention_tree / *_int8 masking and dequant
 *                         semantics, kv_update_int8 truncating quantiser
 * and the acceptance rule that the reference does not have (rejection
 * sampling, Leviathan et al. 2023 / Chen et al. 2023) with the exact
 * arithmetic order of the product's spec, so that decisions can be compared
 * bit for bit.  Each function names the reference file:line it follows.
 *
 * Parity pins: the reference's own known-answer tests (quant.rs, llama_cpu.rs,
 * sampling.rs, speculative.rs, paged_attention.rs, metal_perf_tests.rs) are
 * re-expressed in tests/test_oracle_kats.py.  The stochastic acceptance rule,
 * tree attention over fp16/INT8 pages and the KV commit have no reference
 * implementation: parity for those is UNPINNED (checked against this
 * restatement of the named methods only).
 */
#ifndef VELO_ORACLE_H
#define VELO_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- dtypes (subset of gguf.rs GgmlType used on the verify path) ---- */
enum { VO_F32 = 0, VO_F16 = 1, VO_Q4_0 = 2 };

/* quant.rs:18-34 */
float vo_f16_to_f32(uint16_t bits);
/* IEEE round-to-nearest-even f32 -> f16 (used to build fp16 inputs) */
uint16_t vo_f32_to_f16(float x);
/* quant.rs:50-73 (interleaved nibble order: out[2i]=lo-8, out[2i+1]=hi-8) */
void vo_dequant_q4_0_row(const uint8_t *data, float *out, size_t n);
/* quant.rs:181-191 (F32, F16, Q4_0; Q4_1 maps to Q4_0; others zero-fill) */
void vo_dequant_row(int dtype, const uint8_t *data, float *out, size_t n);
size_t vo_row_bytes(int dtype, size_t cols);
/* q4_0 quantiser (own method: d = absmax/8 signed as ggml, see .c) */
void vo_quantize_q4_0_row(const float *x, size_t n, uint8_t *out);

/* llama_cpu.rs:55-146 */
void vo_rms_norm(float *x, const float *w, size_t n, float eps);
float vo_silu(float x);
void vo_rope(float *q, float *k, size_t pos, size_t n_heads, size_t n_kv_heads,
             size_t head_dim, float freq_base);
void vo_softmax(float *x, size_t n);
/* Threads a matvec's rows may be split over (1 = the reference's single
 * thread; every row stays one sequential dot product, so results do not
 * change).  Test infrastructure: the timed CPU baseline keeps 1. */
void vo_set_threads(int n);
void vo_matvec_quant(float *out, const uint8_t *data, int dtype, const float *x,
                     size_t rows, size_t cols);

/* ---- model (llama_cpu.rs:168-419) ---- */
typedef struct {
    uint32_t n_vocab, n_embd, n_layer, n_head, n_head_kv, n_ff, head_dim, n_ctx;
    float rope_freq_base, norm_eps;
} vo_meta;

/* Tensor order of the `tensors` / `dtypes` arrays:
 *   0 token_embd, 1 output_norm, 2 output (NULL => tied to token_embd),
 *   then per layer l (base 3 + 9*l): attention_norm, wq, wk, wv, wo,
 *   ffn_norm, w1, w2, w3.   Matrices are [rows][cols] row-major bytes. */
typedef struct vo_model vo_model;
vo_model *vo_model_new(const vo_meta *meta, const void *const *tensors,
                       const int *dtypes);
void vo_model_free(vo_model *m);
size_t vo_model_kv_pos(const vo_model *m);
void vo_model_set_kv_pos(vo_model *m, size_t pos);
/* llama_cpu.rs:191-358 (writes KV at pos, attends 0..pos) */
int vo_forward_one(vo_model *m, uint32_t token, size_t pos, float *logits);
/* llama_cpu.rs:363-372 */
int vo_forward_sequence(vo_model *m, const uint32_t *tokens, size_t n,
                        float *last_logits);
/* Tree verify forward with the trait contract (row n predicts the successor
 * of node n).  Node n sits at position n_cached + depth(n); it attends to the
 * cached positions [0, n_cached) and to its own root->n path.  parents[0] ==
 * -1, parents[n] < n.  Node K/V go to a tree scratch (not the cache). */
int vo_verify_tree(vo_model *m, const uint32_t *tokens, const int32_t *parents,
                   size_t n_nodes, size_t n_cached, float *logits);
/* Copy the tree-scratch K/V rows of path[0..len) into cache positions
 * n_cached.. (the commit of an accepted path). */
int vo_commit_path(vo_model *m, const int32_t *path, size_t len, size_t n_cached);
/* Read back cached K or V of one layer, positions [0, n): [n][n_kv*hd] */
int vo_write_kv(vo_model *m, int which, size_t layer, size_t pos0, size_t n, const float *src);
int vo_read_kv(const vo_model *m, int which, size_t layer, size_t n, float *out);

/* ---- sampling.rs:39-58 ---- */
uint32_t vo_greedy(const float *logits, size_t n, const uint8_t *mask,
                   float *confidence);

/* ---- speculative.rs:97-129 ----
 * Returns the number of nodes on the best path, written to path_out (root
 * first); *bonus = expected[best]. */
size_t vo_find_best_path(const int32_t *parents, const uint32_t *tokens,
                         const uint32_t *expected, size_t n, int32_t *path_out,
                         uint32_t *bonus);

/* ---- acceptance (the product's spec; greedy when temperature == 0) ----
 * tgt [B][k+1][V], drf [B][k][V] (unused when greedy), tok [B][k],
 * u [B][k+1] (u[b][i] accept uniform of position i, u[b][k] residual draw).
 * Outputs acc_len[B] (accepted draft tokens) and bonus[B]. */
int vo_accept(const float *tgt, const float *drf, const uint32_t *tok,
              const float *u, int B, int k, int V, float temperature,
              int32_t *acc_len, uint32_t *bonus, int n_threads);
/* The spec's exponential (Cody-Waite reduction + degree-6 Taylor). */
/* Rejection sampling over draft trees (multi-candidate speculative sampling,
 * SpecInfer): tgt [B][N][V] (row n = target logits after node n), drf
 * [B][N-1][V] (row n = the draft distribution node n's children were drawn
 * from), tok / parents [B][N] (node 0 = root, parents[n] < n), u [B][N]
 * (u[c-1] tests child c, u[N-1] draws the bonus).  Outputs: path [B][N]
 * (accepted nodes root first, -1 padded), path_len [B], bonus [B].
 * Chains give vo_accept's decisions.  Returns non-zero on bad input. */
int vo_accept_tree(const float *tgt, const float *drf, const uint32_t *tok,
                   const int32_t *parents, const float *u, int B, int N, int V,
                   float temperature, int32_t *path, int32_t *path_len, uint32_t *bonus);
float vo_spec_exp(float y);
/* Row statistics of the spec: M (scaled max) and Z (normaliser). */
void vo_row_stats(const float *row, int V, float inv_t, float *M, float *Z);

/* ---- paged_attention.rs:92-211 ---- */
size_t vo_pages_for_tokens(size_t tokens, size_t block_size);
typedef struct vo_allocator vo_allocator;
vo_allocator *vo_allocator_new(size_t block_size, size_t total_pages);
void vo_allocator_free(vo_allocator *a);
/* 0 ok; 1 OutOfPages (requested/available written); pages_out gets ids */
int vo_allocator_allocate(vo_allocator *a, uint64_t handle, size_t token_len,
                          uint32_t *pages_out, size_t *n_pages,
                          size_t *requested, size_t *available);
int vo_allocator_release(vo_allocator *a, uint64_t handle);
size_t vo_allocator_free_pages(const vo_allocator *a);

/* ---- KV page pool (product layout) ----
 * pool  [total_pages][n_kv][page][hd]   element = f16 (kv_dtype 0) or i8 (1)
 * scale [total_pages][n_kv][page]       f16, INT8 only
 * Tree attention semantics follow kernels.metal:512-599 (prefix then the
 * node's ancestors), with the node's own K/V included (trait contract). */
enum { VO_KV_F16 = 0, VO_KV_I8 = 1 };
void vo_tree_attention(const float *q, int kv_dtype, const void *k_pool,
                       const void *v_pool, const uint16_t *k_scale,
                       const uint16_t *v_scale, const uint32_t *page_table,
                       size_t n_cached, const uint16_t *k_nodes,
                       const uint16_t *v_nodes, const int32_t *parents,
                       size_t n_nodes, size_t n_head, size_t n_kv, size_t hd,
                       size_t page_size, float *out);
/* kernels.metal:753-802 quantiser, fp16 scale: scale = max|x|/127,
 * q = trunc(x * (127/max)).  x: hd floats. */
void vo_quantize_kv_int8(const float *x, size_t hd, int8_t *q, uint16_t *scale);
/* KV commit: write node rows path[0..len) (f16 [n_nodes][n_kv][hd]) at
 * positions n_cached.. through the page table.  Returns 0, or 5 when a
 * position falls outside the n_bound bound pages. */
int vo_kv_commit(int kv_dtype, void *pool, uint16_t *scale,
                 const uint32_t *page_table, size_t n_bound, size_t n_cached,
                 const uint16_t *node_kv, const int32_t *path, size_t len,
                 size_t n_kv, size_t hd, size_t page_size);

/* ---- sharding.rs:28-126 (tensor parallelism) ----
 * strategy: 0 replicated, 1 column (split rows = output features), 2 row
 * (split cols = input features; q4_0 blocks of 32).  Returns 0, or 1 with the
 * reference's divisibility errors.  out holds the shard, rows_out / cols_out
 * its shape. */
int vo_shard_strategy(const char *name);
int vo_shard_weight(int dtype, const uint8_t *data, size_t rows, size_t cols, int strategy,
                    int tp, int rank, uint8_t *out, size_t *rows_out, size_t *cols_out);

#ifdef __cplusplus
}
#endif
#endif
