/*
 * velo_cuda.h -- C ABI of the B200 (sm_100a) speculative-decoding verify step.
 *
 * This is the drop-in boundary a velo-core backend binds from Rust with an
 * `extern "C"` block.  Plain pointers and sizes only; no
 * CUDA or torch types appear in any signature.  Device pointers are passed as
 * `void*` / typed pointers to device memory and are documented as such.
 *
 * Conventions (mirroring the reference):
 *   - Every entry returns velo_status (int32): 0 = OK.  Codes mirror
 *     SpeculativeError (src/speculative.rs:294-305) and PageManagerError
 *     (src/paged_attention.rs:72-79).  velo_cuda_last_error() returns the
 *     message of the last failure on the calling thread.
 *   - Host arrays are caller-owned and only read (inputs) or written
 *     (outputs) during the call.  Output arrays are caller-allocated.
 *   - A context owns one CUDA stream and its device buffers.  Contexts are not
 *     thread-safe (the reference backends take `&mut self`).
 */
#ifndef VELO_CUDA_H
#define VELO_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VELO_CUDA_ABI_VERSION 2

#if defined(__GNUC__)
#define VELO_API __attribute__((visibility("default")))
#else
#define VELO_API
#endif

typedef enum velo_status {
    VELO_OK = 0,
    VELO_ERR_INVALID_ARGUMENT = 1,     /* SpeculativeError::Model("...") for bad input */
    VELO_ERR_EMPTY_DRAFT_WINDOW = 2,   /* SpeculativeError::EmptyDraftWindow */
    VELO_ERR_DRAFT_TOO_MANY = 3,       /* SpeculativeError::DraftReturnedTooMany */
    VELO_ERR_TARGET_WRONG_LENGTH = 4,  /* SpeculativeError::TargetReturnedWrongLength */
    VELO_ERR_OUT_OF_PAGES = 5,         /* PageManagerError::OutOfPages */
    VELO_ERR_UNKNOWN_HANDLE = 6,       /* PageManagerError::UnknownHandle */
    VELO_ERR_INVALID_BLOCK_SIZE = 7,   /* PageManagerError::InvalidBlockSize */
    VELO_ERR_CUDA = 8,                 /* a CUDA runtime call failed */
    VELO_ERR_NO_DEVICE = 9,            /* no usable sm_100 device */
    VELO_ERR_TIMEOUT = 10,             /* velo_cuda_sync deadline passed */
    VELO_ERR_OUT_OF_MEMORY = 11,
    VELO_ERR_NCCL = 12,
    VELO_ERR_DEVICE_FLAG = 13,         /* a kernel reported a bad input on device */
    VELO_ERR_IO = 14,                  /* LoadError::Io / GgufError::Io (open, short read) */
    VELO_ERR_GGUF = 15,                /* GgufError::{BadMagic, UnsupportedVersion, UnknownType, Malformed} */
    VELO_ERR_MISSING_META = 16,        /* LoadError::MissingMeta */
    VELO_ERR_MISSING_TENSOR = 17,      /* LoadError::MissingTensor */
    VELO_ERR_INVALID_SHAPE = 18        /* LoadError::InvalidShape */
} velo_status;

typedef struct velo_cuda_ctx velo_cuda_ctx;

/* Mirrors MemoryRuntimeConfig (src/runtime.rs:46-61) / EngineConfig
 * (src/engine.rs:60-67) / MetalBackendConfig (src/metal/config.rs:7-22) for
 * what the verify step needs.  Zero fields take the defaults in brackets. */
typedef struct velo_cuda_config {
    uint32_t struct_size;  /* sizeof(velo_cuda_config) */
    uint32_t page_size;    /* tokens per KV page [16] (PagedAttentionConfig::block_size) */
    uint32_t kv_dtype;     /* velo_kv_dtype [VELO_KV_F16] */
    uint32_t max_slots;    /* page-table rows [1] */
    uint32_t total_pages;  /* pages in the pool [0: no KV pool] */
    uint32_t max_pages_per_slot; /* page-table width [total_pages] */
} velo_cuda_config;

/* KV page element type.  VELO_KV_F32 selects the fp32 path of the model: f32
 * pages (the reference's f32 KvCache, src/llama_cpu.rs:22-50), weights of any
 * dtype dequantised to f32 at load, every op in f32 (logits within 1e-4 of
 * LlamaCpuModel); F16 / INT8 pages run q4_0 weights on the tensor cores. */
typedef enum velo_kv_dtype { VELO_KV_F16 = 0, VELO_KV_INT8 = 1, VELO_KV_F32 = 2 } velo_kv_dtype;

/* ---- lifecycle ---------------------------------------------------------- */

/* Create a context on `device` (CUDA ordinal).  tp_rank / tp_size give the
 * tensor-parallel position (1 GPU: 0 / 1); nccl_unique_id (128 bytes) is
 * required when tp_size > 1 and ignored otherwise.
 * Replaces constructing MetalMemoryRuntime + MetalBackend
 * (src/metal/runtime.rs, src/metal/backend.rs:115-286). */
VELO_API int32_t velo_cuda_create(const velo_cuda_config *cfg, int32_t device, int32_t tp_rank,
                         int32_t tp_size, const void *nccl_unique_id,
                         velo_cuda_ctx **out);
VELO_API void velo_cuda_destroy(velo_cuda_ctx *ctx);

/* Write a fresh NCCL unique id (128 bytes) to `out`: rank 0 of a tensor-
 * parallel group makes one and hands it to every rank's velo_cuda_create,
 * which all ranks call concurrently (one host thread or process per GPU).
 * No counterpart in the reference, whose TP all-reduce runs on the CPU
 * (src/metal/tp_model.rs:199-277). */
VELO_API int32_t velo_cuda_nccl_unique_id(void *out);

/* Message of the last failure on the calling thread ("" if none). */
VELO_API const char *velo_cuda_last_error(void);
VELO_API int32_t velo_cuda_abi_version(void);

/* Use `stream` (a cudaStream_t, may be NULL for the context's own stream) for
 * all following asynchronous work of this context. */
VELO_API int32_t velo_cuda_set_stream(velo_cuda_ctx *ctx, void *stream);

/* Wait for the context's stream, giving up after timeout_ns (<0: forever).
 * Returns VELO_ERR_TIMEOUT instead of hanging; also reports a device-side
 * input flag raised by an earlier kernel (VELO_ERR_DEVICE_FLAG). */
VELO_API int32_t velo_cuda_sync(velo_cuda_ctx *ctx, int64_t timeout_ns);

/* ---- acceptance --------------------------------------------------------- */

/* Fused vocabulary-wide softmax + acceptance for linear drafts.
 *
 * Replaces the host loop GreedyTargetModel::verify_batch + GreedySampler
 * (src/backend.rs:337-369, src/sampling.rs:39-58) followed by the prefix rule
 * of SpeculativeSession::draft / commit (src/speculative.rs:441-467, 473-519).
 *
 *   target_logits [B][k+1][V] f32: row i is the target's distribution after
 *                 draft position i-1 (row 0 after the last committed token).
 *   draft_logits  [B][k][V]   f32: row i is the distribution draft token i was
 *                 drawn from (unused, may be NULL, when temperature == 0).
 *   draft_tokens  [B][k]  u32, each < V.
 *   uniforms      [B][k+1] f32 in [0,1): u[b][i] for the accept test of
 *                 position i, u[b][k] for the residual / bonus draw.
 *   temperature   0 => greedy (accept while token == argmax, last maximal
 *                 index wins as GreedySampler), > 0 => rejection sampling:
 *                 accept x_i iff u_i * q(x_i) <= p(x_i); at the first
 *                 rejection draw from norm(max(0, p - q)); if all k are
 *                 accepted draw the bonus from p of row k.
 *   accepted_len  [B] i32 out: accepted draft tokens (0..k).
 *   bonus_token   [B] u32 out: the token emitted after the accepted prefix.
 *
 * Host-buffer form: copies inputs to the device, runs, copies outputs back and
 * waits.  Pinned host memory gives the fastest copies. */
VELO_API int32_t velo_cuda_accept(velo_cuda_ctx *ctx, const float *target_logits,
                         const float *draft_logits, const uint32_t *draft_tokens,
                         const float *uniforms, int32_t B, int32_t k, int32_t V,
                         float temperature, int32_t *accepted_len,
                         uint32_t *bonus_token);

/* Device-buffer form of velo_cuda_accept: every pointer is device memory;
 * asynchronous on the context stream.  Intermediate statistics live in a
 * workspace the context allocates and keeps. */
VELO_API int32_t velo_cuda_accept_device(velo_cuda_ctx *ctx, const float *target_logits,
                                const float *draft_logits, const uint32_t *draft_tokens,
                                const float *uniforms, int32_t B, int32_t k, int32_t V,
                                float temperature, int32_t *accepted_len,
                                uint32_t *bonus_token);

/* Allocation-free form of velo_cuda_accept_device, for callers that must not
 * allocate device memory on this path (an engine that owns all of HBM through
 * its own pools, or a latency-critical loop where cudaMalloc would
 * synchronise).  No counterpart in the reference: velo-core has no device-side
 * acceptance.  Needs no context: runs on the calling thread's current device
 * and on `stream` (a cudaStream_t; NULL = default stream), asynchronously.
 * Inputs and outputs are caller-provided device buffers; intermediate
 * statistics live in a fixed 4 MiB block of device memory inside the library
 * (one per GPU, held until process exit), so it allocates nothing.  Sizes
 * whose statistics exceed that block (roughly B*(2k+1)*ceil(V/1024) > 250k)
 * are rejected with VELO_ERR_INVALID_ARGUMENT.  The first call on each device
 * looks up the block's address; make it before any stream capture.  All calls
 * on a device share the block: calls that overlap on the GPU race and must be
 * serialised by the caller. */
VELO_API int32_t velo_cuda_accept_static(const float *target_logits, const float *draft_logits,
                                         const uint32_t *draft_tokens, const float *uniforms,
                                         int32_t B, int32_t k, int32_t V, float temperature,
                                         int32_t *accepted_len, uint32_t *bonus_token,
                                         void *stream);

/* The input check of the last velo_cuda_accept_static call on the current
 * device: copies its error word (0 = clean; non-zero = a draft token was >= V
 * and was counted as a rejection, which velo_cuda_accept_device reports as
 * VELO_ERR_DEVICE_FLAG at velo_cuda_sync) into *flag_out, a device int32, on
 * `stream`, asynchronously and without allocating.  Issue it on the stream of
 * the call it checks, before the next velo_cuda_accept_static, which clears
 * the word.  No counterpart in the reference (velo-core has no device-side
 * acceptance). */
VELO_API int32_t velo_cuda_accept_static_error(int32_t *flag_out, void *stream);

/* Rejection sampling over draft trees (temperature > 0).  Multi-candidate
 * speculative sampling (SpecInfer, Miao et al. 2024): from the root, the
 * children of the current node are tested in index order, child c with
 * token x accepted iff u[c-1] * q(x) <= p(x); after each rejected child p is
 * replaced by norm(max(0, p - q)); the walk moves to the first accepted child;
 * at a node with no accepted child (or a leaf) the bonus token is drawn from
 * the current p with u[N-1].  On chains this is velo_cuda_accept's rule, bit
 * for bit.  Extends the greedy tree walk of SpeculativeTree::find_best_path
 * (src/speculative.rs:97-129) over trees built by TreeDraftModel::draft_tree
 * (src/backend.rs:255-294), which the reference only verifies greedily.
 *   target_logits [B][N][V] f32: row n = the target's logits after node n
 *   draft_logits  [B][N-1][V] f32: row n = the draft distribution node n's
 *                 children were drawn from (node N-1 has no children)
 *   tokens, parents [B][N]: node 0 is the root (-1), parents[n] < n
 *   uniforms      [B][N] in [0,1)
 *   path [B][N] out: accepted nodes root first, -1 padded; path_len [B] out
 *   (root included); bonus [B] out.
 * Host-buffer form: copies in, runs, copies back and waits. */
VELO_API int32_t velo_cuda_accept_tree(velo_cuda_ctx *ctx, const float *target_logits,
                                       const float *draft_logits, const uint32_t *tokens,
                                       const int32_t *parents, const float *uniforms, int32_t B,
                                       int32_t N, int32_t V, float temperature, int32_t *path,
                                       int32_t *path_len, uint32_t *bonus);

/* Device-buffer form of velo_cuda_accept_tree (every pointer device memory),
 * asynchronous on the context stream; a token >= V is counted as a rejection
 * and reported by velo_cuda_sync (VELO_ERR_DEVICE_FLAG). */
VELO_API int32_t velo_cuda_accept_tree_device(velo_cuda_ctx *ctx, const float *target_logits,
                                              const float *draft_logits, const uint32_t *tokens,
                                              const int32_t *parents, const float *uniforms,
                                              int32_t B, int32_t N, int32_t V, float temperature,
                                              int32_t *path, int32_t *path_len, uint32_t *bonus);

/* ---- q4_0 linear layers ------------------------------------------------- */

/* Epilogues of velo_cuda_gemm_q4_0 (y has row stride ldy elements). */
typedef enum velo_gemm_epilogue {
    VELO_EPI_STORE_F32 = 0, /* y[m][n] = acc                       f32 */
    VELO_EPI_STORE_F16 = 1, /* y[m][n] = acc                       f16 */
    VELO_EPI_ADD_F32 = 2,   /* y[m][n] += acc (residual stream)    f32 */
    VELO_EPI_SWIGLU = 3,    /* y[m][j] = silu(gate_j) * up_j        f16, j < N/2 */
    VELO_EPI_STORE_BF16 = 4 /* y[m][n] = acc                       bf16 */
} velo_gemm_epilogue;

/* Device bytes of a repacked q4_0 weight with N rows of K elements (0 if
 * K is not a positive multiple of 32). */
VELO_API size_t velo_cuda_q4_0_repacked_bytes(int32_t N, int32_t K);

/* Repack q4_0 rows as velo-core stores them ([N][K/32] blocks of 18 bytes:
 * fp16 scale d, then 16 bytes whose byte i holds element 2i (low nibble) and
 * 2i+1 (high nibble), value d * (q - 8); src/quant.rs:50-64) into the tiled
 * layout the tensor-core GEMM streams.  src / src_b / dst are device memory.
 * With src_b != NULL the weight is a SwiGLU pair: src holds the N/2 gate rows
 * (ffn w1) and src_b the N/2 up rows (ffn w3), for VELO_EPI_SWIGLU.
 * Asynchronous on the context stream.  Replaces the per-row dequant_row of
 * matvec_quant (src/llama_cpu.rs:75-90), done once at load instead. */
VELO_API int32_t velo_cuda_q4_0_repack(velo_cuda_ctx *ctx, const void *src, const void *src_b,
                                       int32_t N, int32_t K, void *dst);

/* Y = X * W^T on the tensor cores: X f16 [M][K] (device, 16-byte aligned,
 * row stride K), W a repacked q4_0 weight of N rows, fp32 accumulation, then
 * the epilogue `mode` (velo_gemm_epilogue).  Asynchronous on the context
 * stream.  Replaces matvec_quant (src/llama_cpu.rs:75-90) for all M rows of a
 * verify step at once. */
VELO_API int32_t velo_cuda_gemm_q4_0(velo_cuda_ctx *ctx, const void *w_repacked, const void *x,
                                     int32_t M, int32_t N, int32_t K, void *y, int32_t ldy,
                                     int32_t mode);

/* ---- tree-masked paged attention ---------------------------------------- */

/* Attention of every draft-tree node over the sequence's cached KV pages and
 * its own root->node path, on the tensor cores.  All pointers are device
 * memory; asynchronous on the context stream.
 *   q         [B][n_nodes][n_head][head_dim] f16 (RoPE applied)
 *   k_pool, v_pool  [pool_pages][n_kv][16][head_dim], f16 (kv_dtype
 *             VELO_KV_F16) or int8 (VELO_KV_INT8, value = q * scale)
 *   k_scale, v_scale  [pool_pages][n_kv][16] f16 per-token-per-head scales
 *             (INT8 only, else NULL)
 *   page_table [B][max_pages] u32 page ids; ctx_len [B] cached tokens
 *   node_k, node_v  [B][n_nodes][n_kv][head_dim] f16: K/V of the tree nodes
 *   parents   [B][n_nodes] i32, -1 for the root, parents[n] < n
 *   out       [B][n_nodes][n_head][head_dim], f32 (out_dtype 0) or f16 (1)
 * Node n attends to cached tokens [0, ctx_len) and to the nodes on its
 * root->n path (itself included); scale 1/sqrt(head_dim); GQA head
 * h -> h / (n_head / n_kv).  head_dim must be 128, n_nodes <= 64.  Pools
 * must hold finite values in every slot a page table names (zero-initialise
 * them), since masked keys still pass through the tensor cores with weight 0.
 * Replaces paged_attention_tree / paged_attention_flash_int8
 * (src/kernels.metal:512-599, 672-732) driven by LlamaMetalModel::forward_tree
 * (src/metal/model.rs:574-731). */
VELO_API int32_t velo_cuda_tree_attention(velo_cuda_ctx *ctx, const void *q, const void *k_pool,
                                          const void *v_pool, const void *k_scale,
                                          const void *v_scale, int32_t pool_pages,
                                          const uint32_t *page_table, int32_t max_pages,
                                          const int32_t *ctx_len, const void *node_k,
                                          const void *node_v, const int32_t *parents, int32_t B,
                                          int32_t n_nodes, int32_t n_head, int32_t n_kv,
                                          int32_t head_dim, int32_t kv_dtype, void *out,
                                          int32_t out_dtype);

/* ---- model, KV pages and the verify step -------------------------------- */

typedef enum velo_dtype { VELO_DT_F32 = 0, VELO_DT_F16 = 1, VELO_DT_Q4_0 = 2 } velo_dtype;

/* The Llama hyper-parameters the verify step needs (ModelMeta,
 * src/model_loader.rs:21-37).  head_dim 128 (64 or 128 on the fp32 path). */
typedef struct velo_model_desc {
    uint32_t struct_size;  /* sizeof(velo_model_desc) */
    uint32_t n_vocab, n_embd, n_layer, n_head, n_head_kv, n_ff, head_dim;
    float rope_freq_base, norm_eps;
} velo_model_desc;

/* One named tensor of the WeightStore (src/model_loader.rs:192-234): names
 * "token_embd.weight", "output_norm.weight", "output.weight" (optional: tied
 * to token_embd), "layers.{l}.attention_norm.weight",
 * "layers.{l}.attention.w{q,k,v,o}.weight", "layers.{l}.ffn_norm.weight",
 * "layers.{l}.feed_forward.w{1,2,3}.weight".  data is host memory, rows x
 * cols row-major (rows = output features; q4_0 rows are cols/32 blocks of 18
 * bytes, quant.rs:50-64).  Matrices must be q4_0; embeddings and norms may be
 * f32, f16 or q4_0. */
typedef enum velo_weight_flags {
    VELO_WEIGHT_DEVICE = 1, /* data is device memory of the context's GPU (else host memory) */
    VELO_WEIGHT_SHARD = 2   /* the tensor is already this rank's shard (sharding.rs applied) */
} velo_weight_flags;

typedef struct velo_weight_desc {
    const char *name;
    int32_t dtype;   /* velo_dtype */
    uint32_t flags;  /* velo_weight_flags (0: a host tensor, sharded by the context) */
    const void *data;
    uint64_t rows, cols;
} velo_weight_desc;

/* Tensor-parallel sharding on the host (src/metal/sharding.rs:28-126). */
typedef enum velo_shard_strategy {
    VELO_SHARD_REPLICATED = 0,
    VELO_SHARD_COLUMN = 1, /* split the output rows */
    VELO_SHARD_ROW = 2     /* split the input columns (q4_0: on 32-element blocks) */
} velo_shard_strategy;

/* get_shard_strategy (sharding.rs:112-126): q/k/v, w1/w3 and output.weight
 * Column, wo and w2 Row, everything else Replicated. */
VELO_API int32_t velo_cuda_shard_strategy(const char *name);

/* shard_weight (sharding.rs:28-110) of a host tensor for `rank` of `tp`:
 * copies the shard to `out` (out_bytes large enough) and writes its shape.
 * Same divisibility errors as the reference (VELO_ERR_INVALID_ARGUMENT). */
VELO_API int32_t velo_cuda_shard_weight(const velo_weight_desc *w, int32_t strategy, int32_t tp,
                                        int32_t rank, void *out, size_t out_bytes,
                                        uint64_t *out_rows, uint64_t *out_cols);

/* Upload and repack a model (the context then owns the device copies) and
 * allocate the zero-filled paged KV pool of the context's config (total_pages
 * x n_layer, kv_dtype) and its page table (max_slots x max_pages_per_slot).
 * With tp_size > 1 every rank passes the full tensors and keeps its shard
 * (velo_cuda_shard_weight), or passes its shards (VELO_WEIGHT_SHARD); its pool
 * holds its n_head_kv / tp_size heads.  Device tensors (VELO_WEIGHT_DEVICE)
 * are repacked in place of a host upload; with tp_size > 1 they must be shards.
 * Replaces LlamaCpuModel::from_weights / LlamaMetalModel::new and
 * MetalMemoryRuntime::new (src/llama_cpu.rs:168-190, src/metal/runtime.rs). */
VELO_API int32_t velo_cuda_load_model(velo_cuda_ctx *ctx, const velo_model_desc *desc,
                                      const velo_weight_desc *weights, int32_t n_weights);

/* Bind `slot` (a page-table row) to `pages` (n_pages ids < total_pages); the
 * rest of the row is zeroed.  MemoryRuntime::bind_slot (src/runtime.rs:36,
 * src/metal/runtime.rs:294-319).  VELO_ERR_OUT_OF_PAGES when n_pages exceeds
 * the row or an id exceeds the pool. */
VELO_API int32_t velo_cuda_bind_slot(velo_cuda_ctx *ctx, uint32_t slot, const uint32_t *pages,
                                     size_t n_pages);

/* The context's own page allocator over its KV pool (block size = the page
 * size, total_pages of the config), created by velo_cuda_load_model: one call
 * in place of PagedAttentionBlockManager::allocate + MemoryRuntime::bind_slot
 * (src/paged_attention.rs:155-186, src/runtime.rs:36).  Takes
 * ceil(token_len / page_size) pages for handle `slot` and binds the slot's
 * page-table row to them (the ids are also written to pages_out, or NULL).
 * VELO_ERR_OUT_OF_PAGES when the pool is short (nothing taken) or the row
 * is too small.  Allocating a slot that holds pages replaces its mapping
 * without freeing the old pages, as the reference does.  A context either
 * allocates every slot here or binds every slot itself (velo_cuda_bind_slot),
 * not both. */
VELO_API int32_t velo_cuda_slot_allocate(velo_cuda_ctx *ctx, uint32_t slot, size_t token_len,
                                         uint32_t *pages_out, size_t pages_cap, size_t *n_pages);

/* Return a slot's pages to the back of the free list
 * (PagedAttentionBlockManager::release, src/paged_attention.rs:189-198) and
 * fill its page-table row with an invalid id, so a later step on the slot is
 * reported (VELO_ERR_DEVICE_FLAG) instead of touching pages it no longer
 * owns.  VELO_ERR_UNKNOWN_HANDLE for a slot that holds no allocation. */
VELO_API int32_t velo_cuda_slot_release(velo_cuda_ctx *ctx, uint32_t slot);

/* Free pages left in the context's allocator (free_pages, :201-203). */
VELO_API int32_t velo_cuda_free_pages(velo_cuda_ctx *ctx, size_t *out);

/* The same allocator without a context or a GPU (host only), for a host that
 * manages several pools or wants the page ids before it creates a context.
 * create: VELO_ERR_INVALID_BLOCK_SIZE for block_size 0 (:103-106).
 * allocate: OutOfPages writes requested / available (either may be NULL);
 * pages_out (or NULL) must hold the pages needed.  mapped_pages:
 * VELO_ERR_UNKNOWN_HANDLE when the handle holds nothing. */
typedef struct velo_page_allocator velo_page_allocator;
VELO_API int32_t velo_page_allocator_create(size_t block_size, size_t total_pages,
                                            velo_page_allocator **out);
VELO_API void velo_page_allocator_destroy(velo_page_allocator *a);
VELO_API int32_t velo_page_allocator_allocate(velo_page_allocator *a, uint64_t handle, size_t token_len,
                                              uint32_t *pages_out, size_t pages_cap, size_t *n_pages,
                                              size_t *requested, size_t *available);
VELO_API int32_t velo_page_allocator_release(velo_page_allocator *a, uint64_t handle);
VELO_API int32_t velo_page_allocator_mapped_pages(const velo_page_allocator *a, uint64_t handle,
                                                  uint32_t *pages_out, size_t pages_cap, size_t *n_pages);
VELO_API size_t velo_page_allocator_free_pages(const velo_page_allocator *a);
VELO_API size_t velo_page_allocator_pages_for_tokens(const velo_page_allocator *a, size_t token_len);

/* ---- GGUF model files (host only, no GPU) -------------------------------- */

/* A parsed GGUF file whose tensor data stays memory-mapped until
 * velo_gguf_close.  open = GgufFile::read + read_all_tensors (src/gguf.rs:
 * 227-320): VELO_ERR_IO (missing file, short data), VELO_ERR_GGUF (bad magic,
 * version not 1..3, unknown value or ggml type, more than 4 dims, bad UTF-8). */
typedef struct velo_gguf velo_gguf;
VELO_API int32_t velo_gguf_open(const char *path, velo_gguf **out);
VELO_API void velo_gguf_close(velo_gguf *g);
VELO_API uint32_t velo_gguf_version(const velo_gguf *g);
VELO_API uint64_t velo_gguf_n_tensors(const velo_gguf *g);
VELO_API uint64_t velo_gguf_n_metadata(const velo_gguf *g);
VELO_API uint64_t velo_gguf_data_offset(const velo_gguf *g);

/* One metadata value (GgufValue, gguf.rs:103-118).  type: the GGUF value type
 * id (0 u8 .. 12 f64); integers in u (unsigned, bool) or i (signed), floats
 * in f, strings in s / s_len (owned by g, not NUL-safe), arrays give
 * array_type and array_len (elements via velo_gguf_metadata_elem). */
typedef struct velo_gguf_value {
    int32_t type, array_type;
    uint64_t u;
    int64_t i;
    double f;
    const char *s;
    uint64_t s_len, array_len;
} velo_gguf_value;
/* VELO_ERR_MISSING_META when the key is absent. */
VELO_API int32_t velo_gguf_metadata(const velo_gguf *g, const char *key, velo_gguf_value *out);
VELO_API int32_t velo_gguf_metadata_elem(const velo_gguf *g, const char *key, uint64_t index,
                                         velo_gguf_value *out);

/* TensorInfo (gguf.rs:198-207): shape as stored (innermost first), data
 * points into the mapping.  VELO_ERR_MISSING_TENSOR when absent. */
typedef struct velo_gguf_tensor {
    int32_t ggml_type;
    uint32_t n_dims;
    uint64_t shape[4];
    uint64_t offset, nbytes;
    const void *data;
} velo_gguf_tensor;
VELO_API int32_t velo_gguf_tensor_info(const velo_gguf *g, const char *name, velo_gguf_tensor *out);

/* ModelMeta::from_gguf (src/model_loader.rs:41-127): the velo_model_desc of
 * the file plus arch, n_ctx and the inferred quantization (0 Q4_0, 1 Q4K;
 * :143-153).  VELO_ERR_MISSING_META names the absent key. */
typedef struct velo_gguf_model_meta {
    uint32_t struct_size;  /* sizeof(velo_gguf_model_meta) */
    velo_model_desc desc;
    uint32_t n_ctx;
    int32_t quantization;
    char arch[64];
} velo_gguf_model_meta;
VELO_API int32_t velo_gguf_read_model_meta(const velo_gguf *g, velo_gguf_model_meta *out);

/* WeightStore::validate (:192-234): every tensor of the Llama layout with the
 * reference's shapes, in the reference's order (VELO_ERR_MISSING_TENSOR,
 * VELO_ERR_INVALID_SHAPE). */
VELO_API int32_t velo_gguf_validate(const velo_gguf *g);

/* The weight descriptors velo_cuda_load_model takes, pointing into the
 * mapping (valid until velo_gguf_close): the validated tensors, rows = the
 * second stored dimension (1 for vectors), cols = the first.  F32, F16 and
 * q4_0 tensors only (VELO_ERR_INVALID_ARGUMENT names another type).  q4_0
 * bytes are used as stored, with the reference's element order
 * (src/quant.rs:50-73).  *n gets the count; out may be NULL to ask it. */
VELO_API int32_t velo_gguf_weights(const velo_gguf *g, velo_weight_desc *out, int32_t cap, int32_t *n);

/* load_gguf (:291-309) then velo_cuda_load_model: parse, model meta,
 * validate, upload and repack. */
VELO_API int32_t velo_cuda_load_gguf(velo_cuda_ctx *ctx, const char *path);

/* Write n_tokens K/V rows (host [n_tokens][n_head_kv][head_dim], f16 for f16 /
 * int8 pools, f32 for f32 pools) of one layer at positions pos0.. of `slot`
 * (int8 pools quantise as kv_update_int8, src/kernels.metal:753-802).  The
 * cache a prefill produced; synchronous. */
VELO_API int32_t velo_cuda_write_kv(velo_cuda_ctx *ctx, uint32_t slot, int32_t layer, int32_t pos0,
                                    int32_t n_tokens, const void *k, const void *v);

/* Read back the pool bytes of positions pos0..pos0+n_tokens of `slot` and
 * `layer`: k/v [n_tokens][n_head_kv][head_dim] (pool dtype), scales
 * [n_tokens][n_head_kv] f16 (int8 pools; may be NULL).  Synchronous. */
VELO_API int32_t velo_cuda_read_kv(velo_cuda_ctx *ctx, uint32_t slot, int32_t layer, int32_t pos0,
                                   int32_t n_tokens, void *k_out, void *v_out, void *k_scale_out,
                                   void *v_scale_out);

typedef struct velo_verify_batch {
    uint32_t struct_size;     /* sizeof(velo_verify_batch) */
    int32_t B, n_nodes;       /* sequences, draft-tree nodes per sequence (<= 64) */
    const uint32_t *slots;    /* [B] page-table rows (host) */
    const int32_t *ctx_len;   /* [B] cached tokens per sequence (host) */
    const uint32_t *tokens;   /* [B][n_nodes]: node 0 is the last committed token */
    const int32_t *parents;   /* [B][n_nodes]: -1 for node 0, parents[n] < n */
    float temperature;        /* 0: greedy tree walk; > 0: rejection sampling (chains) */
    const float *draft_logits;/* [B][n_nodes-1][V] host, sampling only */
    const float *uniforms;    /* [B][n_nodes] host, sampling only */
    int32_t commit;           /* 0: no KV write; 1: the accepted path's K/V; 2 (greedy
                                 chains): every node's K/V, accepted_len = n_nodes - 1
                                 and bonus = argmax after the last node (prefill in
                                 chunks of <= 64 tokens, or one draft decode step) */
} velo_verify_batch;

typedef struct velo_verify_result {
    int32_t *accepted_len;    /* [B] accepted draft tokens (path length - 1) */
    int32_t *accepted_nodes;  /* [B][n_nodes] path root first, -1 padded (or NULL) */
    uint32_t *bonus_token;    /* [B] token emitted after the accepted path */
    float *logits;            /* [B][n_nodes][n_vocab] target logits (or NULL) */
    uint32_t *expected;       /* [B][n_nodes] the target's greedy token after each node
                                 (TreeVerifyResult::expected; greedy steps; or NULL) */
} velo_verify_result;

/* One verify step for B sequences: the target forward over every draft-tree
 * node (row n predicts the successor of node n; node n sits at position
 * ctx_len + depth(n) - 1 and attends to the cache and its own root->n path),
 * acceptance (greedy: GreedySampler argmax + find_best_path; sampling: the
 * rejection rule of velo_cuda_accept on chains) and, with commit, the KV of
 * the accepted path written at positions ctx_len.. on the device.  Host
 * buffers; waits for the result.  With tp_size > 1 every rank makes the same
 * call with the same batch (draft logits and uniforms included) and gets the
 * same decisions; logits, when requested, are the full rows.  Replaces TargetModel::verify_tree /
 * verify_batch over CausalLmBackend::verify_logits and the commit of
 * SpeculativeSession (src/speculative.rs:97-129, 217-254, 473-519;
 * src/backend.rs:313-369; src/llama_cpu.rs:401-419). */
VELO_API int32_t velo_cuda_verify_step(velo_cuda_ctx *ctx, const velo_verify_batch *batch,
                                       velo_verify_result *result);

/* ---- step profile ------------------------------------------------------ */

/* Phases of a verify step whose device time velo_cuda_profile accumulates. */
typedef enum velo_phase {
    VELO_PHASE_OTHER = 0,          /* ancestor masks, embedding, RMSNorm, RoPE + split */
    VELO_PHASE_GEMM_QKV = 1,       /* fused q/k/v projection */
    VELO_PHASE_ATTENTION = 2,      /* tree-masked paged attention */
    VELO_PHASE_GEMM_O = 3,         /* o_proj */
    VELO_PHASE_GEMM_FFN_UP = 4,    /* w1/w3 with the SwiGLU epilogue */
    VELO_PHASE_GEMM_FFN_DOWN = 5,  /* w2 */
    VELO_PHASE_ALLREDUCE = 6,      /* tensor-parallel sums after o_proj / w2 */
    VELO_PHASE_LM_HEAD = 7,        /* final RMSNorm excluded: LM head GEMM */
    VELO_PHASE_ACCEPT_COMMIT = 8,  /* acceptance, logits exchange, KV commit */
    VELO_PHASE_COUNT = 9
} velo_phase;

/* enable != 0: the following verify steps run their launches directly (no
 * CUDA graph) with a CUDA event at the start of every phase, and add each
 * phase's device time to per-phase totals; enable == 0 stops it.  Either call
 * clears the totals.  Instrumentation for benchmarks: no counterpart in the
 * reference.  VELO_ERR_INVALID_ARGUMENT without a model. */
VELO_API int32_t velo_cuda_profile(velo_cuda_ctx *ctx, int32_t enable);

/* Copy the per-phase totals in milliseconds (ms[i] for velo_phase i, n >=
 * VELO_PHASE_COUNT) and the number of profiled steps (or NULL). */
VELO_API int32_t velo_cuda_profile_read(velo_cuda_ctx *ctx, double *ms, int32_t n, int32_t *steps);

/* How the row-split GEMMs' partials are summed over the tensor-parallel group
 * (o_proj, down_proj; the reference's all_reduce_sum_and_add,
 * src/metal/tp_model.rs:199-277).  The peer path is set up by the first verify
 * step (every rank maps every rank's partial buffer over CUDA IPC) and taken
 * only when it succeeded on every rank; VELO_TP_AR=nccl in the environment
 * forces NCCL, VELO_TP_AR=peer the unfused peer kernel. */
typedef enum velo_tp_sum {
    VELO_TP_SUM_NONE = 0,  /* one GPU, or the f32 path (NCCL f32 all-reduce) */
    VELO_TP_SUM_NCCL = 1,  /* NCCL bf16 all-reduce */
    VELO_TP_SUM_PEER = 2,  /* one kernel over NVLink peer memory (VELO_TP_AR=peer) */
    VELO_TP_SUM_FUSED = 3, /* the GEMM epilogue pushes each column block to its owner
                              rank, whose gather kernel adds and broadcasts it */
    VELO_TP_SUM_CE = 4     /* VELO_TP_AR=ce: the blocks cross NVLink as copy-engine
                              copies; kernels only add and order them */
} velo_tp_sum;
VELO_API int32_t velo_cuda_tp_sum_path(velo_cuda_ctx *ctx, int32_t *path);

/* Failure-detection check of the peer sums' cross-rank barriers on one GPU
 * (no context): launches the gather kernel as rank 0 of a group of 2 whose
 * rank 1 never arrives; the bounded waits give up (2 s each) and the kernel
 * returns, leaving the GPU usable.  *code = the error the kernel recorded
 * (0x7101: the entry barrier ran out).  Instrumentation, no counterpart in the
 * reference. */
VELO_API int32_t velo_cuda_tp_wait_selftest(int32_t device, int32_t *code);

#ifdef __cplusplus
}
#endif
#endif /* VELO_CUDA_H */
