// verify_ops.h -- the elementwise / row kernels of the verify-step forward and
// the greedy tree acceptance and KV commit (verify_ops.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace velo {

// x[m][:] = emb[tokens[m]][:]  (f32 table, llama_cpu.rs:206-212)
cudaError_t launch_embed(const float* emb, const uint32_t* tokens, int M, int H, int V, float* x,
                         int* err, cudaStream_t s);

// y = f16(x / sqrt(mean(x^2) + eps) * w)  (llama_cpu.rs:55-60), one row per block
cudaError_t launch_rmsnorm_f16(const float* x, const float* w, int M, int H, float eps, __half* y,
                               cudaStream_t s);

// Splits the fused QKV projection (f32 [M][(Hq + 2 Hkv) * 128]) into q, node_k
// (RoPE applied, NeoX half split, llama_cpu.rs:98-132) and node_v, all f16.
// Row m = (b, n) sits at position ctx_len[b] + depth(n) - 1, depth from the
// ancestor mask (popcount).
cudaError_t launch_rope_split(const float* qkv, const uint64_t* anc, const int32_t* ctx_len,
                              int B, int N, int Hq, int Hkv, float freq_base, __half* q,
                              __half* nk, __half* nv, cudaStream_t s);

// Greedy verification of a draft tree per sequence: expected[n] =
// argmax(logits[b][n]) with the GreedySampler rule (last maximal index wins,
// NaN never; sampling.rs:39-58), then find_best_path (speculative.rs:97-129):
// valid[0]; valid[n] = valid[parent] && token[n] == expected[parent]; the
// deepest valid node wins, ties to the later index.  Outputs: path[b][0..len)
// root first (-1 padded to N), path_len[b], bonus[b] = expected[best].
cudaError_t launch_tree_greedy(const float* logits, const uint32_t* tokens, const int32_t* parents,
                               int B, int N, int V, uint32_t* expected, int32_t* path,
                               int32_t* path_len, uint32_t* bonus, cudaStream_t s);

// Tensor parallelism: x += y (the all-reduced partial of a row-split GEMM).
cudaError_t launch_add_f32(float* x, const float* y, size_t n, cudaStream_t s);

// x[m] += sum[m] (bf16, the all-reduced partials of a row-split GEMM), then
// y = f16(x / rms(x) * w) as launch_rmsnorm_f16 (H % 4 == 0, H <= 8192).
cudaError_t launch_add_rmsnorm_f16(float* x, const __nv_bfloat16* sum, const float* w, int M, int H,
                                   float eps, __half* y, cudaStream_t s);
// The same with the sum stored column-blocked (the copy-engine tensor-parallel
// sum): element (m, n) at sum[(n / blk_cols) * blk_stride + m * blk_cols + n % blk_cols].
cudaError_t launch_add_rmsnorm_blocked_f16(float* x, const __nv_bfloat16* sum, int blk_cols, size_t blk_stride,
                                           const float* w, int M, int H, float eps, __half* y, cudaStream_t s);

// Tensor parallelism, vocabulary-sharded LM head: per row the GreedySampler
// maximum of this rank's logits [M][v_loc] as (value, global index) pairs
// (index -1 when the shard has no non-NaN value) ...
cudaError_t launch_row_argmax_pairs(const float* logits, int M, int v_loc, int v_ofs, int2* pairs,
                                    cudaStream_t s);
// ... and the winner over the tp gathered shards [tp][M] (larger value, ties
// to the larger index = the later shard, as one pass over the whole row).
cudaError_t launch_argmax_combine(const int2* pairs, int tp, int M, uint32_t* expected, cudaStream_t s);

// Commit of whole chains (prefill / draft decode): path[b] = 0..N-1,
// path_len[b] = N, bonus[b] = expected[b][N-1].
cudaError_t launch_chain_commit(const uint32_t* expected, int B, int N, int32_t* path,
                                int32_t* path_len, uint32_t* bonus, cudaStream_t s);

// Greedy tree walk alone, on precomputed expected tokens.
cudaError_t launch_tree_walk(const uint32_t* tokens, const int32_t* parents, const uint32_t* expected,
                             int B, int N, int32_t* path, int32_t* path_len, uint32_t* bonus,
                             cudaStream_t s);

// KV commit: node rows path[b][0..path_len[b]) of every layer's tree scratch
// (f16 [L][B*N][Hkv][128], stride layer_rows) are written to the paged pool
// at positions ctx_len[b] + i.  INT8 pools quantise per token and head as
// kv_update_int8 (src/kernels.metal:753-802): scale = max|x| / 127 (f16),
// q = trunc(x * (127 / max|x|)).  A position past the sequence's page-table
// row sets *err.
struct KvCommitArgs {
    const __half* node_k;     // [L][B*N][Hkv][128]
    const __half* node_v;
    const int32_t* path;      // [B][N]
    const int32_t* path_len;  // [B]
    const int32_t* ctx_len;   // [B]
    const uint32_t* slots;    // [B] page-table rows (NULL: row b)
    const uint32_t* page_table;  // [rows][max_pages]
    void* k_pool;             // [L][pages][Hkv][16][128]
    void* v_pool;
    __half* k_scale;          // [L][pages][Hkv][16] (int8)
    __half* v_scale;
    int B, N, L, Hkv, max_pages, pool_pages;
    int kv_int8;
    int* err;
};
cudaError_t launch_kv_commit(const KvCommitArgs& a, cudaStream_t s);

}  // namespace velo
