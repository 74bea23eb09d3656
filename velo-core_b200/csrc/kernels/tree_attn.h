// tree_attn.h -- tree-masked paged attention on the tcgen05 tensor cores
// (tree_attn.cu).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace velo {

constexpr int kAttnHeadDim = 128;   // head_dim handled by the kernel
constexpr int kAttnMaxNodes = 64;   // draft-tree nodes per sequence (u64 masks)
constexpr int kKvPage = 16;         // tokens per KV page

struct TreeAttnArgs {
    const __half* q;             // [B][N][Hq][128] f16, RoPE applied
    const void* k_pool;          // [pool_pages][Hkv][16][128] f16 or int8
    const void* v_pool;
    const __half* k_scale;       // [pool_pages][Hkv][16] f16 (int8 pools)
    const __half* v_scale;
    const uint32_t* page_table;  // [B][max_pages]
    const int32_t* ctx_len;      // [B] cached tokens per sequence
    const __half* node_k;        // [B][N][Hkv][128] f16 K/V of the tree nodes
    const __half* node_v;
    const uint64_t* anc;         // [B][N] bit j: node j is node n or an ancestor
    void* out;                   // [B][N][Hq][128] f32 or f16
    int out_f16;
    int B, N, Hq, Hkv, max_pages, pool_pages;
    float scale_log2;            // log2(e) / sqrt(head_dim)
    int* err;                    // device error word
};

// anc[b][n] from parents[b][n] (-1 for the root, parent < child).
cudaError_t launch_tree_ancestors(const int32_t* parents, int B, int N, uint64_t* anc, int* err,
                                  cudaStream_t stream);

cudaError_t launch_tree_attention(const TreeAttnArgs& a, bool kv_int8, cudaStream_t stream);

}  // namespace velo
