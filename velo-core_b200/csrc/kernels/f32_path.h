// f32_path.h -- the fp32 path of the verify step (f32_path.cu): models whose
// matrices are f32, the precision of the reference's CPU model
// (LlamaCpuModel, src/llama_cpu.rs:191-358, f32 math over f32 weights and an
// f32 KvCache :22-50), with f32 KV pages.  Every contraction is FFMA on the
// CUDA cores: this path answers to a 1e-4 logits tolerance, which TF32 tensor
// cores (10-bit mantissa) cannot meet, and the shapes it serves (hidden 256,
// FFN 688, a few query rows) are latency-bound rather than compute-bound.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace velo {

enum F32Epilogue {
    kF32Store = 0,   // y[m][n] = acc
    kF32Add = 1,     // y[m][n] += acc (residual)
    kF32SwiGLU = 2,  // w holds 2N rows (gate 0..N-1, up N..2N-1): y = silu(gate) * up
};

// y[m][n] (ldy) <- sum_k x[m][k] * w[n][k]   (matvec_quant over f32 rows,
// llama_cpu.rs:75-90, for M rows at once).  x is [M][K] contiguous; K % 4 == 0
// and both pointers 16-byte aligned.
cudaError_t launch_gemm_f32(const float* w, const float* x, int M, int N, int K, float* y, int ldy,
                            int mode, cudaStream_t s);

// y = x / sqrt(mean(x^2) + eps) * w (llama_cpu.rs:55-60), f32 out; H % 4 == 0.
cudaError_t launch_rmsnorm_f32(const float* x, const float* w, int M, int H, float eps, float* y,
                               cudaStream_t s);

// The fused QKV projection [M][(Hq + 2 Hkv) D] split into q [M][Hq][D] and
// node_k / node_v [M][Hkv][D], RoPE (NeoX half split, llama_cpu.rs:113-132)
// on q and k at position ctx_len[b] + depth(n) - 1.  D even, <= 256.
cudaError_t launch_rope_split_f32(const float* qkv, const uint64_t* anc, const int32_t* ctx_len,
                                  int B, int N, int Hq, int Hkv, int D, float freq_base, float* q,
                                  float* nk, float* nv, cudaStream_t s);

struct TreeAttnF32Args {
    const float* q;              // [B][N][Hq][D]
    const float* k_pool;         // [pool_pages][Hkv][16][D]
    const float* v_pool;
    const uint32_t* page_table;  // [B][max_pages]
    const int32_t* ctx_len;      // [B]
    const float* node_k;         // [B][N][Hkv][D]
    const float* node_v;
    const uint64_t* anc;         // [B][N] ancestor masks (self included)
    float* out;                  // [B][N][Hq][D]
    int B, N, Hq, Hkv, D, max_pages, pool_pages;
    int* err;                    // device error word (page id outside the pool)
};

// Tree-masked paged attention in f32 (the GQA attention of llama_cpu.rs:255-284
// over the cached prefix and the node's root->n path); D in {64, 128}.
cudaError_t launch_tree_attention_f32(const TreeAttnF32Args& a, cudaStream_t s);

struct KvCommitF32Args {
    const float* node_k;         // [L][B*N][Hkv][D]
    const float* node_v;
    const int32_t* path;         // [B][N]
    const int32_t* path_len;     // [B]
    const int32_t* ctx_len;      // [B]
    const uint32_t* slots;       // [B] page-table rows (NULL: row b)
    const uint32_t* page_table;  // [rows][max_pages]
    float* k_pool;               // [L][pages][Hkv][16][D]
    float* v_pool;
    int B, N, L, Hkv, D, max_pages, pool_pages;
    int* err;
};

// The accepted path's rows into f32 pages at ctx_len[b] + i (the KvCache store
// of llama_cpu.rs:252, through the page table).
cudaError_t launch_kv_commit_f32(const KvCommitF32Args& a, cudaStream_t s);

}  // namespace velo
