// attention.cu -- C ABI of the tree-masked paged attention (include/velo_cuda.h).
#include <cmath>

#include "kernels/tree_attn.h"
#include "runtime/context.h"

using velo::fail;

extern "C" {

int32_t velo_cuda_tree_attention(velo_cuda_ctx* c, const void* q, const void* k_pool,
                                 const void* v_pool, const void* k_scale, const void* v_scale,
                                 int32_t pool_pages, const uint32_t* page_table, int32_t max_pages,
                                 const int32_t* ctx_len, const void* node_k, const void* node_v,
                                 const int32_t* parents, int32_t B, int32_t n_nodes,
                                 int32_t n_head, int32_t n_kv, int32_t head_dim, int32_t kv_dtype,
                                 void* out, int32_t out_dtype) {
    velo::Range nvtx_range("velo.tree_attention");
    velo::clear_last_error();
    if (!c) return fail(VELO_ERR_INVALID_ARGUMENT, "ctx is NULL");
    if (head_dim != velo::kAttnHeadDim)
        return fail(VELO_ERR_INVALID_ARGUMENT, "tree attention: head_dim %d unsupported (128)", head_dim);
    if (n_nodes < 1 || n_nodes > velo::kAttnMaxNodes)
        return fail(VELO_ERR_INVALID_ARGUMENT, "tree attention: n_nodes %d outside [1, %d]", n_nodes,
                    velo::kAttnMaxNodes);
    if (n_kv < 1 || n_head < n_kv || n_head % n_kv)
        return fail(VELO_ERR_INVALID_ARGUMENT, "tree attention: n_head %d / n_kv %d", n_head, n_kv);
    if (kv_dtype != VELO_KV_F16 && kv_dtype != VELO_KV_INT8)
        return fail(VELO_ERR_INVALID_ARGUMENT, "tree attention: kv_dtype %d", kv_dtype);
    if (out_dtype != 0 && out_dtype != 1)
        return fail(VELO_ERR_INVALID_ARGUMENT, "tree attention: out_dtype %d (0 f32, 1 f16)", out_dtype);
    if (B < 0 || pool_pages < 1 || max_pages < 0)
        return fail(VELO_ERR_INVALID_ARGUMENT, "tree attention: B %d, pool_pages %d, max_pages %d", B,
                    pool_pages, max_pages);
    if (B == 0) return VELO_OK;
    if (!q || !k_pool || !v_pool || !ctx_len || !node_k || !node_v || !parents || !out ||
        (max_pages > 0 && !page_table) || (kv_dtype == VELO_KV_INT8 && (!k_scale || !v_scale)))
        return fail(VELO_ERR_INVALID_ARGUMENT, "tree attention: NULL buffer");
    const uintptr_t al = (uintptr_t)q | (uintptr_t)k_pool | (uintptr_t)v_pool | (uintptr_t)node_k |
                         (uintptr_t)node_v | (uintptr_t)out | (uintptr_t)k_scale | (uintptr_t)v_scale;
    if (al % 16) return fail(VELO_ERR_INVALID_ARGUMENT, "tree attention: buffers must be 16-byte aligned");
    VELO_CUDA_TRY(cudaSetDevice(c->device));
    int32_t st = c->attn_ws.ensure((size_t)B * n_nodes * sizeof(uint64_t), c->stream);
    if (st) return st;
    uint64_t* anc = static_cast<uint64_t*>(c->attn_ws.ptr);
    VELO_CUDA_TRY(velo::launch_tree_ancestors(parents, B, n_nodes, anc, c->err_flag, c->stream));
    velo::TreeAttnArgs a{};
    a.q = static_cast<const __half*>(q);
    a.k_pool = k_pool;
    a.v_pool = v_pool;
    a.k_scale = static_cast<const __half*>(k_scale);
    a.v_scale = static_cast<const __half*>(v_scale);
    a.page_table = page_table;
    a.ctx_len = ctx_len;
    a.node_k = static_cast<const __half*>(node_k);
    a.node_v = static_cast<const __half*>(node_v);
    a.anc = anc;
    a.out = out;
    a.out_f16 = out_dtype;
    a.B = B;
    a.N = n_nodes;
    a.Hq = n_head;
    a.Hkv = n_kv;
    a.max_pages = max_pages;
    a.pool_pages = pool_pages;
    a.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)head_dim));
    a.err = c->err_flag;
    VELO_CUDA_TRY(velo::launch_tree_attention(a, kv_dtype == VELO_KV_INT8, c->stream));
    return VELO_OK;
}

}  // extern "C"
