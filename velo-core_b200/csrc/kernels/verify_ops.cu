// verify_ops.cu -- row / elementwise kernels of the verify forward, greedy
// tree acceptance and the on-device KV commit.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "kernels/verify_ops.h"

namespace velo {
namespace {

constexpr int D = 128;  // head_dim
constexpr int kErrToken = 0x6101, kErrCommit = 0x6102;

__global__ void embed_kernel(const float* __restrict__ emb, const uint32_t* __restrict__ tokens,
                             int H, int V, float* __restrict__ x, int* err) {
    const int m = blockIdx.x;
    uint32_t t = tokens[m];
    if (t >= (uint32_t)V) {
        if (threadIdx.x == 0) atomicCAS(err, 0, kErrToken);
        t = 0;
    }
    const float4* src = reinterpret_cast<const float4*>(emb + (size_t)t * H);
    float4* dst = reinterpret_cast<float4*>(x + (size_t)m * H);
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x) dst[i] = src[i];
}

__device__ __forceinline__ float block_sum(float v, float* sh) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if ((threadIdx.x & 31) == 0) sh[w] = v;
    __syncthreads();
    float t = 0.0f;
    for (int i = 0; i < nw; ++i) t += sh[i];
    __syncthreads();
    return t;
}

// Four floats as four f16 (round to nearest) in one 8-byte word.
__device__ __forceinline__ uint2 pack_half4(float a, float b, float c, float d) {
    const __half2 lo = __floats2half2_rn(a, b), hi = __floats2half2_rn(c, d);
    return make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
}

__global__ void rmsnorm_f16_kernel(const float* __restrict__ x, const float* __restrict__ w, int H,
                                   float eps, __half* __restrict__ y) {
    __shared__ float sh[32];
    const int m = blockIdx.x;
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)m * H);
    float ss = 0.0f;
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x) {
        const float4 v = xr[i];
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    ss = block_sum(ss, sh);
    const float rms = sqrtf(ss / (float)H + eps);
    const float4* wr = reinterpret_cast<const float4*>(w);
    uint2* yr = reinterpret_cast<uint2*>(y + (size_t)m * H);
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x) {
        const float4 v = xr[i], g = wr[i];
        yr[i] = pack_half4((v.x / rms) * g.x, (v.y / rms) * g.y, (v.z / rms) * g.z, (v.w / rms) * g.w);
    }
}

// The same for rows of at most kNormMaxPer x 1024 elements: one read of x, the
// row kept in registers between the sum of squares and the scaling.
constexpr int kNormMaxPer = 8;
__global__ void __launch_bounds__(256) rmsnorm_f16_reg_kernel(const float* __restrict__ x,
                                                              const float* __restrict__ w, int H, float eps,
                                                              __half* __restrict__ y) {
    __shared__ float sh[32];
    const int m = blockIdx.x;
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)m * H);
    float4 keep[kNormMaxPer];
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < kNormMaxPer; ++j) {
        const int i = threadIdx.x + j * 256;
        if (i < H / 4) {
            keep[j] = xr[i];
            ss += keep[j].x * keep[j].x + keep[j].y * keep[j].y + keep[j].z * keep[j].z + keep[j].w * keep[j].w;
        }
    }
    ss = block_sum(ss, sh);
    const float rms = sqrtf(ss / (float)H + eps);
    const float4* wr = reinterpret_cast<const float4*>(w);
    uint2* yr = reinterpret_cast<uint2*>(y + (size_t)m * H);
#pragma unroll
    for (int j = 0; j < kNormMaxPer; ++j) {
        const int i = threadIdx.x + j * 256;
        if (i < H / 4) {
            const float4 v = keep[j], g = wr[i];
            yr[i] = pack_half4((v.x / rms) * g.x, (v.y / rms) * g.y, (v.z / rms) * g.z, (v.w / rms) * g.w);
        }
    }
}

// Tensor parallelism: x[m] += sum (the bf16 all-reduced partials of a
// row-split GEMM), then the RMSNorm of the new x as rmsnorm_f16_kernel.  The
// block keeps its row in registers between the two passes (H <= 8192: at most
// 8 float4 per thread of 256).
// blk_cols > 0: the sum is stored column-blocked, element (m, n) at
// sum[(n / blk_cols) * blk_stride + m * blk_cols + n % blk_cols] (blk_cols % 4 == 0).
__global__ void add_rmsnorm_f16_kernel(float* __restrict__ x, const __nv_bfloat16* __restrict__ sum,
                                       const float* __restrict__ w, int H, float eps,
                                       __half* __restrict__ y, int blk_cols, size_t blk_stride) {
    __shared__ float sh[32];
    constexpr int kMaxPer = 8;
    const int m = blockIdx.x;
    float4* xr = reinterpret_cast<float4*>(x + (size_t)m * H);
    float4 keep[kMaxPer];
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < kMaxPer; ++j) {
        const int i = threadIdx.x + j * blockDim.x;
        if (i < H / 4) {
            float4 v = xr[i];
            const int n = 4 * i;
            const size_t si = blk_cols > 0 ? (size_t)(n / blk_cols) * blk_stride + (size_t)m * blk_cols + n % blk_cols
                                           : (size_t)m * H + n;
            const uint2 sv = *reinterpret_cast<const uint2*>(sum + si);  // four bf16 of the sum
            const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&sv.x));
            const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&sv.y));
            v.x += a.x;
            v.y += a.y;
            v.z += b.x;
            v.w += b.y;
            xr[i] = v;
            keep[j] = v;
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
    }
    ss = block_sum(ss, sh);
    const float rms = sqrtf(ss / (float)H + eps);
    const float4* wr = reinterpret_cast<const float4*>(w);
    uint2* yr = reinterpret_cast<uint2*>(y + (size_t)m * H);
#pragma unroll
    for (int j = 0; j < kMaxPer; ++j) {
        const int i = threadIdx.x + j * blockDim.x;
        if (i < H / 4) {
            const float4 v = keep[j], g = wr[i];
            yr[i] = pack_half4((v.x / rms) * g.x, (v.y / rms) * g.y, (v.z / rms) * g.z, (v.w / rms) * g.w);
        }
    }
}

// one block per row m: the 64 rotation angles of the row's position are
// computed once (theta = pos / base^(2i/128), llama_cpu.rs:121-123), then
// every head of q / k / v is rotated (q, k) or copied (v), 8 values a thread
__global__ void rope_split_kernel(const float* __restrict__ qkv, const uint64_t* __restrict__ anc,
                                  const int32_t* __restrict__ ctx_len, int B, int N, int Hq,
                                  int Hkv, float freq_base, __half* __restrict__ q,
                                  __half* __restrict__ nk, __half* __restrict__ nv) {
    __shared__ float cs[D / 2], sn[D / 2];
    const int m = blockIdx.x;
    const int b = m / N;
    const int pos = ctx_len[b] + __popcll(anc[m]) - 1;
    if (threadIdx.x < D / 2) {
        const int i = threadIdx.x;
        const float theta = (float)pos / powf(freq_base, (2.0f * (float)i) / (float)D);
        sincosf(theta, &sn[i], &cs[i]);
    }
    __syncthreads();
    const int heads = Hq + 2 * Hkv;
    // work item: (head, group of 8 rotation pairs)
    for (int w = threadIdx.x; w < heads * (D / 16); w += blockDim.x) {
        const int hh = w / (D / 16), i0 = (w % (D / 16)) * 8;
        const float* src = qkv + ((size_t)m * heads + hh) * D;
        float4 a0 = *reinterpret_cast<const float4*>(src + i0);
        float4 a1 = *reinterpret_cast<const float4*>(src + i0 + 4);
        float4 b0 = *reinterpret_cast<const float4*>(src + i0 + D / 2);
        float4 b1 = *reinterpret_cast<const float4*>(src + i0 + D / 2 + 4);
        float x0[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        float x1[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        if (hh < Hq + Hkv) {
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float c = cs[i0 + e], s = sn[i0 + e];
                const float r0 = x0[e] * c - x1[e] * s;
                const float r1 = x0[e] * s + x1[e] * c;
                x0[e] = r0;
                x1[e] = r1;
            }
        }
        __half* dst;
        if (hh < Hq)
            dst = q + ((size_t)m * Hq + hh) * D;
        else if (hh < Hq + Hkv)
            dst = nk + ((size_t)m * Hkv + (hh - Hq)) * D;
        else
            dst = nv + ((size_t)m * Hkv + (hh - Hq - Hkv)) * D;
        uint4 o0, o1;
        __half2 h[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            h[e] = __floats2half2_rn(x0[2 * e], x0[2 * e + 1]);
            h[4 + e] = __floats2half2_rn(x1[2 * e], x1[2 * e + 1]);
        }
        o0 = make_uint4(*reinterpret_cast<uint32_t*>(&h[0]), *reinterpret_cast<uint32_t*>(&h[1]),
                        *reinterpret_cast<uint32_t*>(&h[2]), *reinterpret_cast<uint32_t*>(&h[3]));
        o1 = make_uint4(*reinterpret_cast<uint32_t*>(&h[4]), *reinterpret_cast<uint32_t*>(&h[5]),
                        *reinterpret_cast<uint32_t*>(&h[6]), *reinterpret_cast<uint32_t*>(&h[7]));
        *reinterpret_cast<uint4*>(dst + i0) = o0;
        *reinterpret_cast<uint4*>(dst + i0 + D / 2) = o1;
    }
}

// argmax with the GreedySampler rule: candidates in increasing index order,
// `x >= best` replaces (last maximal index wins), NaN never replaces.
struct ArgMax {
    float v;
    int i;  // -1: nothing seen
};
__device__ __forceinline__ ArgMax am_combine(ArgMax a, ArgMax b) {
    if (a.i < 0) return b;
    if (b.i < 0) return a;
    if (b.v > a.v || (b.v == a.v && b.i > a.i)) return b;
    return a;
}

// one block per (sequence, node) row
__global__ void row_argmax_kernel(const float* __restrict__ logits, int V,
                                  uint32_t* __restrict__ expected) {
    __shared__ float sv[32];
    __shared__ int si[32];
    const float* row = logits + (size_t)blockIdx.x * V;
    ArgMax best{-INFINITY, -1};
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const float x = row[i];
        if (x >= best.v) best = ArgMax{x, i};  // NaN compares false
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        ArgMax other{__shfl_xor_sync(0xffffffffu, best.v, o), __shfl_xor_sync(0xffffffffu, best.i, o)};
        best = am_combine(best, other);
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        sv[w] = best.v;
        si[w] = best.i;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        ArgMax r{-INFINITY, -1};
        for (int k = 0; k < (int)(blockDim.x >> 5); ++k) r = am_combine(r, ArgMax{sv[k], si[k]});
        expected[blockIdx.x] = r.i < 0 ? 0u : (uint32_t)r.i;
    }
}

// per row: (value, global index) of this shard's GreedySampler maximum
__global__ void row_argmax_pairs_kernel(const float* __restrict__ logits, int v_loc, int v_ofs,
                                        int2* __restrict__ pairs) {
    __shared__ float sv[32];
    __shared__ int si[32];
    const float* row = logits + (size_t)blockIdx.x * v_loc;
    ArgMax best{-INFINITY, -1};
    for (int i = threadIdx.x; i < v_loc; i += blockDim.x) {
        const float x = row[i];
        if (x >= best.v) best = ArgMax{x, i};
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        ArgMax other{__shfl_xor_sync(0xffffffffu, best.v, o), __shfl_xor_sync(0xffffffffu, best.i, o)};
        best = am_combine(best, other);
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        sv[w] = best.v;
        si[w] = best.i;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        ArgMax r{-INFINITY, -1};
        for (int k = 0; k < (int)(blockDim.x >> 5); ++k) r = am_combine(r, ArgMax{sv[k], si[k]});
        pairs[blockIdx.x] = make_int2(__float_as_int(r.v), r.i < 0 ? -1 : r.i + v_ofs);
    }
}

__global__ void argmax_combine_kernel(const int2* __restrict__ pairs, int tp, int M,
                                      uint32_t* __restrict__ expected) {
    const int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m >= M) return;
    ArgMax r{-INFINITY, -1};
    for (int t = 0; t < tp; ++t) {
        const int2 p = pairs[(size_t)t * M + m];
        r = am_combine(r, ArgMax{__int_as_float(p.x), p.y});
    }
    expected[m] = r.i < 0 ? 0u : (uint32_t)r.i;
}

__global__ void add_f32_kernel(float* __restrict__ x, const float* __restrict__ y, size_t n4) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n4) return;
    float4 a = reinterpret_cast<float4*>(x)[i];
    const float4 b = reinterpret_cast<const float4*>(y)[i];
    a.x += b.x;
    a.y += b.y;
    a.z += b.z;
    a.w += b.w;
    reinterpret_cast<float4*>(x)[i] = a;
}

// one thread per sequence: find_best_path on the expected tokens
__global__ void tree_walk_kernel(const uint32_t* __restrict__ tokens, const int32_t* __restrict__ parents,
                                 const uint32_t* __restrict__ expected, int B, int N,
                                 int32_t* __restrict__ path, int32_t* __restrict__ path_len,
                                 uint32_t* __restrict__ bonus) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    const uint32_t* tk = tokens + (size_t)b * N;
    const int32_t* par = parents + (size_t)b * N;
    const uint32_t* ex = expected + (size_t)b * N;
    uint64_t valid = 1ull;  // N <= 64
    int depth[64];
    depth[0] = 1;
    int best = 0, best_len = 1;
    for (int n = 1; n < N; ++n) {
        const int p = par[n];
        depth[n] = (p >= 0 && p < n) ? depth[p] + 1 : 1;
        if (p >= 0 && p < n && ((valid >> p) & 1ull) && tk[n] == ex[p]) valid |= 1ull << n;
        if (((valid >> n) & 1ull) && depth[n] >= best_len) {
            best_len = depth[n];
            best = n;
        }
    }
    int32_t* out = path + (size_t)b * N;
    for (int i = best_len; i < N; ++i) out[i] = -1;
    int k = best_len;
    for (int c = best; c >= 0 && k > 0; c = par[c]) out[--k] = c;
    path_len[b] = best_len;
    bonus[b] = ex[best];
}

// one warp per (sequence, path position, layer, kv head): 128 values
__global__ void kv_commit_kernel(const KvCommitArgs a) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const long total = (long)a.B * a.N * a.L * a.Hkv;
    if (warp >= total) return;
    const int h = warp % a.Hkv;
    const int l = (warp / a.Hkv) % a.L;
    const int i = (warp / (a.Hkv * a.L)) % a.N;
    const int b = warp / (a.Hkv * a.L * a.N);
    if (i >= a.path_len[b]) return;
    const int node = a.path[(size_t)b * a.N + i];
    const int pos = a.ctx_len[b] + i;
    const int pi = pos / 16, slot = pos % 16;
    const uint32_t row = a.slots ? a.slots[b] : (uint32_t)b;
    if (node < 0 || node >= a.N || pi >= a.max_pages) {
        if (lane == 0) atomicCAS(a.err, 0, kErrCommit);
        return;
    }
    const uint32_t pg = a.page_table[(size_t)row * a.max_pages + pi];
    if (pg >= (uint32_t)a.pool_pages) {
        if (lane == 0) atomicCAS(a.err, 0, kErrCommit);
        return;
    }
    const size_t src_row = (((size_t)l * a.B * a.N + (size_t)b * a.N + node) * a.Hkv + h) * D;
    const size_t dst_tok = (((size_t)l * a.pool_pages + pg) * a.Hkv + h) * 16 + slot;
#pragma unroll
    for (int kv = 0; kv < 2; ++kv) {
        const __half* src = (kv ? a.node_v : a.node_k) + src_row;
        const __half2 v01 = reinterpret_cast<const __half2*>(src)[2 * lane];
        const __half2 v23 = reinterpret_cast<const __half2*>(src)[2 * lane + 1];
        if (!a.kv_int8) {
            __half2* dst = reinterpret_cast<__half2*>(static_cast<__half*>(kv ? a.v_pool : a.k_pool) + dst_tok * D);
            dst[2 * lane] = v01;
            dst[2 * lane + 1] = v23;
        } else {
            const float x0 = __low2float(v01), x1 = __high2float(v01), x2 = __low2float(v23),
                        x3 = __high2float(v23);
            float mx = fmaxf(fmaxf(fabsf(x0), fabsf(x1)), fmaxf(fabsf(x2), fabsf(x3)));
#pragma unroll
            for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float inv = mx > 0.0f ? __fdiv_rn(127.0f, mx) : 0.0f;
            char4 qv;
            qv.x = (signed char)(int)__fmul_rn(x0, inv);  // truncation toward zero
            qv.y = (signed char)(int)__fmul_rn(x1, inv);
            qv.z = (signed char)(int)__fmul_rn(x2, inv);
            qv.w = (signed char)(int)__fmul_rn(x3, inv);
            reinterpret_cast<char4*>(static_cast<int8_t*>(kv ? a.v_pool : a.k_pool) + dst_tok * D)[lane] = qv;
            if (lane == 0) (kv ? a.v_scale : a.k_scale)[dst_tok] = __float2half_rn(__fdiv_rn(mx, 127.0f));
        }
    }
}

__global__ void chain_commit_kernel(const uint32_t* __restrict__ expected, int B, int N,
                                    int32_t* __restrict__ path, int32_t* __restrict__ path_len,
                                    uint32_t* __restrict__ bonus) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * N) return;
    const int b = i / N, n = i - b * N;
    path[i] = n;
    if (n == N - 1) {
        path_len[b] = N;
        bonus[b] = expected[i];
    }
}

}  // namespace

cudaError_t launch_chain_commit(const uint32_t* expected, int B, int N, int32_t* path,
                                int32_t* path_len, uint32_t* bonus, cudaStream_t s) {
    if (B * N == 0) return cudaSuccess;
    chain_commit_kernel<<<(B * N + 127) / 128, 128, 0, s>>>(expected, B, N, path, path_len, bonus);
    return cudaGetLastError();
}

cudaError_t launch_embed(const float* emb, const uint32_t* tokens, int M, int H, int V, float* x,
                         int* err, cudaStream_t s) {
    if (M == 0) return cudaSuccess;
    embed_kernel<<<M, 256, 0, s>>>(emb, tokens, H, V, x, err);
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm_f16(const float* x, const float* w, int M, int H, float eps, __half* y,
                               cudaStream_t s) {
    if (M == 0) return cudaSuccess;
    if (H % 4) return cudaErrorInvalidValue;
    if (H / 4 <= 256 * kNormMaxPer)
        rmsnorm_f16_reg_kernel<<<M, 256, 0, s>>>(x, w, H, eps, y);
    else
        rmsnorm_f16_kernel<<<M, 256, 0, s>>>(x, w, H, eps, y);
    return cudaGetLastError();
}

cudaError_t launch_add_rmsnorm_f16(float* x, const __nv_bfloat16* sum, const float* w, int M, int H,
                                   float eps, __half* y, cudaStream_t s) {
    if (M == 0) return cudaSuccess;
    if (H % 4 || H / 4 > 256 * 8) return cudaErrorInvalidValue;
    add_rmsnorm_f16_kernel<<<M, 256, 0, s>>>(x, sum, w, H, eps, y, 0, 0);
    return cudaGetLastError();
}

cudaError_t launch_add_rmsnorm_blocked_f16(float* x, const __nv_bfloat16* sum, int blk_cols, size_t blk_stride,
                                           const float* w, int M, int H, float eps, __half* y, cudaStream_t s) {
    if (M == 0) return cudaSuccess;
    if (H % 4 || H / 4 > 256 * 8 || blk_cols <= 0 || blk_cols % 4 || H % blk_cols) return cudaErrorInvalidValue;
    add_rmsnorm_f16_kernel<<<M, 256, 0, s>>>(x, sum, w, H, eps, y, blk_cols, blk_stride);
    return cudaGetLastError();
}

cudaError_t launch_rope_split(const float* qkv, const uint64_t* anc, const int32_t* ctx_len,
                              int B, int N, int Hq, int Hkv, float freq_base, __half* q,
                              __half* nk, __half* nv, cudaStream_t s) {
    if (B * N == 0) return cudaSuccess;
    rope_split_kernel<<<B * N, 256, 0, s>>>(qkv, anc, ctx_len, B, N, Hq, Hkv, freq_base, q, nk, nv);
    return cudaGetLastError();
}

cudaError_t launch_tree_greedy(const float* logits, const uint32_t* tokens, const int32_t* parents,
                               int B, int N, int V, uint32_t* expected, int32_t* path,
                               int32_t* path_len, uint32_t* bonus, cudaStream_t s) {
    if (B == 0) return cudaSuccess;
    row_argmax_kernel<<<B * N, 512, 0, s>>>(logits, V, expected);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    tree_walk_kernel<<<(B + 63) / 64, 64, 0, s>>>(tokens, parents, expected, B, N, path, path_len, bonus);
    return cudaGetLastError();
}

cudaError_t launch_add_f32(float* x, const float* y, size_t n, cudaStream_t s) {
    const size_t n4 = n / 4;  // n is a multiple of 128 here
    if (n4 == 0) return cudaSuccess;
    add_f32_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, s>>>(x, y, n4);
    return cudaGetLastError();
}

cudaError_t launch_row_argmax_pairs(const float* logits, int M, int v_loc, int v_ofs, int2* pairs,
                                    cudaStream_t s) {
    if (M == 0) return cudaSuccess;
    row_argmax_pairs_kernel<<<M, 512, 0, s>>>(logits, v_loc, v_ofs, pairs);
    return cudaGetLastError();
}

cudaError_t launch_argmax_combine(const int2* pairs, int tp, int M, uint32_t* expected, cudaStream_t s) {
    if (M == 0) return cudaSuccess;
    argmax_combine_kernel<<<(M + 127) / 128, 128, 0, s>>>(pairs, tp, M, expected);
    return cudaGetLastError();
}

cudaError_t launch_tree_walk(const uint32_t* tokens, const int32_t* parents, const uint32_t* expected,
                             int B, int N, int32_t* path, int32_t* path_len, uint32_t* bonus,
                             cudaStream_t s) {
    if (B == 0) return cudaSuccess;
    tree_walk_kernel<<<(B + 63) / 64, 64, 0, s>>>(tokens, parents, expected, B, N, path, path_len, bonus);
    return cudaGetLastError();
}

cudaError_t launch_kv_commit(const KvCommitArgs& a, cudaStream_t s) {
    const long warps = (long)a.B * a.N * a.L * a.Hkv;
    if (warps == 0) return cudaSuccess;
    kv_commit_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace velo
