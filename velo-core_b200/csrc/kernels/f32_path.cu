// f32_path.cu -- fp32 kernels of the verify step: FFMA GEMM with the step's
// epilogues, RMSNorm, RoPE + split, tree-masked paged attention over f32
// pages, and the KV commit into f32 pages.
#include <cmath>

#include "common/smem_attr.cuh"
#include "kernels/f32_path.h"

namespace velo {
namespace {

constexpr int kErrPageF32 = 0x7101, kErrCommitF32 = 0x7102;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ------------------------------------------------------------------- GEMM
// A block of 8 warps stages MT rows of x in shared memory; each warp owns one
// output column n at a time, streams its weight row(s) with 16-byte loads
// (lane k4 = lane, lane + 32, ...) and keeps MT partial dot products, reduced
// across the warp at the end.  The weights are read once per MT rows.
constexpr int kGemmWarps = 8;

template <int MT, int MODE>
__global__ void __launch_bounds__(kGemmWarps * 32) gemm_f32_kernel(const float* __restrict__ w,
                                                                   const float* __restrict__ x,
                                                                   int M, int N, int K,
                                                                   float* __restrict__ y, int ldy) {
    extern __shared__ float4 xs[];  // [MT][K/4]
    const int K4 = K >> 2;
    const int m0 = blockIdx.y * MT;
    const int mt = min(MT, M - m0);
    const float4* xg = reinterpret_cast<const float4*>(x + (size_t)m0 * K);
    for (int i = threadIdx.x; i < mt * K4; i += blockDim.x) xs[i] = xg[i];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int n = blockIdx.x * kGemmWarps + warp; n < N; n += gridDim.x * kGemmWarps) {
        float acc[MT], acc2[MT];
#pragma unroll
        for (int r = 0; r < MT; ++r) acc[r] = acc2[r] = 0.0f;
        const float4* wr = reinterpret_cast<const float4*>(w + (size_t)n * K);
        const float4* wu = reinterpret_cast<const float4*>(w + (size_t)(n + N) * K);
        for (int k4 = lane; k4 < K4; k4 += 32) {
            const float4 a = __ldg(wr + k4);
            float4 u = make_float4(0.f, 0.f, 0.f, 0.f);
            if (MODE == kF32SwiGLU) u = __ldg(wu + k4);
#pragma unroll
            for (int r = 0; r < MT; ++r) {
                if (r < mt) {
                    const float4 xv = xs[r * K4 + k4];
                    acc[r] = fmaf(a.x, xv.x, acc[r]);
                    acc[r] = fmaf(a.y, xv.y, acc[r]);
                    acc[r] = fmaf(a.z, xv.z, acc[r]);
                    acc[r] = fmaf(a.w, xv.w, acc[r]);
                    if (MODE == kF32SwiGLU) {
                        acc2[r] = fmaf(u.x, xv.x, acc2[r]);
                        acc2[r] = fmaf(u.y, xv.y, acc2[r]);
                        acc2[r] = fmaf(u.z, xv.z, acc2[r]);
                        acc2[r] = fmaf(u.w, xv.w, acc2[r]);
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < MT; ++r) {
            acc[r] = warp_sum(acc[r]);
            if (MODE == kF32SwiGLU) acc2[r] = warp_sum(acc2[r]);
        }
        // lane r writes row r (static register indexing through the unrolled select)
#pragma unroll
        for (int r = 0; r < MT; ++r) {
            if (lane == r && r < mt) {
                float* dst = y + (size_t)(m0 + r) * ldy + n;
                if (MODE == kF32Store) {
                    *dst = acc[r];
                } else if (MODE == kF32Add) {
                    *dst += acc[r];
                } else {
                    const float g = acc[r];
                    *dst = g * (1.0f / (1.0f + expf(-g))) * acc2[r];  // silu(g) * up, llama_cpu.rs:94
                }
            }
        }
    }
}

template <int MT, int MODE>
cudaError_t gemm_launch(const float* w, const float* x, int M, int N, int K, float* y, int ldy,
                        cudaStream_t s) {
    const size_t smem = (size_t)MT * K * sizeof(float);
    static SmemAttr attr;
    const cudaError_t ea = ensure_smem(attr, gemm_f32_kernel<MT, MODE>, (int)smem);
    if (ea != cudaSuccess) return ea;
    int gx = (N + kGemmWarps - 1) / kGemmWarps;
    if (gx > 65535) gx = 65535;
    const dim3 grid(gx, (M + MT - 1) / MT);
    gemm_f32_kernel<MT, MODE><<<grid, kGemmWarps * 32, smem, s>>>(w, x, M, N, K, y, ldy);
    return cudaGetLastError();
}

template <int MODE>
cudaError_t gemm_mode(const float* w, const float* x, int M, int N, int K, float* y, int ldy,
                      cudaStream_t s) {
    constexpr size_t kMaxSmem = 200 * 1024;
    const size_t row = (size_t)K * sizeof(float);
    if (M >= 8 && 8 * row <= kMaxSmem) return gemm_launch<8, MODE>(w, x, M, N, K, y, ldy, s);
    if (M > 4 && 8 * row <= kMaxSmem) return gemm_launch<8, MODE>(w, x, M, N, K, y, ldy, s);
    if (M > 2 && 4 * row <= kMaxSmem) return gemm_launch<4, MODE>(w, x, M, N, K, y, ldy, s);
    if (M > 1 && 2 * row <= kMaxSmem) return gemm_launch<2, MODE>(w, x, M, N, K, y, ldy, s);
    if (row <= kMaxSmem) return gemm_launch<1, MODE>(w, x, M, N, K, y, ldy, s);
    return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------- RMSNorm
__global__ void rmsnorm_f32_kernel(const float* __restrict__ x, const float* __restrict__ w, int H,
                                   float eps, float* __restrict__ y) {
    __shared__ float sh[32];
    const int m = blockIdx.x;
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)m * H);
    float ss = 0.0f;
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x) {
        const float4 v = xr[i];
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = ss;
    __syncthreads();
    float t = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += sh[i];
    const float rms = sqrtf(t / (float)H + eps);
    const float4* wr = reinterpret_cast<const float4*>(w);
    float4* yr = reinterpret_cast<float4*>(y + (size_t)m * H);
    for (int i = threadIdx.x; i < H / 4; i += blockDim.x) {
        const float4 v = xr[i], g = wr[i];
        yr[i] = make_float4((v.x / rms) * g.x, (v.y / rms) * g.y, (v.z / rms) * g.z, (v.w / rms) * g.w);
    }
}

// ------------------------------------------------------------ RoPE + split
__global__ void rope_split_f32_kernel(const float* __restrict__ qkv, const uint64_t* __restrict__ anc,
                                      const int32_t* __restrict__ ctx_len, int N, int Hq, int Hkv,
                                      int D, float freq_base, float* __restrict__ q,
                                      float* __restrict__ nk, float* __restrict__ nv) {
    __shared__ float cs[128], sn[128];
    const int m = blockIdx.x, b = m / N, half = D / 2;
    const int pos = ctx_len[b] + __popcll(anc[m]) - 1;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        const float theta = (float)pos / powf(freq_base, 2.0f * (float)i / (float)D);
        sn[i] = sinf(theta);
        cs[i] = cosf(theta);
    }
    __syncthreads();
    const int heads = Hq + 2 * Hkv;
    for (int wi = threadIdx.x; wi < heads * half; wi += blockDim.x) {
        const int hh = wi / half, i = wi - hh * half;
        const float* src = qkv + ((size_t)m * heads + hh) * D;
        float x0 = src[i], x1 = src[i + half];
        if (hh < Hq + Hkv) {
            const float c = cs[i], s = sn[i];
            const float r0 = x0 * c - x1 * s, r1 = x0 * s + x1 * c;
            x0 = r0;
            x1 = r1;
        }
        float* dst = hh < Hq         ? q + ((size_t)m * Hq + hh) * D
                     : hh < Hq + Hkv ? nk + ((size_t)m * Hkv + (hh - Hq)) * D
                                     : nv + ((size_t)m * Hkv + (hh - Hq - Hkv)) * D;
        dst[i] = x0;
        dst[i + half] = x1;
    }
}

// -------------------------------------------------------- tree attention
// One CTA (4 warps) per query row (b, n, head).  The keys -- the cached prefix
// [0, ctx_len) through the page table, then the tree nodes j whose bit is set
// in anc[b][n] -- come in chunks of 32, one key per lane; warp w takes chunks
// w, w + 4, ...  A lane scores its key against the q row (broadcast from
// shared memory) while cp.async copies its V row into the warp's staging
// rows; P V then runs with lane-owned dimensions (d = lane + 32 i) over the
// staged rows, so every load of a chunk is in flight at once.  Each warp
// keeps an online softmax; the four states are merged at the end.
constexpr int kAttnWarps = 4;

__host__ __device__ constexpr int attn_f32_smem(int D) {
    return (D + kAttnWarps * 32 * D + kAttnWarps * (D + 2)) * 4;
}

template <int DW>
__global__ void __launch_bounds__(kAttnWarps * 32) tree_attn_f32_kernel(const TreeAttnF32Args a) {
    constexpr int D = DW * 32;
    extern __shared__ __align__(16) float sm[];
    float* qs = sm;                                 // [D]
    float* vs = qs + D;                             // [warps][32][D]
    float* os = vs + kAttnWarps * 32 * D;           // [warps][D]
    float* ms = os + kAttnWarps * D;                // [warps]
    float* ls = ms + kAttnWarps;                    // [warps]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x;
    const int hq = row % a.Hq, bn = row / a.Hq, b = bn / a.N;
    const int hkv = hq / (a.Hq / a.Hkv);
    for (int d = threadIdx.x; d < D; d += blockDim.x) qs[d] = a.q[(size_t)row * D + d];
    __syncthreads();
    const float4* q4 = reinterpret_cast<const float4*>(qs);
    float* vw = vs + warp * 32 * D;
    const float inv_sqrt_d = 1.0f / sqrtf((float)D);
    const int ctx = a.ctx_len[b];
    const uint64_t amask = a.anc[bn];
    const int total = ctx + a.N;
    const uint32_t* pt = a.page_table + (size_t)b * a.max_pages;
    float m_run = -INFINITY, l_run = 0.0f, o[DW];
#pragma unroll
    for (int i = 0; i < DW; ++i) o[i] = 0.0f;
    for (int c0 = 32 * warp; c0 < total; c0 += 32 * kAttnWarps) {
        const int t = c0 + lane;
        const float* kp = nullptr;
        const float* vp = nullptr;
        if (t < ctx) {
            const int pi = t >> 4;
            const uint32_t pg = pi < a.max_pages ? pt[pi] : 0xffffffffu;
            if (pg < (uint32_t)a.pool_pages) {
                const size_t tok = ((size_t)pg * a.Hkv + hkv) * 16 + (t & 15);
                kp = a.k_pool + tok * D;
                vp = a.v_pool + tok * D;
            } else {
                atomicCAS(a.err, 0, kErrPageF32);
            }
        } else if (t < total) {
            const int j = t - ctx;
            if ((amask >> j) & 1ull) {
                const size_t r = (((size_t)b * a.N + j) * a.Hkv + hkv) * D;
                kp = a.node_k + r;
                vp = a.node_v + r;
            }
        }
        if (vp) {  // V row -> this lane's staging row, asynchronously
            const unsigned dst = (unsigned)__cvta_generic_to_shared(vw + lane * D);
#pragma unroll
            for (int d4 = 0; d4 < D / 4; ++d4)
                asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(dst + 16 * d4),
                             "l"(vp + 4 * d4)
                             : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        float s = -INFINITY;
        if (kp) {
            const float4* k4 = reinterpret_cast<const float4*>(kp);
            float dot = 0.0f;
#pragma unroll
            for (int d4 = 0; d4 < D / 4; ++d4) {
                const float4 kv = __ldg(k4 + d4), qv = q4[d4];
                dot = fmaf(qv.x, kv.x, dot);
                dot = fmaf(qv.y, kv.y, dot);
                dot = fmaf(qv.z, kv.z, dot);
                dot = fmaf(qv.w, kv.w, dot);
            }
            s = dot * inv_sqrt_d;
        }
        const unsigned live = __ballot_sync(0xffffffffu, kp != nullptr);
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncwarp();
        if (live) {
            const float cmax = warp_max(s);
            const float m_new = fmaxf(m_run, cmax);
            const float corr = expf(m_run - m_new);  // 0 on the first visible chunk
            const float p = kp ? expf(s - m_new) : 0.0f;
            l_run = l_run * corr + warp_sum(p);
#pragma unroll
            for (int i = 0; i < DW; ++i) o[i] *= corr;
#pragma unroll 8
            for (int j = 0; j < 32; ++j) {
                const float pj = __shfl_sync(0xffffffffu, p, j);
                if ((live >> j) & 1u) {
#pragma unroll
                    for (int i = 0; i < DW; ++i) o[i] = fmaf(pj, vw[j * D + lane + 32 * i], o[i]);
                }
            }
            m_run = m_new;
        }
        __syncwarp();  // the staging rows are rewritten by the next chunk
    }
    // merge the warps' states
#pragma unroll
    for (int i = 0; i < DW; ++i) os[warp * D + lane + 32 * i] = o[i];
    if (lane == 0) {
        ms[warp] = m_run;
        ls[warp] = l_run;
    }
    __syncthreads();
    if (warp == 0) {
        float M = -INFINITY;
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, ms[w]);
        float L = 0.0f, acc[DW];
#pragma unroll
        for (int i = 0; i < DW; ++i) acc[i] = 0.0f;
        for (int w = 0; w < kAttnWarps; ++w) {
            const float f = ls[w] > 0.0f ? expf(ms[w] - M) : 0.0f;
            L += ls[w] * f;
#pragma unroll
            for (int i = 0; i < DW; ++i) acc[i] = fmaf(os[w * D + lane + 32 * i], f, acc[i]);
        }
        const float inv_l = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll
        for (int i = 0; i < DW; ++i) a.out[(size_t)row * D + lane + 32 * i] = acc[i] * inv_l;
    }
}

// -------------------------------------------------------------- KV commit
// one warp per (sequence, path position, layer, kv head)
__global__ void kv_commit_f32_kernel(const KvCommitF32Args a) {
    const long warp = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const long total = (long)a.B * a.N * a.L * a.Hkv;
    if (warp >= total) return;
    const int h = (int)(warp % a.Hkv);
    const int l = (int)((warp / a.Hkv) % a.L);
    const int i = (int)((warp / ((long)a.Hkv * a.L)) % a.N);
    const int b = (int)(warp / ((long)a.Hkv * a.L * a.N));
    if (i >= a.path_len[b]) return;
    const int node = a.path[(size_t)b * a.N + i];
    const int pos = a.ctx_len[b] + i;
    const int pi = pos / 16;
    const uint32_t row = a.slots ? a.slots[b] : (uint32_t)b;
    if (node < 0 || node >= a.N || pi >= a.max_pages) {
        if (lane == 0) atomicCAS(a.err, 0, kErrCommitF32);
        return;
    }
    const uint32_t pg = a.page_table[(size_t)row * a.max_pages + pi];
    if (pg >= (uint32_t)a.pool_pages) {
        if (lane == 0) atomicCAS(a.err, 0, kErrCommitF32);
        return;
    }
    const size_t src = (((size_t)l * a.B * a.N + (size_t)b * a.N + node) * a.Hkv + h) * a.D;
    const size_t dst = ((((size_t)l * a.pool_pages + pg) * a.Hkv + h) * 16 + pos % 16) * a.D;
    const float4* sk = reinterpret_cast<const float4*>(a.node_k + src);
    const float4* sv = reinterpret_cast<const float4*>(a.node_v + src);
    float4* dk = reinterpret_cast<float4*>(a.k_pool + dst);
    float4* dv = reinterpret_cast<float4*>(a.v_pool + dst);
    for (int d4 = lane; d4 < a.D / 4; d4 += 32) {
        dk[d4] = sk[d4];
        dv[d4] = sv[d4];
    }
}

}  // namespace

cudaError_t launch_gemm_f32(const float* w, const float* x, int M, int N, int K, float* y, int ldy,
                            int mode, cudaStream_t s) {
    if (M == 0 || N == 0) return cudaSuccess;
    if (K % 4 || (reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x)) & 15)
        return cudaErrorInvalidValue;
    switch (mode) {
        case kF32Store: return gemm_mode<kF32Store>(w, x, M, N, K, y, ldy, s);
        case kF32Add: return gemm_mode<kF32Add>(w, x, M, N, K, y, ldy, s);
        case kF32SwiGLU: return gemm_mode<kF32SwiGLU>(w, x, M, N, K, y, ldy, s);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_rmsnorm_f32(const float* x, const float* w, int M, int H, float eps, float* y,
                               cudaStream_t s) {
    if (M == 0) return cudaSuccess;
    rmsnorm_f32_kernel<<<M, 256, 0, s>>>(x, w, H, eps, y);
    return cudaGetLastError();
}

cudaError_t launch_rope_split_f32(const float* qkv, const uint64_t* anc, const int32_t* ctx_len,
                                  int B, int N, int Hq, int Hkv, int D, float freq_base, float* q,
                                  float* nk, float* nv, cudaStream_t s) {
    if (B * N == 0) return cudaSuccess;
    if (D % 2 || D > 256) return cudaErrorInvalidValue;
    rope_split_f32_kernel<<<B * N, 256, 0, s>>>(qkv, anc, ctx_len, N, Hq, Hkv, D, freq_base, q, nk, nv);
    return cudaGetLastError();
}

template <int DW>
cudaError_t attn_f32_launch(const TreeAttnF32Args& a, unsigned grid, cudaStream_t s) {
    constexpr int smem = attn_f32_smem(DW * 32);
    static SmemAttr attr;
    const cudaError_t ea = ensure_smem(attr, tree_attn_f32_kernel<DW>, smem);
    if (ea != cudaSuccess) return ea;
    tree_attn_f32_kernel<DW><<<grid, kAttnWarps * 32, smem, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_tree_attention_f32(const TreeAttnF32Args& a, cudaStream_t s) {
    const long rows = (long)a.B * a.N * a.Hq;
    if (rows == 0) return cudaSuccess;
    if (a.N > 64 || a.Hkv <= 0 || a.Hq % a.Hkv) return cudaErrorInvalidValue;
    if (a.D == 64) return attn_f32_launch<2>(a, (unsigned)rows, s);
    if (a.D == 128) return attn_f32_launch<4>(a, (unsigned)rows, s);
    return cudaErrorInvalidValue;
}

cudaError_t launch_kv_commit_f32(const KvCommitF32Args& a, cudaStream_t s) {
    const long warps = (long)a.B * a.N * a.L * a.Hkv;
    if (warps == 0) return cudaSuccess;
    if (a.D % 4) return cudaErrorInvalidValue;
    kv_commit_f32_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace velo
