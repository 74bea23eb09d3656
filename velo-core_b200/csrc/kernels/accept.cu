// accept.cu -- fused vocabulary-wide softmax + acceptance (one launch).
//
// Replaces, for the verify step, GreedyTargetModel::verify_batch's host
// GreedySampler scan (src/backend.rs:337-369, src/sampling.rs:39-58) and the
// prefix rule of SpeculativeSession::draft / commit (src/speculative.rs:441-467,
// 473-519); adds rejection sampling (Leviathan et al. 2023; Chen et al. 2023),
// which the reference does not have.
//
// Work decomposition (no thread ever waits on another):
//  Kernel A (stream), persistent grid.  The vocabulary of each row is cut into
//   tiles of 1024 logits; a warp reads one (sequence, row, tile) item with
//   eight 16-byte loads per lane (lane l owns elements 1024t + 128i + 4l + c,
//   i < 8, c < 4) and stores (max, sum of exponentials) -- or (max, last
//   argmax) for greedy -- to the workspace, plus the logit at the row's draft
//   token when the token falls in the tile.  Warps stride over all items.
//  Kernel B (finish), launched as a programmatic dependent of A so its launch
//   overlaps A's tail.  Every CTA of a sequence stages the sequence's tile
//   statistics in shared memory with asynchronous copies (one round trip),
//   reduces each row in tile order (a thread per row) and runs the accept
//   tests (a thread per position).  Greedy: one CTA per sequence writes the
//   result.  Sampling: ceil(ntiles / 8) CTAs per sequence each weigh 8 tiles
//   of the row pair the draw needs (a warp per tile; the draw is compute
//   bound, so it is spread over the GPU), and the CTA taking the sequence's
//   last ticket selects the token by a three-level inverse CDF
//   (tile -> lane -> element).
//
// The per-element exponentials use packed f32x2 FMAs (two IEEE operations per
// instruction).  The arithmetic order is the spec the CPU oracle restates;
// decisions and tokens are bit-identical given the same logits and uniforms.
#include <cuda_runtime.h>
#include <cstdint>

#include "common/smem_attr.cuh"
#include "common/spec_math.cuh"
#include "kernels/accept.h"

namespace velo {
namespace {

constexpr int kTile = 1024;
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kFinThreads = 256;    // finish kernel: ceil(ntiles / 8) CTAs per sequence
constexpr int kFinWarps = kFinThreads / 32;

// Load `n4` consecutive float4 groups (i = i0 .. i0+n4-1) of the elements lane
// `lane` owns in tile t.  Absent elements read as -inf.
template <int n4>
__device__ __forceinline__ void load_groups(const float* __restrict__ row, int V, int t, int lane,
                                            int i0, bool vec, float* x) {
    const int base = t * kTile + 4 * lane;
#pragma unroll
    for (int q = 0; q < n4; ++q) {
        const int e = base + 128 * (i0 + q);
        if (vec) {
            if (e < V) {
                const float4 v = __ldg(reinterpret_cast<const float4*>(row + e));
                x[4 * q + 0] = v.x;
                x[4 * q + 1] = v.y;
                x[4 * q + 2] = v.z;
                x[4 * q + 3] = v.w;
            } else {
#pragma unroll
                for (int c = 0; c < 4; ++c) x[4 * q + c] = -INFINITY;
            }
        } else {
#pragma unroll
            for (int c = 0; c < 4; ++c) x[4 * q + c] = (e + c < V) ? __ldg(row + e + c) : -INFINITY;
        }
    }
}

__device__ __forceinline__ bool elem_valid(int V, int t, int lane, int i, int c) {
    return t * kTile + 128 * i + 4 * lane + c < V;
}

// (m_t, z_t) of the spec for one tile.
template <bool kFullTile>
__device__ __forceinline__ float2 tile_stats(const float* x, int V, int t, int lane, float inv_t) {
    // maximum as a tree (max is exact in any order): 32 -> 11 -> 4 -> 1
    float m1[11];
#pragma unroll
    for (int j = 0; j < 10; ++j) m1[j] = max3(x[3 * j], x[3 * j + 1], x[3 * j + 2]);
    m1[10] = fmaxf(x[30], x[31]);
    const float m2a = max3(m1[0], m1[1], m1[2]), m2b = max3(m1[3], m1[4], m1[5]);
    const float m2c = max3(m1[6], m1[7], m1[8]), m2d = fmaxf(m1[9], m1[10]);
    float mx = fmaxf(max3(m2a, m2b, m2c), m2d);
    mx = warp_max(mx);
    const float m = __fmul_rn(mx, inv_t);
    const float2 it = f2(inv_t), nm = f2(-m);
    float2 a01 = f2(0.0f), a23 = f2(0.0f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float2 e01 = spec_exp2(__ffma2_rn(make_float2(x[4 * i], x[4 * i + 1]), it, nm));
        float2 e23 = spec_exp2(__ffma2_rn(make_float2(x[4 * i + 2], x[4 * i + 3]), it, nm));
        if (!kFullTile) {  // absent elements add exactly +0 (same as skipping them)
            if (!elem_valid(V, t, lane, i, 0)) e01.x = 0.0f;
            if (!elem_valid(V, t, lane, i, 1)) e01.y = 0.0f;
            if (!elem_valid(V, t, lane, i, 2)) e23.x = 0.0f;
            if (!elem_valid(V, t, lane, i, 3)) e23.y = 0.0f;
        }
        a01 = __fadd2_rn(a01, e01);
        a23 = __fadd2_rn(a23, e23);
    }
    const float z = warp_butterfly_sum(lane_combine(a01, a23));
    return make_float2(m, z);
}

template <bool kFullTile>
__device__ __forceinline__ ArgMax tile_argmax(const float* x, int V, int t, int lane) {
    ArgMax best{-INFINITY, -1};
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int e = t * kTile + 128 * i + 4 * lane + c;
            if ((kFullTile || e < V) && x[4 * i + c] >= best.v) {
                best.v = x[4 * i + c];
                best.idx = e;
            }
        }
    return warp_argmax(best);
}

__device__ __forceinline__ const float* target_row(const AcceptParams& p, int b, int row) {
    return p.tgt + ((size_t)b * (p.k + 1) + row) * (size_t)p.V;
}
__device__ __forceinline__ const float* draft_row(const AcceptParams& p, int b, int row) {
    return p.drf + ((size_t)b * p.k + row) * (size_t)p.V;
}

// ---------------------------------------------------------------- kernel A
template <bool kGreedy>
__global__ void __launch_bounds__(kThreads, 4) accept_stream_kernel(AcceptParams p) {
    // the finish kernel may be scheduled as soon as SMs free up; it waits for
    // this grid's completion (griddepcontrol.wait) before reading its results
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gw = blockIdx.x * kWarps + warp, nw = gridDim.x * kWarps;
    const int per_seq = p.nrows * p.ntiles;
    const int items = p.B * per_seq;
    for (int it = gw; it < items; it += nw) {
        const int b = it / per_seq, rem = it - b * per_seq;
        const int row = rem / p.ntiles, t = rem - row * p.ntiles;
        const float* rp = row <= p.k ? target_row(p, b, row) : draft_row(p, b, row - p.k - 1);
        // draft token of this row (rows 0..k-1 target, k+1..2k draft)
        const int pos = row < p.k ? row : row - p.k - 1;
        uint32_t x = 0xffffffffu;
        if (!kGreedy && row != p.k && lane == 0) x = __ldg(p.tok + (size_t)b * p.k + pos);
        const bool full = (t + 1) * kTile <= p.V;
        float2 part;
        {
            float xv[32];
            load_groups<8>(rp, p.V, t, lane, 0, p.vec4, xv);
            if (kGreedy) {
                const ArgMax a = full ? tile_argmax<true>(xv, p.V, t, lane)
                                      : tile_argmax<false>(xv, p.V, t, lane);
                part = make_float2(a.v, __int_as_float(a.idx));
            } else {
                part = full ? tile_stats<true>(xv, p.V, t, lane, p.inv_t)
                            : tile_stats<false>(xv, p.V, t, lane, p.inv_t);
            }
        }
        if (lane == 0) {
            p.part[(size_t)b * per_seq + rem] = part;
            if (!kGreedy && x < (uint32_t)p.V && (int)(x >> 10) == t)
                p.tokval[(size_t)b * p.nrows + row] = __ldg(rp + x);
        }
    }
}

// ---------------------------------------------------------------- kernel B
struct FinishLayout {
    int stage, rowM, rowR, lane_w, tile_w, elem_w, misc, bytes;
};

__host__ __device__ inline FinishLayout finish_layout(int nrows, int ntiles) {
    auto up = [](int x) { return (x + 15) & ~15; };
    FinishLayout L;
    int o = 0;
    L.stage = o;  o += up((nrows * ntiles + 2) * 8);
    L.rowM = o;   o += up(nrows * 4);
    L.rowR = o;   o += up(nrows * 4);
    L.lane_w = o; o += up(ntiles * 32 * 4);  // every tile's lane weights (the drawing CTA)
    L.tile_w = o; o += up(ntiles * 4);
    L.elem_w = o; o += up(32 * 4);
    L.misc = o;   o += 64;
    L.bytes = o;
    return L;
}

struct Draw {
    int r, resid;
    float Mt, Rt, Md, Rd;
};

__device__ __forceinline__ float elem_weight(const Draw& d, float inv_t, float tv, float dv) {
    const float P = __fmul_rn(spec_exp(__fmaf_rn(tv, inv_t, -d.Mt)), d.Rt);
    if (!d.resid) return P;
    const float Q = __fmul_rn(spec_exp(__fmaf_rn(dv, inv_t, -d.Md)), d.Rd);
    return P > Q ? __fadd_rn(P, -Q) : 0.0f;
}

// Two weights at once (identical bits to elem_weight on each component).
__device__ __forceinline__ float2 elem_weight2(const Draw& d, float inv_t, float2 tv, float2 dv) {
    const float2 P = __fmul2_rn(spec_exp2(__ffma2_rn(tv, f2(inv_t), f2(-d.Mt))), f2(d.Rt));
    if (!d.resid) return P;
    const float2 Q = __fmul2_rn(spec_exp2(__ffma2_rn(dv, f2(inv_t), f2(-d.Md))), f2(d.Rd));
    const float2 D = __ffma2_rn(Q, f2(-1.0f), P);  // P - Q with one rounding
    return make_float2(P.x > Q.x ? D.x : 0.0f, P.y > Q.y ? D.y : 0.0f);
}

// Weigh tile t of the draw row pair: lane weight -> lane_w[t*32 + lane],
// tile weight (warp butterfly) -> tile_w[t].  Both rows' tile is loaded up
// front (one round trip to memory).
__device__ void weigh_tile(const AcceptParams& p, const float* trow, const float* drow,
                           const Draw& d, int t, int lane, float* lane_w, float* tile_w) {
    const bool full = (t + 1) * kTile <= p.V;
    float tx[32], dx[32];
    load_groups<8>(trow, p.V, t, lane, 0, p.vec4, tx);
    if (d.resid) load_groups<8>(drow, p.V, t, lane, 0, p.vec4, dx);
    float2 a01 = f2(0.0f), a23 = f2(0.0f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float2 w01 = elem_weight2(d, p.inv_t, make_float2(tx[4 * i], tx[4 * i + 1]),
                                  d.resid ? make_float2(dx[4 * i], dx[4 * i + 1]) : f2(0.0f));
        float2 w23 = elem_weight2(d, p.inv_t, make_float2(tx[4 * i + 2], tx[4 * i + 3]),
                                  d.resid ? make_float2(dx[4 * i + 2], dx[4 * i + 3]) : f2(0.0f));
        if (!full) {
            if (!elem_valid(p.V, t, lane, i, 0)) w01.x = 0.0f;
            if (!elem_valid(p.V, t, lane, i, 1)) w01.y = 0.0f;
            if (!elem_valid(p.V, t, lane, i, 2)) w23.x = 0.0f;
            if (!elem_valid(p.V, t, lane, i, 3)) w23.y = 0.0f;
        }
        a01 = __fadd2_rn(a01, w01);
        a23 = __fadd2_rn(a23, w23);
    }
    const float lw = lane_combine(a01, a23);
    lane_w[t * 32 + lane] = lw;
    const float tw = warp_butterfly_sum(lw);
    if (lane == 0) tile_w[t] = tw;
}

// Sequential selection rule of the spec over n weights in shared memory:
// the first child whose running sum exceeds tau (and whose weight is
// positive); fallback: the last positive child, tau' = its weight.
__device__ int select_level(const float* w, int n, float tau, float* tau_out) {
    float acc = 0.0f;
    int last = -1;
    for (int i0 = 0; i0 < n; i0 += 8) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = i0 + j < n ? w[i0 + j] : 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (i0 + j >= n) break;
            const float nxt = __fadd_rn(acc, v[j]);
            if (v[j] > 0.0f) {
                last = i0 + j;
                if (nxt > tau) {
                    *tau_out = __fadd_rn(tau, -acc);
                    return i0 + j;
                }
            }
            acc = nxt;
        }
    }
    if (last >= 0) *tau_out = w[last];
    return last;
}

template <bool kGreedy>
__global__ void __launch_bounds__(kFinThreads) accept_finish_kernel(AcceptParams p, int ctas_per_seq) {
    extern __shared__ __align__(16) unsigned char smem[];
    const FinishLayout L = finish_layout(p.nrows, p.ntiles);
    float2* stage = reinterpret_cast<float2*>(smem + L.stage);
    float* rowM = reinterpret_cast<float*>(smem + L.rowM);
    float* rowR = reinterpret_cast<float*>(smem + L.rowR);
    float* lane_w = reinterpret_cast<float*>(smem + L.lane_w);
    float* tile_w = reinterpret_cast<float*>(smem + L.tile_w);
    float* elem_w = reinterpret_cast<float*>(smem + L.elem_w);
    int* misc = reinterpret_cast<int*>(smem + L.misc);
    float* miscf = reinterpret_cast<float*>(smem + L.misc);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int b = blockIdx.x / ctas_per_seq, cb = blockIdx.x % ctas_per_seq;

    asm volatile("griddepcontrol.wait;" ::: "memory");  // kernel A complete and visible

    // ---- stage the tile statistics (async copies, L2 only) --------------
    const int n = p.nrows * p.ntiles;
    const float2* src = p.part + (size_t)b * n;
    const int a = ((uintptr_t)src & 15) ? 1 : 0;  // element e lands at stage[e + a]
    {
        const float4* src16 = reinterpret_cast<const float4*>(src - a);
        const int n16 = (n + a + 1) / 2;
        for (int j = tid; j < n16; j += kFinThreads) {
            const unsigned dst = (unsigned)__cvta_generic_to_shared(&stage[2 * j]);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src16 + j) : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    // accept-test inputs, loaded while the copies fly (thread i: position i)
    uint32_t xi[2] = {0u, 0u};
    float tv[2] = {0.0f, 0.0f}, dv[2] = {0.0f, 0.0f}, ui[2] = {0.0f, 0.0f};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int i = tid + h * kFinThreads;
        if (i < p.k) {
            xi[h] = __ldg(p.tok + (size_t)b * p.k + i);
            if (!kGreedy) {
                tv[h] = __ldcg(p.tokval + (size_t)b * p.nrows + i);
                dv[h] = __ldcg(p.tokval + (size_t)b * p.nrows + p.k + 1 + i);
                ui[h] = __ldg(p.u + (size_t)b * (p.k + 1) + i);
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();

    // ---- row statistics ----------------------------------------------------
    // (1) a warp per row: max over tiles (exact, any order) or greedy argmax
    for (int row = warp; row < p.nrows; row += kFinWarps) {
        const float2* rp = stage + a + row * p.ntiles;
        if (kGreedy) {
            ArgMax best{-INFINITY, -1};
            for (int t = lane; t < p.ntiles; t += 32)
                best = argmax_combine(best, ArgMax{rp[t].x, __float_as_int(rp[t].y)});
            best = warp_argmax(best);
            if (lane == 0) rowM[row] = __int_as_float(best.idx < 0 ? 0 : best.idx);
        } else {
            float M = -INFINITY;
            for (int t = lane; t < p.ntiles; t += 32) M = fmaxf(M, rp[t].x);
            M = warp_max(M);
            if (lane == 0) rowM[row] = M;
        }
    }
    if (!kGreedy) {
        __syncthreads();
        // (2) one exponential per (row, tile): m_t is replaced by E(m_t - M)
        for (int e = tid; e < n; e += kFinThreads) {
            const int row = e / p.ntiles;
            float2& v = stage[a + e];
            v.x = spec_exp(__fadd_rn(v.x, -rowM[row]));
        }
        __syncthreads();
        // (3) a thread per row: Z = fma chain over tiles in order
        for (int row = tid; row < p.nrows; row += kFinThreads) {
            const float2* rp = stage + a + row * p.ntiles;
            float Z = 0.0f;
            int t = 0;
            for (; t + 8 <= p.ntiles; t += 8) {
                float2 v[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = rp[t + j];
#pragma unroll
                for (int j = 0; j < 8; ++j) Z = __fmaf_rn(v[j].y, v[j].x, Z);
            }
            for (; t < p.ntiles; ++t) Z = __fmaf_rn(rp[t].y, rp[t].x, Z);
            rowR[row] = __fdiv_rn(1.0f, Z);
        }
    }
    if (tid == 0) misc[0] = p.k;
    __syncthreads();

    // ---- accept tests: a thread per position, first rejection wins ------
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int i = tid + h * kFinThreads;
        if (i < p.k) {
            bool rej;
            if (xi[h] >= (uint32_t)p.V) {  // bad input on the device path
                if (cb == 0) atomicOr(p.err_flag, 1);
                rej = true;
            } else if (kGreedy) {
                rej = (int)xi[h] != __float_as_int(rowM[i]);
            } else {
                const float P = __fmul_rn(spec_exp(__fmaf_rn(tv[h], p.inv_t, -rowM[i])), rowR[i]);
                const float Q = __fmul_rn(spec_exp(__fmaf_rn(dv[h], p.inv_t, -rowM[p.k + 1 + i])),
                                          rowR[p.k + 1 + i]);
                rej = !(__fmul_rn(ui[h], Q) <= P);
            }
            if (rej) atomicMin(&misc[0], i);
        }
    }
    __syncthreads();
    const int r = misc[0];
    if (kGreedy) {
        if (tid == 0) {
            p.acc_len[b] = r;
            p.bonus[b] = (uint32_t)__float_as_int(rowM[r]);
        }
        return;
    }

    // ---- residual / bonus weights of this CTA's tiles -------------------
    Draw d;
    d.r = r;
    d.resid = r < p.k;
    d.Mt = rowM[r];
    d.Rt = rowR[r];
    d.Md = d.resid ? rowM[p.k + 1 + r] : 0.0f;
    d.Rd = d.resid ? rowR[p.k + 1 + r] : 0.0f;
    const float* trow = target_row(p, b, r);
    const float* drow = d.resid ? draft_row(p, b, r) : nullptr;
    float* g_lane_w = p.lane_w + (size_t)b * p.ntiles * 32;
    float* g_tile_w = p.tile_w + (size_t)b * p.ntiles;
    for (int t = cb * kFinWarps + warp; t < p.ntiles; t += ctas_per_seq * kFinWarps)
        weigh_tile(p, trow, drow, d, t, lane, g_lane_w, g_tile_w);
    __threadfence();
    __syncthreads();
    if (tid == 0) misc[5] = (int)atomicAdd(&p.done[b], 1u);
    __syncthreads();
    if (misc[5] != ctas_per_seq - 1) return;
    // ---- the CTA with the last ticket draws the token --------------------
    if (tid == 0) p.done[b] = 0u;  // every CTA of b counted: zero for the next launch
    __threadfence();
    // tile and lane weights of every tile in one round trip to L2
    for (int t = tid; t < p.ntiles; t += kFinThreads) tile_w[t] = __ldcg(g_tile_w + t);
    for (int e = tid; e < p.ntiles * 32; e += kFinThreads) lane_w[e] = __ldcg(g_lane_w + e);
    __syncthreads();
    if (tid == 0) {
        float total = 0.0f;
        for (int t0 = 0; t0 < p.ntiles; t0 += 8) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = t0 + j < p.ntiles ? tile_w[t0 + j] : 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (t0 + j < p.ntiles) total = __fadd_rn(total, v[j]);
        }
        miscf[1] = total;
    }
    __syncthreads();
    if (!(miscf[1] > 0.0f) && d.resid) {
        // residual mass vanished: weigh p of the same row instead (this CTA)
        d.resid = 0;
        drow = nullptr;
        for (int t = warp; t < p.ntiles; t += kFinWarps) weigh_tile(p, trow, drow, d, t, lane, g_lane_w, tile_w);
        __threadfence();
        __syncthreads();
        for (int e = tid; e < p.ntiles * 32; e += kFinThreads) lane_w[e] = __ldcg(g_lane_w + e);
        if (tid == 0) {
            float total = 0.0f;
            for (int t = 0; t < p.ntiles; ++t) total = __fadd_rn(total, tile_w[t]);
            miscf[1] = total;
        }
        __syncthreads();
    }
    // tile level (thread 0), lane level (thread 0), element level (warp 0)
    if (tid == 0) {
        float tau1 = 0.0f;
        const float total = miscf[1];
        const float tau = __fmul_rn(__ldg(p.u + (size_t)b * (p.k + 1) + p.k), total);
        int ts = -1;
        if (total > 0.0f) ts = select_level(tile_w, p.ntiles, tau, &tau1);
        misc[2] = ts;
        miscf[4] = tau1;
    }
    __syncthreads();
    if (warp == 0) {
        const int ts = misc[2];
        int token = 0;
        if (ts >= 0) {
            float tau2 = 0.0f;
            int ls = -1;
            if (lane == 0) ls = select_level(lane_w + ts * 32, 32, miscf[4], &tau2);
            ls = __shfl_sync(0xffffffffu, ls, 0);
            tau2 = __shfl_sync(0xffffffffu, tau2, 0);
            if (ls >= 0) {
                const int e = ts * kTile + 128 * (lane >> 2) + 4 * ls + (lane & 3);
                float ew = 0.0f;
                if (e < p.V) ew = elem_weight(d, p.inv_t, __ldg(trow + e), d.resid ? __ldg(drow + e) : 0.0f);
                elem_w[lane] = ew;
                __syncwarp();
                if (lane == 0) {
                    float tau3;
                    const int es = select_level(elem_w, 32, tau2, &tau3);
                    token = es >= 0 ? ts * kTile + 128 * (es >> 2) + 4 * ls + (es & 3) : 0;
                }
            }
        }
        if (lane == 0) {
            p.acc_len[b] = r;
            p.bonus[b] = (uint32_t)token;
        }
    }
}

// ---------------------------------------------------------------- draft trees
// Rejection sampling over a draft tree (multi-candidate speculative sampling,
// SpecInfer: Miao et al. 2024, Algorithm 2), one CTA of 16 warps per
// sequence.  The walk is sequential by nature (a node's children are tested
// only after the node was accepted), so the CTA walks it and spreads each
// vocabulary pass over its warps (warp w takes tiles w, w + 16, ...):
//   stats pass   target row and draft row of the current node: tile (m, z) as
//                kernel A, then the row reduction of the finish kernel;
//   child test   one thread: u * Q(x) <= P_level(x);
//   residual     after a rejected child, the next level's weights
//                W_{j+1} = max(0, W_j R_j - Q) (W_1 = max(0, P - Q)) of every
//                element, their lane / tile sums and the ordered total;
//   draw         tile -> lane -> element inverse CDF of the final level, as
//                the finish kernel's draw.
// Every operation is the spec the CPU oracle restates (vo_accept_tree); on
// chains it is the chain rule above bit for bit.
constexpr int kTreeWarps = 16;
constexpr int kTreeThreads = kTreeWarps * 32;
constexpr int kTreeMaxLevel = 64;

// W_level of one element (level 0: P)
__device__ __forceinline__ float tree_weight(float tv, float dv, float inv_t, float Mt, float Rt,
                                             float Md, float Rd, const float* Rlev, int level) {
    float P = __fmul_rn(spec_exp(__fmaf_rn(tv, inv_t, -Mt)), Rt);
    if (level == 0) return P;
    const float Q = __fmul_rn(spec_exp(__fmaf_rn(dv, inv_t, -Md)), Rd);
    float W = 0.0f;
    for (int j = 1; j <= level; ++j) {
        W = P > Q ? __fadd_rn(P, -Q) : 0.0f;
        if (j < level) P = __fmul_rn(W, Rlev[j]);
    }
    return W;
}

// tree_weight of two elements at once (two IEEE operations per packed
// instruction: the same bits as two scalar calls; P - Q as fma(Q, -1, P), one
// rounding like the subtraction)
__device__ __forceinline__ float2 tree_weight2(float2 tv, float2 dv, float inv_t, float Mt, float Rt, float Md,
                                               float Rd, const float* Rlev, int level) {
    float2 P = __fmul2_rn(spec_exp2(__ffma2_rn(tv, f2(inv_t), f2(-Mt))), f2(Rt));
    if (level == 0) return P;
    const float2 Q = __fmul2_rn(spec_exp2(__ffma2_rn(dv, f2(inv_t), f2(-Md))), f2(Rd));
    float2 W = f2(0.0f);
    for (int j = 1; j <= level; ++j) {
        const float2 D = __ffma2_rn(Q, f2(-1.0f), P);
        W = make_float2(P.x > Q.x ? D.x : 0.0f, P.y > Q.y ? D.y : 0.0f);
        if (j < level) P = __fmul2_rn(W, f2(Rlev[j]));
    }
    return W;
}

// Weigh tile t at `level`: lane weight -> lane_w[t * 32 + lane], tile weight
// (warp butterfly) -> tile_w[t]; lane sums (acc0 + acc1) + (acc2 + acc3), acc_c
// sequential over i, as the chain draw.
__device__ __forceinline__ void tree_weigh_tile(const float* trow, const float* drow, int V, int t, int lane,
                                                bool vec4, float inv_t, float Mt, float Rt, float Md, float Rd,
                                                const float* Rlev, int level, float* lane_w, float* tile_w) {
    const bool full = (t + 1) * kTile <= V;
    float tx[32], dx[32];
    load_groups<8>(trow, V, t, lane, 0, vec4, tx);
    if (level > 0) load_groups<8>(drow, V, t, lane, 0, vec4, dx);
    float2 a01 = f2(0.0f), a23 = f2(0.0f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float2 w01 = tree_weight2(make_float2(tx[4 * i], tx[4 * i + 1]),
                                  level > 0 ? make_float2(dx[4 * i], dx[4 * i + 1]) : f2(0.0f), inv_t, Mt, Rt,
                                  Md, Rd, Rlev, level);
        float2 w23 = tree_weight2(make_float2(tx[4 * i + 2], tx[4 * i + 3]),
                                  level > 0 ? make_float2(dx[4 * i + 2], dx[4 * i + 3]) : f2(0.0f), inv_t, Mt,
                                  Rt, Md, Rd, Rlev, level);
        if (!full) {
            if (!elem_valid(V, t, lane, i, 0)) w01.x = 0.0f;
            if (!elem_valid(V, t, lane, i, 1)) w01.y = 0.0f;
            if (!elem_valid(V, t, lane, i, 2)) w23.x = 0.0f;
            if (!elem_valid(V, t, lane, i, 3)) w23.y = 0.0f;
        }
        a01 = __fadd2_rn(a01, w01);
        a23 = __fadd2_rn(a23, w23);
    }
    const float lw = lane_combine(a01, a23);
    lane_w[t * 32 + lane] = lw;
    const float tw = warp_butterfly_sum(lw);
    if (lane == 0) tile_w[t] = tw;
}

__global__ void __launch_bounds__(kTreeThreads) accept_tree_kernel(AcceptTreeParams p) {
    __shared__ float2 st_t[kAcceptMaxTiles], st_d[kAcceptMaxTiles];
    __shared__ float tile_w[kAcceptMaxTiles];
    __shared__ float lane_w[kAcceptMaxTiles * 32];
    __shared__ float Rlev[kTreeMaxLevel + 1];
    __shared__ float elem_w[32];
    __shared__ float sf[8];
    __shared__ int si[4];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int b = blockIdx.x, N = p.N, V = p.V;
    const int ntiles = (V + kTile - 1) / kTile;
    const float* tbase = p.tgt + (size_t)b * N * V;
    const float* dbase = p.drf + (size_t)b * (N - 1) * V;
    const uint32_t* tok = p.tok + (size_t)b * N;
    const int32_t* par = p.par + (size_t)b * N;
    const float* u = p.u + (size_t)b * N;
    int32_t* path = p.path + (size_t)b * N;
    for (int n = tid; n < N; n += kTreeThreads) path[n] = n == 0 ? 0 : -1;
    const float inv_t = p.inv_t;
    int cur = 0, len = 1;
    for (;;) {
        bool has_child = false;
        for (int c = cur + 1; c < N; ++c) has_child |= __ldg(par + c) == cur;
        const float* trow = tbase + (size_t)cur * V;
        const float* drow = has_child ? dbase + (size_t)cur * V : nullptr;
        // ---- stats pass over the node's target (and draft) row ----------
        for (int t = warp; t < ntiles; t += kTreeWarps) {
            const bool full = (t + 1) * kTile <= V;
            float x[32];
            load_groups<8>(trow, V, t, lane, 0, p.vec4, x);
            const float2 a = full ? tile_stats<true>(x, V, t, lane, inv_t) : tile_stats<false>(x, V, t, lane, inv_t);
            if (lane == 0) st_t[t] = a;
            if (has_child) {
                load_groups<8>(drow, V, t, lane, 0, p.vec4, x);
                const float2 d = full ? tile_stats<true>(x, V, t, lane, inv_t) : tile_stats<false>(x, V, t, lane, inv_t);
                if (lane == 0) st_d[t] = d;
            }
        }
        __syncthreads();
        if (warp < 2 && (warp == 0 || has_child)) {
            const float2* st = warp == 0 ? st_t : st_d;
            float M = -INFINITY;
            for (int t = lane; t < ntiles; t += 32) M = fmaxf(M, st[t].x);
            M = warp_max(M);
            if (lane == 0) sf[2 * warp] = M;
        }
        __syncthreads();
        for (int e = tid; e < 2 * ntiles; e += kTreeThreads) {
            const int row = e / ntiles, t = e - row * ntiles;
            if (row == 1 && !has_child) continue;
            float2* st = row == 0 ? st_t : st_d;
            st[t].x = spec_exp(__fadd_rn(st[t].x, -sf[2 * row]));
        }
        __syncthreads();
        if ((tid == 0) || (tid == 32 && has_child)) {
            const float2* st = tid == 0 ? st_t : st_d;
            float Z = 0.0f;
            for (int t = 0; t < ntiles; ++t) Z = __fmaf_rn(st[t].y, st[t].x, Z);
            sf[tid == 0 ? 1 : 3] = __fdiv_rn(1.0f, Z);
        }
        __syncthreads();
        const float Mt = sf[0], Rt = sf[1], Md = has_child ? sf[2] : 0.0f, Rd = has_child ? sf[3] : 0.0f;
        // ---- children in index order -------------------------------------
        int level = 0, weighed = -1, accepted = -1;
        float total = 0.0f;
        for (int c = cur + 1; c < N; ++c) {
            if (__ldg(par + c) != cur) continue;
            if (tid == 0) {
                const uint32_t x = __ldg(tok + c);
                int acc = 0;
                if (x >= (uint32_t)V) {
                    atomicOr(p.err_flag, 1);  // bad input: counted as a rejection
                } else {
                    const float tv = __ldg(trow + x), dv = __ldg(drow + x);
                    float P = tree_weight(tv, dv, inv_t, Mt, Rt, Md, Rd, Rlev, level);
                    if (level > 0) P = __fmul_rn(P, Rlev[level]);
                    const float Q = __fmul_rn(spec_exp(__fmaf_rn(dv, inv_t, -Md)), Rd);
                    acc = __fmul_rn(__ldg(u + c - 1), Q) <= P;
                }
                si[0] = acc;
            }
            __syncthreads();
            if (si[0]) {
                accepted = c;
                break;
            }
            ++level;  // the residual of this rejection: weights, sums, total
            for (int t = warp; t < ntiles; t += kTreeWarps)
                tree_weigh_tile(trow, drow, V, t, lane, p.vec4, inv_t, Mt, Rt, Md, Rd, Rlev, level, lane_w, tile_w);
            __syncthreads();
            if (tid == 0) {
                float tot = 0.0f;
                for (int t = 0; t < ntiles; ++t) tot = __fadd_rn(tot, tile_w[t]);
                sf[4] = tot;
                if (tot > 0.0f) {
                    Rlev[level] = __fdiv_rn(1.0f, tot);
                    si[1] = level;
                } else {
                    si[1] = 0;  // residual mass vanished: back to p
                }
            }
            __syncthreads();
            weighed = level;
            level = si[1];
            total = sf[4];
        }
        if (accepted >= 0) {
            if (tid == 0) path[len] = accepted;
            ++len;
            cur = accepted;
            __syncthreads();
            continue;
        }
        // ---- draw from the final level's weights ---------------------------
        if (weighed != level || level == 0) {
            for (int t = warp; t < ntiles; t += kTreeWarps)
                tree_weigh_tile(trow, drow, V, t, lane, p.vec4, inv_t, Mt, Rt, Md, Rd, Rlev, level, lane_w, tile_w);
            __syncthreads();
            if (tid == 0) {
                float tot = 0.0f;
                for (int t = 0; t < ntiles; ++t) tot = __fadd_rn(tot, tile_w[t]);
                sf[4] = tot;
            }
            __syncthreads();
            total = sf[4];
        }
        if (tid == 0) {
            float tau1 = 0.0f;
            const float tau = __fmul_rn(__ldg(u + N - 1), total);
            int ts = -1;
            if (total > 0.0f) ts = select_level(tile_w, ntiles, tau, &tau1);
            si[2] = ts;
            sf[5] = tau1;
        }
        __syncthreads();
        if (warp == 0) {
            const int ts = si[2];
            int token = 0;
            if (ts >= 0) {
                float tau2 = 0.0f;
                int ls = -1;
                if (lane == 0) ls = select_level(lane_w + ts * 32, 32, sf[5], &tau2);
                ls = __shfl_sync(0xffffffffu, ls, 0);
                tau2 = __shfl_sync(0xffffffffu, tau2, 0);
                if (ls >= 0) {
                    const int e = ts * kTile + 128 * (lane >> 2) + 4 * ls + (lane & 3);
                    float ew = 0.0f;
                    if (e < V)
                        ew = tree_weight(__ldg(trow + e), level > 0 ? __ldg(drow + e) : 0.0f, inv_t, Mt, Rt, Md,
                                         Rd, Rlev, level);
                    elem_w[lane] = ew;
                    __syncwarp();
                    if (lane == 0) {
                        float tau3;
                        const int es = select_level(elem_w, 32, tau2, &tau3);
                        token = es >= 0 ? ts * kTile + 128 * (es >> 2) + 4 * ls + (es & 3) : 0;
                    }
                }
            }
            if (lane == 0) {
                p.path_len[b] = len;
                p.bonus[b] = (uint32_t)token;
            }
        }
        break;
    }
}

size_t align_up(size_t x) { return (x + 255) & ~(size_t)255; }

template <bool kGreedy>
cudaError_t launch_finish(const AcceptParams& p, cudaStream_t stream) {
    const FinishLayout L = finish_layout(p.nrows, p.ntiles);
    static SmemAttr smem_attr;
    const cudaError_t ea = ensure_smem(smem_attr, accept_finish_kernel<kGreedy>, L.bytes);
    if (ea != cudaSuccess) return ea;
    const int ctas_per_seq = kGreedy ? 1 : (p.ntiles + kFinWarps - 1) / kFinWarps;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(p.B * ctas_per_seq));
    cfg.blockDim = dim3(kFinThreads);
    cfg.dynamicSmemBytes = (size_t)L.bytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, accept_finish_kernel<kGreedy>, p, ctas_per_seq);
}

}  // namespace

cudaError_t launch_accept_tree(const AcceptTreeParams& p, cudaStream_t stream) {
    if (p.B == 0) return cudaSuccess;
    if (p.N < 1 || p.N > kTreeMaxLevel || p.V < 1 || p.V > kAcceptMaxV) return cudaErrorInvalidValue;
    accept_tree_kernel<<<p.B, kTreeThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

size_t accept_workspace_bytes(int B, int k, int V, bool greedy) {
    const size_t ntiles = (size_t)(V + kTile - 1) / kTile;
    const size_t nrows = greedy ? k + 1 : 2 * k + 1;
    return align_up((size_t)B * nrows * ntiles * sizeof(float2)) +
           align_up((size_t)B * nrows * sizeof(float)) +
           align_up((size_t)B * ntiles * 32 * sizeof(float)) +
           align_up((size_t)B * ntiles * sizeof(float));
}

size_t accept_counter_bytes(int B) { return align_up((size_t)B * sizeof(unsigned)); }

void accept_bind_buffers(AcceptParams& p, void* ws, void* cnt, bool greedy) {
    const size_t ntiles = (size_t)(p.V + kTile - 1) / kTile;
    const size_t nrows = greedy ? p.k + 1 : 2 * p.k + 1;
    char* w = (char*)ws;
    p.part = (float2*)w;
    w += align_up((size_t)p.B * nrows * ntiles * sizeof(float2));
    p.tokval = (float*)w;
    w += align_up((size_t)p.B * nrows * sizeof(float));
    p.lane_w = (float*)w;
    w += align_up((size_t)p.B * ntiles * 32 * sizeof(float));
    p.tile_w = (float*)w;
    p.done = (unsigned*)cnt;
}

cudaError_t launch_accept(const AcceptParams& prm, bool greedy, int sm_count, cudaStream_t stream) {
    AcceptParams p = prm;
    p.ntiles = (p.V + kTile - 1) / kTile;
    p.nrows = greedy ? p.k + 1 : 2 * p.k + 1;
    const int items = p.B * p.nrows * p.ntiles;
    const int ctas_needed = (items + kWarps - 1) / kWarps;
    int grid = p.grid > 0 ? p.grid : sm_count * 4;
    if (grid > ctas_needed) grid = ctas_needed;
    if (grid < 1) grid = 1;
    if (greedy)
        accept_stream_kernel<true><<<grid, kThreads, 0, stream>>>(p);
    else
        accept_stream_kernel<false><<<grid, kThreads, 0, stream>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    return greedy ? launch_finish<true>(p, stream) : launch_finish<false>(p, stream);
}

}  // namespace velo
