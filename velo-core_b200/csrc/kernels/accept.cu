// accept.cu -- fused vocabulary-wide softmax + acceptance (one launch).
//
// Replaces, for the verify step, GreedyTargetModel::verify_batch's host
// GreedySampler scan (src/backend.rs:337-369, src/sampling.rs:39-58) and the
// prefix rule of SpeculativeSession::draft / commit (src/speculative.rs:441-467,
// 473-519); adds rejection sampling (Leviathan et al. 2023; Chen et al. 2023),
// which the reference does not have.
//
// Shape of the work.  The vocabulary of each row is cut into tiles of 1024
// logits.  One warp reads one (row, tile) with eight 16-byte loads per lane
// (lane l owns elements 1024t + 128i + 4l + c, i < 8, c < 4) and writes the
// tile's statistics to a workspace: (max, sum of exponentials) for sampling,
// or (max, last argmax index) for greedy.  A CTA of 8 warps takes 8 consecutive
// (row, tile) items of one sequence.  Every CTA bumps its sequence's counter;
// the CTA that arrives last (no spinning: an atomic ticket) combines the tile
// statistics in tile order, makes the accept/reject decisions, re-reads the
// single row pair the residual (or bonus) draw needs, draws the token by a
// three-level inverse CDF (tile -> lane -> element) and resets the counter.
// Every logit is read from HBM once, plus one row pair per sequence.
//
// The arithmetic order is the spec the CPU oracle restates; decisions and
// tokens are bit-identical given the same logits and uniforms.
#include <cuda_runtime.h>
#include <cstdint>

#include "common/spec_math.cuh"
#include "kernels/accept.h"

namespace velo {
namespace {

constexpr int kTile = 1024;
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

struct LaneTile {
    float x[32];
};

// Load the 32 logits lane `lane` owns in tile t of `row` (absent => not read).
__device__ __forceinline__ void load_lane(const float* __restrict__ row, int V, int t, int lane,
                                          bool vec, LaneTile& d) {
    const int base = t * kTile + 4 * lane;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int e = base + 128 * i;
        if (vec) {
            if (e < V) {
                const float4 v = __ldg(reinterpret_cast<const float4*>(row + e));
                d.x[4 * i + 0] = v.x;
                d.x[4 * i + 1] = v.y;
                d.x[4 * i + 2] = v.z;
                d.x[4 * i + 3] = v.w;
            } else {
#pragma unroll
                for (int c = 0; c < 4; ++c) d.x[4 * i + c] = 0.0f;
            }
        } else {
#pragma unroll
            for (int c = 0; c < 4; ++c) d.x[4 * i + c] = (e + c < V) ? __ldg(row + e + c) : 0.0f;
        }
    }
}

__device__ __forceinline__ bool elem_valid(int V, int t, int lane, int i, int c) {
    return t * kTile + 128 * i + 4 * lane + c < V;
}

// (m_t, z_t) of the spec for one tile.
__device__ __forceinline__ float2 tile_stats(const LaneTile& d, int V, int t, int lane, bool full,
                                             float inv_t) {
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 32; ++j)
        if (full || elem_valid(V, t, lane, j >> 2, j & 3)) mx = fmaxf(mx, d.x[j]);
    mx = warp_max(mx);
    const float m = __fmul_rn(mx, inv_t);
    const float neg_m = -m;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c)
            if (full || elem_valid(V, t, lane, i, c))
                acc[c] = __fadd_rn(acc[c], spec_exp(__fmaf_rn(d.x[4 * i + c], inv_t, neg_m)));
    const float z = warp_butterfly_sum(lane_combine(acc));
    return make_float2(m, z);
}

__device__ __forceinline__ ArgMax tile_argmax(const LaneTile& d, int V, int t, int lane, bool full) {
    ArgMax best{-INFINITY, -1};
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int e = t * kTile + 128 * i + 4 * lane + c;
            if ((full || e < V) && d.x[4 * i + c] >= best.v) {
                best.v = d.x[4 * i + c];
                best.idx = e;
            }
        }
    return warp_argmax(best);
}

struct WeightParams {
    const float* trow;
    const float* drow;  // nullptr => weight = P (bonus draw / fallback)
    float inv_t, Mt, Rt, Md, Rd;
};

__device__ __forceinline__ float elem_weight(const WeightParams& w, float tv, float dv) {
    const float P = __fmul_rn(spec_exp(__fmaf_rn(tv, w.inv_t, -w.Mt)), w.Rt);
    if (w.drow == nullptr) return P;
    const float Q = __fmul_rn(spec_exp(__fmaf_rn(dv, w.inv_t, -w.Md)), w.Rd);
    return P > Q ? __fsub_rn(P, Q) : 0.0f;
}

// Sequential selection rule of the spec (first child whose running sum
// exceeds tau; fallback: last positive child, tau' = its weight).
__device__ int select_level(const float* w, int n, float tau, float* tau_out) {
    float acc = 0.0f;
    int last = -1;
    for (int i = 0; i < n; ++i) {
        const float nxt = __fadd_rn(acc, w[i]);
        if (w[i] > 0.0f) {
            last = i;
            if (nxt > tau) {
                *tau_out = __fsub_rn(tau, acc);
                return i;
            }
        }
        acc = nxt;
    }
    if (last >= 0) *tau_out = w[last];
    return last;
}

struct FinalSmem {
    float M[kAcceptMaxRows];
    float R[kAcceptMaxRows];
    int g[kAcceptMaxRows];
    float lane_w[kAcceptMaxTiles * 32];
    float tile_w[kAcceptMaxTiles];
    float elem_w[32];
    int elem_idx[32];
    float total;
    int r;
    int token;
};

// Weight pass over one row pair: lane / tile weights into shared memory.
__device__ void weight_pass(const WeightParams& w, int V, int ntiles, bool vec, FinalSmem& s) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int t = warp; t < ntiles; t += kWarps) {
        const bool full = (t + 1) * kTile <= V;
        LaneTile dt, dd;
        load_lane(w.trow, V, t, lane, vec, dt);
        if (w.drow) load_lane(w.drow, V, t, lane, vec, dd);
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int c = 0; c < 4; ++c)
                if (full || elem_valid(V, t, lane, i, c))
                    acc[c] = __fadd_rn(acc[c], elem_weight(w, dt.x[4 * i + c], w.drow ? dd.x[4 * i + c] : 0.0f));
        const float lw = lane_combine(acc);
        s.lane_w[t * 32 + lane] = lw;
        const float tw = warp_butterfly_sum(lw);
        if (lane == 0) s.tile_w[t] = tw;
    }
}

template <bool kGreedy>
__global__ void __launch_bounds__(kThreads) accept_kernel(AcceptParams p) {
    __shared__ FinalSmem s;
    __shared__ int s_last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.x / p.ctas_per_seq;
    const int j = blockIdx.x % p.ctas_per_seq;
    const int items = p.nrows * p.ntiles;
    const size_t V = (size_t)p.V;

    // ---- phase 1: tile statistics --------------------------------------
    const int item = j * kWarps + warp;
    if (item < items) {
        const int row = item / p.ntiles, t = item % p.ntiles;
        const float* rp = row <= p.k ? p.tgt + ((size_t)b * (p.k + 1) + row) * V
                                     : p.drf + ((size_t)b * p.k + (row - p.k - 1)) * V;
        const bool full = (t + 1) * kTile <= p.V;
        LaneTile d;
        load_lane(rp, p.V, t, lane, p.vec4, d);
        float2 part;
        if (kGreedy) {
            const ArgMax a = tile_argmax(d, p.V, t, lane, full);
            part = make_float2(a.v, __int_as_float(a.idx));
        } else {
            part = tile_stats(d, p.V, t, lane, full, p.inv_t);
        }
        if (lane == 0) p.part[((size_t)b * p.nrows + row) * p.ntiles + t] = part;
    }

    // ---- completion ticket (last CTA of the sequence finishes) ----------
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned ticket = atomicAdd(&p.counters[b], 1u);
        s_last = (ticket == (unsigned)(p.ctas_per_seq - 1));
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();

    const float2* part = p.part + (size_t)b * p.nrows * p.ntiles;

    // ---- phase 2a: row statistics --------------------------------------
    for (int row = warp; row < p.nrows; row += kWarps) {
        const float2* rpart = part + (size_t)row * p.ntiles;
        if (kGreedy) {
            ArgMax best{-INFINITY, -1};
            for (int t = lane; t < p.ntiles; t += 32) {
                const float2 v = __ldcg(rpart + t);
                best = argmax_combine(best, ArgMax{v.x, __float_as_int(v.y)});
            }
            best = warp_argmax(best);
            if (lane == 0) s.g[row] = best.idx < 0 ? 0 : best.idx;
        } else {
            float mt[kAcceptMaxTiles / 32], zt[kAcceptMaxTiles / 32];
            float M = -INFINITY;
#pragma unroll
            for (int q = 0; q < kAcceptMaxTiles / 32; ++q) {
                const int t = q * 32 + lane;
                float2 v = make_float2(-INFINITY, 0.0f);
                if (t < p.ntiles) v = __ldcg(rpart + t);
                mt[q] = v.x;
                zt[q] = v.y;
                M = fmaxf(M, v.x);
            }
            M = warp_max(M);
            float Z = 0.0f;
#pragma unroll
            for (int q = 0; q < kAcceptMaxTiles / 32; ++q) {
                if (q * 32 >= p.ntiles) break;
                const float e = spec_exp(__fsub_rn(mt[q], M));
                for (int l = 0; l < 32; ++l) {
                    if (q * 32 + l >= p.ntiles) break;
                    const float ze = __shfl_sync(0xffffffffu, zt[q], l);
                    const float ee = __shfl_sync(0xffffffffu, e, l);
                    Z = __fmaf_rn(ze, ee, Z);
                }
            }
            if (lane == 0) {
                s.M[row] = M;
                s.R[row] = __fdiv_rn(1.0f, Z);
            }
        }
    }
    __syncthreads();

    // ---- phase 2b: accept / reject ------------------------------------
    const uint32_t* tok = p.tok + (size_t)b * p.k;
    const float* u = p.u + (size_t)b * (p.k + 1);
    if (threadIdx.x == 0) {
        int r = p.k;
        for (int i = 0; i < p.k; ++i) {
            const uint32_t x = tok[i];
            if (x >= (uint32_t)p.V) {  // bad input on the device path
                atomicOr(p.err_flag, 1);
                r = i;
                break;
            }
            if (kGreedy) {
                if ((int)x != s.g[i]) { r = i; break; }
            } else {
                const float tv = p.tgt[((size_t)b * (p.k + 1) + i) * V + x];
                const float dv = p.drf[((size_t)b * p.k + i) * V + x];
                const float P = __fmul_rn(spec_exp(__fmaf_rn(tv, p.inv_t, -s.M[i])), s.R[i]);
                const float Q = __fmul_rn(spec_exp(__fmaf_rn(dv, p.inv_t, -s.M[p.k + 1 + i])), s.R[p.k + 1 + i]);
                if (!(__fmul_rn(u[i], Q) <= P)) { r = i; break; }
            }
        }
        s.r = r;
        if (kGreedy) s.token = s.g[r];
    }
    __syncthreads();

    // ---- phase 2c: residual / bonus draw (sampling only) ---------------
    if (!kGreedy) {
        const int r = s.r;
        WeightParams w;
        w.inv_t = p.inv_t;
        w.trow = p.tgt + ((size_t)b * (p.k + 1) + r) * V;
        w.Mt = s.M[r];
        w.Rt = s.R[r];
        w.drow = r < p.k ? p.drf + ((size_t)b * p.k + r) * V : nullptr;
        w.Md = r < p.k ? s.M[p.k + 1 + r] : 0.0f;
        w.Rd = r < p.k ? s.R[p.k + 1 + r] : 0.0f;
        for (int attempt = 0; attempt < 2; ++attempt) {
            weight_pass(w, p.V, p.ntiles, p.vec4, s);
            __syncthreads();
            if (threadIdx.x == 0) {
                float total = 0.0f;
                for (int t = 0; t < p.ntiles; ++t) total = __fadd_rn(total, s.tile_w[t]);
                s.total = total;
            }
            __syncthreads();
            if (s.total > 0.0f || w.drow == nullptr) break;
            w.drow = nullptr;  // residual mass vanished: draw from p of the row
            __syncthreads();
        }
        // tile and lane selection (thread 0), then the element level (warp 0)
        __shared__ int s_sel[2];
        __shared__ float s_tau;
        if (threadIdx.x == 0) {
            float tau1 = 0.0f, tau2 = 0.0f;
            const float tau = __fmul_rn(u[p.k], s.total);
            int ts = select_level(s.tile_w, p.ntiles, tau, &tau1);
            int ls = ts >= 0 ? select_level(&s.lane_w[ts * 32], 32, tau1, &tau2) : -1;
            s_sel[0] = ts;
            s_sel[1] = ls;
            s_tau = tau2;
        }
        __syncthreads();
        if (warp == 0) {
            const int ts = s_sel[0], ls = s_sel[1];
            if (ts >= 0 && ls >= 0) {
                const int i = lane >> 2, c = lane & 3;
                const int e = ts * kTile + 128 * i + 4 * ls + c;
                float wv = 0.0f;
                if (e < p.V) wv = elem_weight(w, __ldg(w.trow + e), w.drow ? __ldg(w.drow + e) : 0.0f);
                s.elem_w[lane] = wv;
                s.elem_idx[lane] = e;
            }
            __syncwarp();
            if (lane == 0) {
                int tokv = 0;
                if (ts >= 0 && ls >= 0) {
                    float tau3;
                    const int es = select_level(s.elem_w, 32, s_tau, &tau3);
                    tokv = es >= 0 ? s.elem_idx[es] : 0;
                }
                s.token = tokv;
            }
        }
        __syncthreads();
    }

    if (threadIdx.x == 0) {
        p.acc_len[b] = s.r;
        p.bonus[b] = (uint32_t)s.token;
        p.counters[b] = 0u;  // ready for the next launch
    }
}

}  // namespace

size_t accept_workspace_bytes(int B, int k, int V, bool greedy) {
    const int ntiles = (V + kTile - 1) / kTile;
    const int nrows = greedy ? k + 1 : 2 * k + 1;
    return (size_t)B * nrows * ntiles * sizeof(float2);
}

cudaError_t launch_accept(const AcceptParams& prm, bool greedy, cudaStream_t stream) {
    AcceptParams p = prm;
    p.ntiles = (p.V + kTile - 1) / kTile;
    p.nrows = greedy ? p.k + 1 : 2 * p.k + 1;
    p.ctas_per_seq = (p.nrows * p.ntiles + kWarps - 1) / kWarps;
    const dim3 grid((unsigned)(p.B * p.ctas_per_seq));
    if (greedy)
        accept_kernel<true><<<grid, kThreads, 0, stream>>>(p);
    else
        accept_kernel<false><<<grid, kThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace velo
