// tree_attn.cu -- tree-masked paged attention for the verify step on the
// sm_100a tensor cores.
//
// Semantics follow the reference's tree attention (src/kernels.metal:512-599
// paged_attention_tree, :672-732 the INT8 flash variant): every query row of
// tree node n attends to the sequence's cached tokens [0, ctx_len) through
// its 16-token page table, and to the tree nodes on its own root -> n path;
// scores are q.k / sqrt(head_dim), softmax over that key set, output the
// probability-weighted V.  INT8 pages carry one fp16 scale per token and
// head (value = q * scale).  GQA: query head hq reads KV head hq / (Hq/Hkv).
//
// One CTA = one (sequence, KV head, QT x 128 query rows) item, QT = 1 or 2
// query tiles.  Query rows are the (node, group head) pairs of the KV head,
// node-major.  Keys stream in tiles of 64 (4 pages), the tree nodes form a
// final tile with an ancestor mask.  With QT = 2 (more than 128 rows per KV
// head) both query tiles share every K/V tile: it is read from HBM, and for
// int8 pools converted, once.
//   warp 0     producer: TMA (f16 pools, 128-byte swizzle straight into the
//              operand tiles) or bulk copies of the raw int8 pages + scales
//   warp 1     one thread issues, per query tile, S = Q K^T (M=128, N=64)
//              into a double-buffered TMEM tile and O += P V (M=128, N=128,
//              V MN-major), in the order their inputs arrive
//   warp 2     TMEM allocation (per query tile S0, S1: 64 columns each; O: 128)
//   warps 4-11 softmax: S from TMEM, exp2 on the SFU, P (f16) to shared
//              memory for the PV MMA; O rescaled in TMEM only when the running
//              max grows by > 2^8.  QT = 1: two threads per query row (32 keys
//              each); QT = 2: warps 4-7 own query tile 0 and warps 8-11 tile 1,
//              one thread per row (all 64 keys)
//   warps 12-15 (int8 pools) int8 -> f16 conversion of every K/V tile into
//              the swizzled operand layout, and the tree tile from the node K/V
//              (f16 pools: the producer loads the tree tile with a 3-D TMA)
#include <cuda_fp16.h>

#include <cstdlib>
#include <mutex>

#include "common/sm100.cuh"
#include "common/spec_math.cuh"  // max3
#include "kernels/q4gemm.h"  // make_tmap_f16_2d
#include "kernels/tree_attn.h"

namespace velo {
namespace {

using namespace sm100;

constexpr int D = kAttnHeadDim;        // 128
constexpr int TK = 64;                 // keys per tile
constexpr int BMQ = 128;               // query rows per CTA
constexpr int kThreads = 512;
constexpr int Q_BYTES = BMQ * D * 2;           // 32 KiB (two 64-wide halves)
constexpr int KV_HALF = TK * 64 * 2;           // 8 KiB: 64 keys x 64 dims
constexpr int KV_STAGE = 4 * KV_HALF;          // K halves + V halves: 32 KiB
constexpr int P_BYTES = BMQ * TK * 2;          // 16 KiB
constexpr int RAW_KV = TK * D;                 // int8 tile of K (or V): 8 KiB
constexpr int RAW_STAGE = 2 * RAW_KV + 2 * TK * 2;  // K, V, K scales, V scales
constexpr float kRescaleLog2 = 8.0f;           // lazy O rescale threshold

constexpr int kErrPage = 0x5101, kErrWait = 0x5102;

template <bool INT8, int QT>
struct AttnCfg {
    static_assert(QT == 1 || QT == 2, "one or two query tiles per CTA");
    // f16 operand ring (cached tokens + tree tile) and raw int8 ring
    static constexpr int KS = QT == 1 ? (INT8 ? 3 : 5) : (INT8 ? 2 : 4);
    static constexpr int RS = INT8 ? 3 : 0;
    // P buffers per query tile: two let the softmax write P_j while PV_{j-1}
    // still reads P_{j-1}; with two query tiles the budget holds one each
    static constexpr int PB = QT == 1 ? 2 : 1;
    static constexpr int kSoftmaxPerQt = QT == 1 ? 256 : 128;  // softmax threads per tile
    static constexpr uint32_t kTmemCols = QT * 256;
    // Q, the ring, P, raw ring, scales, alignment, barriers, row exchange (QT = 1)
    static constexpr size_t kSmem = (size_t)QT * Q_BYTES + (size_t)KS * KV_STAGE +
                                    (size_t)QT * PB * P_BYTES + (size_t)RS * RAW_STAGE +
                                    (INT8 ? (size_t)KS * 2 * TK * 4 : 0) + 1024 + 512 +
                                    (QT == 1 ? 2 * BMQ * 4 : 0);
    static_assert(kSmem <= 232448, "shared memory budget (227 KiB per block)");
};

// swizzled byte offset of 16-byte chunk c of row r in a 128-byte-row tile
__device__ __forceinline__ uint32_t sw128(int r, int c) {
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// Named barrier of the two softmax warps that share TMEM lane quadrant q.
__device__ __forceinline__ void pair_sync(int q) {
    asm volatile("bar.sync %0, 64;" ::"r"(1 + q) : "memory");
}

// Four int8 (little-endian in w) -> f16 pairs (b0,b1), (b2,b3), exactly:
// flipping the sign bit gives u = x + 128, 0x6400 | u is 1024 + u in f16, and
// subtracting 1152 leaves x.
__device__ __forceinline__ void i8x4_to_f16(uint32_t w, uint32_t& lo, uint32_t& hi) {
    const uint32_t u = w ^ 0x80808080u;
    const uint32_t r01 = __byte_perm(u, 0x64646464u, 0x5140);
    const uint32_t r23 = __byte_perm(u, 0x64646464u, 0x5342);
    const __half2 k = __half2half2(__ushort_as_half(0x6480));  // 1152
    const __half2 a = __hsub2(*reinterpret_cast<const __half2*>(&r01), k);
    const __half2 c = __hsub2(*reinterpret_cast<const __half2*>(&r23), k);
    lo = *reinterpret_cast<const uint32_t*>(&a);
    hi = *reinterpret_cast<const uint32_t*>(&c);
}

// Maximum of 32 raw scores of a query row.  Int8 pages: each score is first
// multiplied by its key's scale, in place.  kMasked: scores of keys without
// a bit in kmask become -inf (the tree tile and a ragged last tile only).
template <bool INT8, bool kMasked>
__device__ __forceinline__ float raw_max32(uint32_t (&x32)[32], uint32_t kmask, const float* ks) {
    if constexpr (INT8) {
#pragma unroll
        for (int t4 = 0; t4 < 8; ++t4) {
            const float4 k4 = *reinterpret_cast<const float4*>(ks + 4 * t4);  // broadcast
            x32[4 * t4 + 0] = __float_as_uint(__uint_as_float(x32[4 * t4 + 0]) * k4.x);
            x32[4 * t4 + 1] = __float_as_uint(__uint_as_float(x32[4 * t4 + 1]) * k4.y);
            x32[4 * t4 + 2] = __float_as_uint(__uint_as_float(x32[4 * t4 + 2]) * k4.z);
            x32[4 * t4 + 3] = __float_as_uint(__uint_as_float(x32[4 * t4 + 3]) * k4.w);
        }
    }
    if constexpr (kMasked) {
#pragma unroll
        for (int t = 0; t < 32; ++t)
            if (!((kmask >> t) & 1u)) x32[t] = __float_as_uint(-INFINITY);
    }
    // 32 -> 11 -> 4 -> 1 with three-input maxima (exact in any order)
    float m1[11];
#pragma unroll
    for (int i = 0; i < 10; ++i)
        m1[i] = max3(__uint_as_float(x32[3 * i]), __uint_as_float(x32[3 * i + 1]), __uint_as_float(x32[3 * i + 2]));
    m1[10] = fmaxf(__uint_as_float(x32[30]), __uint_as_float(x32[31]));
    return fmaxf(max3(max3(m1[0], m1[1], m1[2]), max3(m1[3], m1[4], m1[5]), max3(m1[6], m1[7], m1[8])),
                 fmaxf(m1[9], m1[10]));
}

// p = 2^(x * sl2 - ms) of 32 keys (one packed FMA per pair), times the V
// scale for int8 pages, as f16 into chunks c0 .. c0+3 of P row r; returns the
// pairwise sums of the unscaled p.
template <bool INT8>
__device__ __forceinline__ float2 exp_pack_store(const uint32_t (&x32)[32], float sl2, float ms,
                                                 const float* vs, uint8_t* pbuf, int r, int c0) {
    float2 acc = make_float2(0.0f, 0.0f);
    const float2 s2 = make_float2(sl2, sl2), nm = make_float2(-ms, -ms);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int t = c * 8 + 2 * e;
            const float2 y = __ffma2_rn(make_float2(__uint_as_float(x32[t]), __uint_as_float(x32[t + 1])), s2, nm);
            float2 pp = make_float2(ex2_approx(y.x), ex2_approx(y.y));  // masked (-inf) -> 0
            acc = __fadd2_rn(acc, pp);
            if constexpr (INT8) pp = __fmul2_rn(pp, *reinterpret_cast<const float2*>(vs + t));
            __half2 hp = __floats2half2_rn(pp.x, pp.y);
            w[e] = *reinterpret_cast<uint32_t*>(&hp);
        }
        *reinterpret_cast<uint4*>(pbuf + sw128(r, c0 + c)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    return acc;
}

// Softmax of a CTA with two query tiles: warps 4-7 own tile 0, warps 8-11
// tile 1, one thread per query row over all 64 keys of every K tile (no
// exchange between threads).  Each tile has one P buffer, so P_j is written
// only after PV_{j-1} completed.  Returns early (the CTA then exits) when a
// wait runs out or another role aborted.
template <bool INT8, int KS>
__device__ __forceinline__ void softmax_rows(const TreeAttnArgs& a, int warp, int lane, int mt, int b,
                                             int h, int L, int T_pre, int T, int G, int rows_total,
                                             uint32_t tmem, uint64_t* qbars, uint8_t* sp,
                                             const float* sscale, uint64_t* kv_full,
                                             volatile int* abort_flag) {
    const int qt = (warp - 4) >> 2, q = warp & 3;
    const int r = q * 32 + lane;                       // TMEM lane = query row of tile qt
    const int row = mt * (2 * BMQ) + qt * BMQ + r;
    const bool row_ok = row < rows_total;
    const int node = row_ok ? row / G : 0;
    const uint64_t anc = row_ok ? a.anc[(size_t)b * a.N + node] : 0ull;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const uint32_t tq = tmem + qt * 256;               // S0, S1, O of tile qt
    uint64_t* qb = qbars + qt * 8;                     // s_full, s_free, p_full, pv_done, o_full
    uint8_t* pbuf = sp + qt * P_BYTES;
    if (!__any_sync(0xffffffffu, row_ok)) {
        // no query row of this warp exists: its P rows stay zero and it only
        // keeps the barrier counts (arriving on P_j after PV_{j-1} completed,
        // as the other warps of its tile do)
#pragma unroll
        for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(pbuf + sw128(r, c)) = make_uint4(0, 0, 0, 0);
        fence_async_smem();
        for (int j = 0; j < T; ++j) {
            const int sb = j & 1;
            bool got = mbar_wait(&qb[sb], (j >> 1) & 1, a.err, kErrWait, abort_flag, 32);
            if (!__all_sync(0xffffffffu, got)) return;
            mbar_arrive(&qb[2 + sb]);
            if (j > 0) {
                got = mbar_wait(&qb[6], (j - 1) & 1, a.err, kErrWait, abort_flag, 32);
                if (!__all_sync(0xffffffffu, got)) return;
            }
            mbar_arrive(&qb[4]);
        }
        return;
    }
    float m = -INFINITY, l = 0.0f;
    for (int j = 0; j < T; ++j) {
        const int sb = j & 1, s = j % KS;
        bool got = mbar_wait(&qb[sb], (j >> 1) & 1, a.err, kErrWait, abort_flag);
        if (!__all_sync(0xffffffffu, got)) return;
        tc_fence_after();
        uint32_t xa[32], xb[32];
        tmem_ld_32x32b_x32(tq + lane_base + sb * TK, xa);
        tmem_ld_32x32b_x32(tq + lane_base + sb * TK + 32, xb);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(&qb[2 + sb]);
        const float* ks = sscale + s * 2 * TK;
        if constexpr (INT8) {
            // scales of this stage were written by the converter warps
            got = mbar_wait(&kv_full[s], (j / KS) & 1, a.err, kErrWait, abort_flag);
            if (!__all_sync(0xffffffffu, got)) return;
        }
        // maximum of the row's raw scores (scale_log2 > 0 commutes with max):
        // full tiles of cached tokens need no mask; the tree tile keeps the
        // node's ancestors, a ragged last tile the tokens below ctx_len
        float mx;
        if (j < T_pre && L - j * TK >= TK) {
            mx = fmaxf(raw_max32<INT8, false>(xa, 0u, ks), raw_max32<INT8, false>(xb, 0u, ks + 32));
        } else {
            uint64_t kmask;
            if (j == T_pre) {
                kmask = anc;
            } else {
                const int nvalid = L - j * TK;
                kmask = nvalid <= 0 ? 0ull : (1ull << nvalid) - 1ull;  // nvalid < 64 here
            }
            mx = fmaxf(raw_max32<INT8, true>(xa, (uint32_t)kmask, ks),
                       raw_max32<INT8, true>(xb, (uint32_t)(kmask >> 32), ks + 32));
        }
        mx *= a.scale_log2;  // the scaled maximum, exactly (rounding is monotonic)
        // P_j replaces P_{j-1} and O may be rescaled: PV_{j-1} must be done.
        // Its phase is the only one in doubt: S_j was issued after PV_{j-2}
        // (so phase j-2 is complete) and PV_j needs this tile's P (so phase j
        // is not), hence a parity wait is exact here.
        if (j > 0) {
            got = mbar_wait(&qb[6], (j - 1) & 1, a.err, kErrWait, abort_flag);
            if (!__all_sync(0xffffffffu, got)) return;
            tc_fence_after();
        }
        // lazy rescale, decided per warp so the TMEM accesses stay convergent
        if (__any_sync(0xffffffffu, mx > m + kRescaleLog2)) {
            const float m_new = fmaxf(m, mx);
            const float f = m == -INFINITY ? 0.0f : ex2_approx(m - m_new);
            l *= f;
            if (j > 0) {
#pragma unroll 1
                for (int c = 0; c < 8; ++c) {  // 16 columns at a time: xa, xb stay in registers
                    uint32_t o[16];
                    const uint32_t oc = tq + 128 + lane_base + c * 16;
                    tmem_ld_32x32b_x16(oc, o);
                    tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
                    tmem_st_32x32b_x16(oc, o);
                }
                tmem_st_wait();
            }
            m = m_new;
        }
        const float ms = m == -INFINITY ? 0.0f : m;  // all keys masked so far: p = 0
        const float* vs = ks + TK;
        const float2 sa = exp_pack_store<INT8>(xa, a.scale_log2, ms, vs, pbuf, r, 0);
        const float2 sb2 = exp_pack_store<INT8>(xb, a.scale_log2, ms, vs + 32, pbuf, r, 4);
        l += (sa.x + sa.y) + (sb2.x + sb2.y);
        fence_async_smem();
        tc_fence_before();
        mbar_arrive(&qb[4]);
    }
    // epilogue: O / l after the last PV
    {
        const bool ok = mbar_wait(&qb[7], 0, a.err, kErrWait, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) return;
    }
    tc_fence_after();
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
    const int g = row_ok ? row % G : 0;
    const size_t obase = (((size_t)b * a.N + node) * a.Hq + h * G + g) * D;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        const int col = c * 32;
        tmem_ld_32x32b_x32(tq + 128 + lane_base + col, o);
        tmem_ld_wait();
        if (!row_ok) continue;
        if (a.out_f16) {
            __half* dst = static_cast<__half*>(a.out) + obase + col;
#pragma unroll
            for (int qq = 0; qq < 4; ++qq) {
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    __half2 hv = __floats2half2_rn(__uint_as_float(o[qq * 8 + 2 * e]) * inv,
                                                   __uint_as_float(o[qq * 8 + 2 * e + 1]) * inv);
                    w[e] = *reinterpret_cast<uint32_t*>(&hv);
                }
                reinterpret_cast<uint4*>(dst)[qq] = make_uint4(w[0], w[1], w[2], w[3]);
            }
        } else {
            float* dst = static_cast<float*>(a.out) + obase + col;
#pragma unroll
            for (int qq = 0; qq < 8; ++qq)
                reinterpret_cast<float4*>(dst)[qq] =
                    make_float4(__uint_as_float(o[4 * qq]) * inv, __uint_as_float(o[4 * qq + 1]) * inv,
                                __uint_as_float(o[4 * qq + 2]) * inv, __uint_as_float(o[4 * qq + 3]) * inv);
        }
    }
}

__global__ void tree_ancestors_kernel(const int32_t* __restrict__ parents, int B, int N,
                                      uint64_t* __restrict__ anc, int* err) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * N) return;
    const int b = i / N, n = i % N;
    uint64_t m = 0;
    int c = n;
    for (int step = 0; step <= N && c >= 0; ++step) {
        m |= 1ull << c;
        const int p = parents[b * N + c];
        if (p >= c || p < -1) {  // parents must precede their children
            atomicCAS(err, 0, kErrPage + 16);
            break;
        }
        c = p;
    }
    anc[i] = m;
}

template <bool INT8, int QT>
__global__ void __launch_bounds__(kThreads, 1)
    tree_attn_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                     const __grid_constant__ CUtensorMap tnk, const __grid_constant__ CUtensorMap tnv,
                     const TreeAttnArgs a) {
    using C = AttnCfg<INT8, QT>;
    constexpr int KS = C::KS, RS = C::RS, PB = C::PB;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sq = base;                                // Q: per tile 2 halves x 16 KiB
    uint8_t* skv = sq + QT * Q_BYTES;                  // KS x (K0 K1 V0 V1) 8 KiB each
    uint8_t* sp = skv + KS * KV_STAGE;                 // P: [QT][PB] x 16 KiB
    uint8_t* sraw = sp + QT * PB * P_BYTES;            // RS x raw int8 stage
    float* sscale = reinterpret_cast<float*>(sraw + RS * RAW_STAGE);  // KS x (ks[64], vs[64])
    uint64_t* bars = reinterpret_cast<uint64_t*>(sscale + (INT8 ? KS * 2 * TK : 0));
    uint64_t* kv_full = bars;
    uint64_t* kv_empty = kv_full + KS;
    uint64_t* raw_full = kv_empty + KS;                // RS entries (int8)
    uint64_t* raw_empty = raw_full + (RS ? RS : 1);
    // per query tile qt, at qt * 8: s_full[2], s_free[2], p_full[2] (PB used),
    // pv_done (phase j <-> PV_j done), o_full (the last PV done)
    uint64_t* qbars = raw_empty + (RS ? RS : 1);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(qbars + QT * 8);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    float* sxch = reinterpret_cast<float*>(tmem_slot + 4);  // [2][128] row exchange (QT = 1)

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = a.Hq / a.Hkv;
    const int rows_total = a.N * G;
    const int MT = (rows_total + QT * BMQ - 1) / (QT * BMQ);
    const int mt = blockIdx.x % MT;
    const int h = (blockIdx.x / MT) % a.Hkv;
    const int b = blockIdx.x / (MT * a.Hkv);
    const int L = a.ctx_len[b] > 0 ? a.ctx_len[b] : 0;
    const int T_pre = (L + TK - 1) / TK;
    const int T = T_pre + 1;  // + the tree tile

    if (threadIdx.x == 0) {
        for (int s = 0; s < KS; ++s) {
            mbar_init(&kv_full[s], INT8 ? 128 : 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int s = 0; s < RS; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], 128);
        }
        for (int qt = 0; qt < QT; ++qt) {
            uint64_t* qb = qbars + qt * 8;
            for (int i = 0; i < 2; ++i) {
                mbar_init(&qb[i], 1);                      // s_full
                mbar_init(&qb[2 + i], C::kSoftmaxPerQt);   // s_free
                mbar_init(&qb[4 + i], C::kSoftmaxPerQt);   // p_full
            }
            mbar_init(&qb[6], 1);
            mbar_init(&qb[7], 1);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 2) {
        tmem_alloc(tmem_slot, C::kTmemCols);
        tmem_relinquish();
    }
    // Q tiles (all threads): row r = node-major (node, group head), 16 chunks
    for (int idx = threadIdx.x; idx < QT * BMQ * 16; idx += kThreads) {
        const int rr = idx >> 4, c = idx & 15;
        const int qt = rr / BMQ, r = rr % BMQ;
        const int row = mt * (QT * BMQ) + rr;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (row < rows_total) {
            const int node = row / G, g = row % G;
            const __half* src = a.q + (((size_t)b * a.N + node) * a.Hq + h * G + g) * D + c * 8;
            v = *reinterpret_cast<const uint4*>(src);
        }
        *reinterpret_cast<uint4*>(sq + qt * Q_BYTES + (c >> 3) * (Q_BYTES / 2) + sw128(r, c & 7)) = v;
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;  // query tile qt: S0, S1, O at qt * 256 + 0, 64, 128

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const uint32_t* pt = a.page_table + (size_t)b * a.max_pages;
            // page ids of the next tile are read one iteration early, so the
            // global-memory latency hides behind the wait for a free slot
            uint32_t pg_next[TK / kKvPage];
            auto fetch = [&](int j, uint32_t (&dst)[TK / kKvPage]) {
#pragma unroll
                for (int i = 0; i < TK / kKvPage; ++i) {
                    const int pi = j * (TK / kKvPage) + i;
                    dst[i] = (j < T_pre && pi < a.max_pages) ? pt[pi] : 0u;
                }
            };
            fetch(0, pg_next);
            for (int j = 0; j < (INT8 ? T_pre : T); ++j) {
                uint32_t pg_cur[TK / kKvPage];
#pragma unroll
                for (int i = 0; i < TK / kKvPage; ++i) pg_cur[i] = pg_next[i];
                fetch(j + 1, pg_next);
                if constexpr (!INT8) {
                    const int s = j % KS;
                    if (!mbar_wait(&kv_empty[s], ((j / KS) & 1) ^ 1, a.err, kErrWait, abort_flag, 64))
                        goto done;
                    if (j == T_pre) {
                        // tree tile: node K/V rows b*N .. b*N+63 of KV head h (3-D
                        // maps [B*N][Hkv][128]); rows past this sequence's nodes are
                        // masked, rows past the tensor read as zero
                        mbar_arrive_expect_tx(&kv_full[s], KV_STAGE);
                        uint8_t* st = skv + s * KV_STAGE;
                        for (int dh = 0; dh < 2; ++dh) {
                            tma_load_3d(st + dh * KV_HALF, &tnk, &kv_full[s], dh * 64, h, b * a.N);
                            tma_load_3d(st + 2 * KV_HALF + dh * KV_HALF, &tnv, &kv_full[s], dh * 64, h, b * a.N);
                        }
                        continue;
                    }
                    mbar_arrive_expect_tx(&kv_full[s], KV_STAGE);
                    uint8_t* st = skv + s * KV_STAGE;
                    for (int i = 0; i < TK / kKvPage; ++i) {
                        uint32_t pg = pg_cur[i];
                        if (pg >= (uint32_t)a.pool_pages) {
                            atomicCAS(a.err, 0, kErrPage);
                            pg = 0;
                        }
                        const int row = (int)((pg * a.Hkv + h) * kKvPage);
                        for (int dh = 0; dh < 2; ++dh) {
                            tma_load_2d(st + dh * KV_HALF + i * 2048, &tmk, &kv_full[s], dh * 64, row);
                            tma_load_2d(st + 2 * KV_HALF + dh * KV_HALF + i * 2048, &tmv, &kv_full[s],
                                        dh * 64, row);
                        }
                    }
                } else {
                    const int r = j % RS;
                    if (!mbar_wait(&raw_empty[r], ((j / RS) & 1) ^ 1, a.err, kErrWait, abort_flag, 64))
                        goto done;
                    mbar_arrive_expect_tx(&raw_full[r], RAW_STAGE);
                    uint8_t* st = sraw + r * RAW_STAGE;
                    for (int i = 0; i < TK / kKvPage; ++i) {
                        uint32_t pg = pg_cur[i];
                        if (pg >= (uint32_t)a.pool_pages) {
                            atomicCAS(a.err, 0, kErrPage);
                            pg = 0;
                        }
                        const size_t blk = (size_t)pg * a.Hkv + h;  // (page, head) block
                        bulk_load(st + i * 2048, static_cast<const int8_t*>(a.k_pool) + blk * 2048, 2048,
                                  &raw_full[r]);
                        bulk_load(st + RAW_KV + i * 2048, static_cast<const int8_t*>(a.v_pool) + blk * 2048,
                                  2048, &raw_full[r]);
                        bulk_load(st + 2 * RAW_KV + i * 32, a.k_scale + blk * kKvPage, 32, &raw_full[r]);
                        bulk_load(st + 2 * RAW_KV + TK * 2 + i * 32, a.v_scale + blk * kKvPage, 32,
                                  &raw_full[r]);
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issue
        if (lane == 0) {
            const uint32_t id_s = idesc_f16_f32(BMQ, TK);
            const uint32_t id_pv = idesc_f16_f32(BMQ, D, /*b_mn_major=*/true);
            // Per query tile, issue S_j and PV_j in whichever order their
            // inputs arrive: S_j needs its K tile and a free S buffer, PV_j the
            // softmax's P_j.  S_j also waits until PV_{j-2} is issued, so that
            // when S_j completes every PV before j-1 has completed (the softmax
            // relies on that to wait for PV_{j-1} by parity alone).  A K/V
            // stage is released after the last query tile's PV of it.
            int ns[QT], npv[QT];
#pragma unroll
            for (int qt = 0; qt < QT; ++qt) ns[qt] = npv[qt] = 0;
            const uint64_t t0 = global_ns();
            uint32_t spins = 0;
            for (;;) {
                bool progressed = false, all_done = true;
#pragma unroll
                for (int qt = 0; qt < QT; ++qt) {
                    uint64_t* qb = qbars + qt * 8;
                    const uint32_t tq = tmem + qt * 256;
                    if (ns[qt] < T && npv[qt] >= ns[qt] - 1) {
                        const int j = ns[qt], s = j % KS, sb = j & 1;
                        if (mbar_test_wait(smem_u32(&kv_full[s]), (j / KS) & 1) &&
                            mbar_test_wait(smem_u32(&qb[2 + sb]), ((j >> 1) & 1) ^ 1)) {
                            tc_fence_after();
                            const uint32_t q_addr = smem_u32(sq + qt * Q_BYTES);
                            const uint32_t k_addr = smem_u32(skv + s * KV_STAGE);
#pragma unroll
                            for (int k = 0; k < D / 16; ++k) {
                                const uint64_t ad = desc_kmajor_sw128(q_addr + (k >> 2) * (Q_BYTES / 2)) + (k & 3) * 2;
                                const uint64_t bd = desc_kmajor_sw128(k_addr + (k >> 2) * KV_HALF) + (k & 3) * 2;
                                mma_f16_ss(tq + sb * TK, ad, bd, id_s, k > 0);
                            }
                            mma_commit(&qb[sb]);
                            ++ns[qt];
                            progressed = true;
                        }
                    }
                    if (npv[qt] < ns[qt]) {
                        const int jj = npv[qt], sv = jj % KS;
                        const int pb = PB == 2 ? (jj & 1) : 0;
                        const uint32_t par = PB == 2 ? ((jj >> 1) & 1) : (jj & 1);
                        if (mbar_test_wait(smem_u32(&qb[4 + pb]), par)) {
                            tc_fence_after();
                            const uint32_t p_addr = smem_u32(sp + (qt * PB + pb) * P_BYTES);
                            const uint32_t v_addr = smem_u32(skv + sv * KV_STAGE + 2 * KV_HALF);
#pragma unroll
                            for (int kk = 0; kk < TK / 16; ++kk) {
                                const uint64_t ad = desc_kmajor_sw128(p_addr) + kk * 2;
                                const uint64_t bd = desc_mnmajor_sw128(v_addr + kk * 2048, KV_HALF);
                                mma_f16_ss(tq + 128, ad, bd, id_pv, (jj | kk) != 0);
                            }
                            bool last_of_stage = true;
#pragma unroll
                            for (int o = 0; o < QT; ++o)
                                if (o != qt && npv[o] <= jj) last_of_stage = false;
                            if (last_of_stage) mma_commit(&kv_empty[sv]);
                            mma_commit(&qb[6]);
                            if (jj == T - 1) mma_commit(&qb[7]);
                            ++npv[qt];
                            progressed = true;
                        }
                    }
                    if (npv[qt] < T) all_done = false;
                }
                if (all_done) break;
                if (!progressed && (++spins & 255u) == 0) {
                    if (*abort_flag) goto done;
                    if (global_ns() - t0 > kWaitLimitNs * 8) {  // a whole item, not one wait
                        atomicCAS(a.err, 0, kErrWait);
                        *abort_flag = 1;
                        goto done;
                    }
                }
            }
        }
    } else if (warp >= 4 && warp < 12) {
        // ------------------------------------------------------------ softmax
        if constexpr (QT == 1) {
            uint64_t* s_full = qbars;
            uint64_t* s_free = qbars + 2;
            uint64_t* p_full = qbars + 4;
            uint64_t* pv_done = qbars + 6;
            uint64_t* o_full = qbars + 7;
            const uint32_t tmem_o = tmem + 128;
            // warps w and w + 4 share TMEM lane quadrant q = w % 4 (query rows
            // 32q..32q+31); half ch = 0 takes keys 0..31 and O columns 0..63, ch = 1
            // keys 32..63 and O columns 64..127.  Row maxima and sums meet in
            // shared memory behind a named barrier of the warp pair.
            const int q = warp & 3, ch = (warp - 4) >> 2;
            const int r = q * 32 + lane;               // TMEM lane = query row
            const int row = mt * BMQ + r;
            const bool row_ok = row < rows_total;
            const int node = row_ok ? row / G : 0;
            const uint64_t anc = row_ok ? a.anc[(size_t)b * a.N + node] : 0ull;
            const uint32_t lane_base = (uint32_t)(q * 32) << 16;
            float* xch = sxch + ch * BMQ;              // this half's row values
            const float* xoth = sxch + (ch ^ 1) * BMQ; // the partner's
            const int kbase = ch * 32;
            float m = -INFINITY, l = 0.0f;             // l: this half's partial sum
            if (!__any_sync(0xffffffffu, row_ok)) {
                // no query row of this warp exists (few nodes x heads, e.g. 16 rows
                // of 128): its P rows stay zero and it only keeps the barrier
                // counts, leaving the SFU and issue slots to the warps with rows
#pragma unroll
                for (int pb = 0; pb < 2; ++pb)
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        *reinterpret_cast<uint4*>(sp + pb * P_BYTES + sw128(r, ch * 4 + c)) = make_uint4(0, 0, 0, 0);
                fence_async_smem();
                for (int j = 0; j < T; ++j) {
                    const int sb = j & 1;
                    const bool got = mbar_wait(&s_full[sb], (j >> 1) & 1, a.err, kErrWait, abort_flag, 32);
                    if (!__all_sync(0xffffffffu, got)) goto done;
                    mbar_arrive(&s_free[sb]);
                    mbar_arrive(&p_full[sb]);
                }
                goto done;
            }
            for (int j = 0; j < T; ++j) {
                const int sb = j & 1, s = j % KS;
                const bool got = mbar_wait(&s_full[sb], (j >> 1) & 1, a.err, kErrWait, abort_flag);
                if (!__all_sync(0xffffffffu, got)) goto done;
                tc_fence_after();
                uint32_t x32[32];
                tmem_ld_32x32b_x32(tmem + lane_base + sb * TK + kbase, x32);
                tmem_ld_wait();
                tc_fence_before();
                mbar_arrive(&s_free[sb]);
                const bool tree = j == T_pre;
                const float* ks = sscale + s * 2 * TK + kbase;
                if constexpr (INT8) {
                    // scales of this stage were written by the converter warps
                    const bool ok = mbar_wait(&kv_full[s], (j / KS) & 1, a.err, kErrWait, abort_flag);
                    if (!__all_sync(0xffffffffu, ok)) goto done;
                }
                // this thread's 32 keys as a bit mask: the node's ancestors in the
                // tree tile, the cached tokens below ctx_len otherwise
                uint32_t kmask;
                if (tree) {
                    kmask = (uint32_t)(anc >> kbase);
                } else {
                    const int nvalid = L - (j * TK + kbase);
                    kmask = nvalid >= 32 ? 0xffffffffu : nvalid <= 0 ? 0u : (1u << nvalid) - 1u;
                }
                // scaled scores (log2 domain) overwrite the raw ones in place
                float* x = reinterpret_cast<float*>(x32);
                float pm[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                for (int t = 0; t < 32; ++t) {
                    float v = x[t] * a.scale_log2;
                    if constexpr (INT8) v *= ks[t];
                    v = ((kmask >> t) & 1u) ? v : -INFINITY;
                    x[t] = v;
                    pm[t & 3] = fmaxf(pm[t & 3], v);
                }
                float mx = fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3]));
                xch[r] = mx;
                pair_sync(q);
                mx = fmaxf(mx, xoth[r]);
                // lazy rescale, decided per warp (identically in both warps of the
                // pair) so the TMEM accesses stay convergent
                if (__any_sync(0xffffffffu, mx > m + kRescaleLog2)) {
                    const float m_new = fmaxf(m, mx);
                    const float f = m == -INFINITY ? 0.0f : ex2_approx(m - m_new);
                    l *= f;
                    if (j > 0) {
                        // O holds PV_0..PV_{j-1}; wait for PV_{j-1}.  Its phase is the
                        // only one in doubt: S_j was issued after PV_{j-2} (so phase
                        // j-2 is complete) and PV_j needs this tile's P (so phase j
                        // is not), hence a parity wait is exact here.
                        const bool ok = mbar_wait(pv_done, (j - 1) & 1, a.err, kErrWait, abort_flag);
                        if (!__all_sync(0xffffffffu, ok)) goto done;
                        tc_fence_after();
#pragma unroll 1
                        for (int c = 0; c < 2; ++c) {
                            uint32_t o[32];
                            const uint32_t oc = tmem_o + lane_base + ch * 64 + c * 32;
                            tmem_ld_32x32b_x32(oc, o);
                            tmem_ld_wait();
#pragma unroll
                            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
                            tmem_st_32x32b_x32(oc, o);
                        }
                        tmem_st_wait();
                    }
                    m = m_new;
                }
                // P (times the V scale for int8 pages) -> f16, this half of row r
                uint8_t* prow = sp + sb * P_BYTES;
                const float* vs = ks + TK;
                const float ms = m == -INFINITY ? 0.0f : m;  // all keys masked so far: p = 0
                float ls[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t w[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int t = c * 8 + 2 * e;
                        float p0 = ex2_approx(x[t] - ms);      // masked (-inf) -> 0
                        float p1 = ex2_approx(x[t + 1] - ms);
                        ls[e] += p0 + p1;
                        if constexpr (INT8) {
                            p0 *= vs[t];
                            p1 *= vs[t + 1];
                        }
                        __half2 hp = __floats2half2_rn(p0, p1);
                        w[e] = *reinterpret_cast<uint32_t*>(&hp);
                    }
                    *reinterpret_cast<uint4*>(prow + sw128(r, ch * 4 + c)) = make_uint4(w[0], w[1], w[2], w[3]);
                }
                l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
                fence_async_smem();
                tc_fence_before();
                mbar_arrive(&p_full[sb]);
            }
            // epilogue: O / (both halves' sums) after the last PV
            {
                const bool ok = mbar_wait(o_full, 0, a.err, kErrWait, abort_flag);
                if (!__all_sync(0xffffffffu, ok)) goto done;
            }
            tc_fence_after();
            pair_sync(q);  // the partner finished reading xch for the last tile
            xch[r] = l;
            pair_sync(q);
            {
                const float lt = l + xoth[r];
                const float inv = lt > 0.0f ? 1.0f / lt : 0.0f;
                const int g = row_ok ? row % G : 0;
                const size_t obase = (((size_t)b * a.N + node) * a.Hq + h * G + g) * D;
#pragma unroll 1
                for (int c = 0; c < 2; ++c) {
                    uint32_t o[32];
                    const int col = ch * 64 + c * 32;
                    tmem_ld_32x32b_x32(tmem_o + lane_base + col, o);
                    tmem_ld_wait();
                    if (!row_ok) continue;
                    if (a.out_f16) {
                        __half* dst = static_cast<__half*>(a.out) + obase + col;
#pragma unroll
                        for (int qq = 0; qq < 4; ++qq) {
                            uint32_t w[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                __half2 hv = __floats2half2_rn(__uint_as_float(o[qq * 8 + 2 * e]) * inv,
                                                               __uint_as_float(o[qq * 8 + 2 * e + 1]) * inv);
                                w[e] = *reinterpret_cast<uint32_t*>(&hv);
                            }
                            reinterpret_cast<uint4*>(dst)[qq] = make_uint4(w[0], w[1], w[2], w[3]);
                        }
                    } else {
                        float* dst = static_cast<float*>(a.out) + obase + col;
#pragma unroll
                        for (int qq = 0; qq < 8; ++qq)
                            reinterpret_cast<float4*>(dst)[qq] =
                                make_float4(__uint_as_float(o[4 * qq]) * inv, __uint_as_float(o[4 * qq + 1]) * inv,
                                            __uint_as_float(o[4 * qq + 2]) * inv, __uint_as_float(o[4 * qq + 3]) * inv);
                    }
                }
            }
        } else {
            softmax_rows<INT8, KS>(a, warp, lane, mt, b, h, L, T_pre, T, G, rows_total, tmem, qbars, sp,
                                   sscale, kv_full, abort_flag);
        }
    } else if (warp >= 12) {
        // ------------------------------------------------------------ converters
        // int8 pools only: every tile of the ring (the cached tokens converted
        // from the raw stage, the tree tile from the node K/V rows)
        if constexpr (INT8) {
            const int t = threadIdx.x - 384;    // 0..127
            const int kr = t >> 1, hh = t & 1;  // key row, 64-dim half
            for (int j = 0; j < T; ++j) {
                const int s = j % KS;
                if (!mbar_wait(&kv_empty[s], ((j / KS) & 1) ^ 1, a.err, kErrWait, abort_flag)) goto done;
                uint8_t* st = skv + s * KV_STAGE;
                float* ssc = sscale + s * 2 * TK;
                if (j == T_pre) {
                    // node K/V rows (f16), zero past the last node
                    const bool ok = kr < a.N;
                    const size_t src = (((size_t)b * a.N + (ok ? kr : 0)) * a.Hkv + h) * D + hh * 64;
#pragma unroll
                    for (int kvs = 0; kvs < 2; ++kvs) {
                        const uint4* g = reinterpret_cast<const uint4*>((kvs ? a.node_v : a.node_k) + src);
                        uint4 v[8];
#pragma unroll
                        for (int c = 0; c < 8; ++c) v[c] = ok ? g[c] : make_uint4(0, 0, 0, 0);
#pragma unroll
                        for (int c = 0; c < 8; ++c)
                            *reinterpret_cast<uint4*>(st + kvs * 2 * KV_HALF + hh * KV_HALF + sw128(kr, c)) = v[c];
                    }
                    ssc[t] = 1.0f;  // node K/V are not scaled
                } else {
                    const int r = j % RS;
                    if (!mbar_wait(&raw_full[r], (j / RS) & 1, a.err, kErrWait, abort_flag)) goto done;
                    const uint8_t* rs = sraw + r * RAW_STAGE;
#pragma unroll
                    for (int kvs = 0; kvs < 2; ++kvs) {
                        const uint4* src = reinterpret_cast<const uint4*>(rs + kvs * RAW_KV + kr * D + hh * 64);
                        uint8_t* dst = st + kvs * 2 * KV_HALF + hh * KV_HALF;
#pragma unroll
                        for (int c4 = 0; c4 < 4; ++c4) {
                            // chunks in a per-row rotation: the 16 rows a warp reads
                            // (128 B apart) then spread over all banks
                            const int cc = (c4 + kr) & 3;
                            const uint4 raw = src[cc];  // 16 int8 -> two 16-byte f16 chunks
                            uint32_t o[8];
                            i8x4_to_f16(raw.x, o[0], o[1]);
                            i8x4_to_f16(raw.y, o[2], o[3]);
                            i8x4_to_f16(raw.z, o[4], o[5]);
                            i8x4_to_f16(raw.w, o[6], o[7]);
                            *reinterpret_cast<uint4*>(dst + sw128(kr, 2 * cc)) = make_uint4(o[0], o[1], o[2], o[3]);
                            *reinterpret_cast<uint4*>(dst + sw128(kr, 2 * cc + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
                        }
                    }
                    const __half* sc = reinterpret_cast<const __half*>(rs + 2 * RAW_KV);
                    ssc[t] = __half2float(sc[t]);  // t < 64: K scales, t >= 64: V scales
                    mbar_arrive(&raw_empty[r]);    // after every read of the raw stage
                }
                fence_async_smem();
                mbar_arrive(&kv_full[s]);
            }
        }
    }
done:
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, C::kTmemCols);
    }
}

template <bool INT8, int QT>
cudaError_t launch_impl(const TreeAttnArgs& a, cudaStream_t stream) {
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(once, [] {
        attr_err = cudaFuncSetAttribute(tree_attn_kernel<INT8, QT>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)AttnCfg<INT8, QT>::kSmem);
    });
    if (attr_err != cudaSuccess) return attr_err;
    CUtensorMap tk{}, tv{}, tnk{}, tnv{};
    if (!INT8) {
        const uint64_t rows = (uint64_t)a.pool_pages * a.Hkv * kKvPage;
        cudaError_t e = make_tmap_f16_2d(&tk, a.k_pool, rows, D, D * 2, kKvPage);
        if (e == cudaSuccess) e = make_tmap_f16_2d(&tv, a.v_pool, rows, D, D * 2, kKvPage);
        const uint64_t nodes = (uint64_t)a.B * a.N;
        if (e == cudaSuccess)
            e = make_tmap_f16_3d(&tnk, a.node_k, D, a.Hkv, nodes, D * 2, (uint64_t)a.Hkv * D * 2, TK);
        if (e == cudaSuccess)
            e = make_tmap_f16_3d(&tnv, a.node_v, D, a.Hkv, nodes, D * 2, (uint64_t)a.Hkv * D * 2, TK);
        if (e != cudaSuccess) return e;
    }
    const int G = a.Hq / a.Hkv;
    const int MT = (a.N * G + QT * BMQ - 1) / (QT * BMQ);
    const long grid = (long)a.B * a.Hkv * MT;
    tree_attn_kernel<INT8, QT><<<(unsigned)grid, kThreads, AttnCfg<INT8, QT>::kSmem, stream>>>(tk, tv, tnk,
                                                                                              tnv, a);
    return cudaGetLastError();
}

// VELO_ATTN_QUERY_TILES=1 in the environment keeps one query tile per CTA at
// every size (read at each launch; for comparisons of the two layouts).
bool force_one_tile() {
    const char* e = std::getenv("VELO_ATTN_QUERY_TILES");
    return e != nullptr && e[0] == '1' && e[1] == '\0';
}

// Query rows per KV head (nodes x group heads) above 128 take two query tiles
// per CTA, so each K/V tile is fetched (and converted) once for both.
template <bool INT8>
cudaError_t launch_rows(const TreeAttnArgs& a, cudaStream_t stream) {
    const int rows = a.N * (a.Hq / a.Hkv);
    if (rows > BMQ && !force_one_tile()) return launch_impl<INT8, 2>(a, stream);
    return launch_impl<INT8, 1>(a, stream);
}

}  // namespace

cudaError_t launch_tree_ancestors(const int32_t* parents, int B, int N, uint64_t* anc, int* err,
                                  cudaStream_t stream) {
    const int n = B * N;
    tree_ancestors_kernel<<<(n + 127) / 128, 128, 0, stream>>>(parents, B, N, anc, err);
    return cudaGetLastError();
}

cudaError_t launch_tree_attention(const TreeAttnArgs& a, bool kv_int8, cudaStream_t stream) {
    return kv_int8 ? launch_rows<true>(a, stream) : launch_rows<false>(a, stream);
}

}  // namespace velo
