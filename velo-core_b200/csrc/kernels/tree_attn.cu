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
// final tile with an ancestor mask.  S = Q K^T (M=128, N=64) and O += P V
// (M=128, N=128, V MN-major) take Q and P as A operands from tensor memory,
// so the tensor core reads only K and V from shared memory; O accumulates in
// TMEM and is rescaled there only when a row's running max grows by > 2^8.
// Roles: a producer warp (TMA of f16 pages with 128-byte swizzle straight into
// the operand tiles, the tree tile by a 3-D TMA; or raw bulk copies of int8
// pages and scales), one MMA-issuing thread, softmax warps (a thread per query
// row: S from TMEM, exp2 on the SFU, P as f16 pairs back into TMEM) and, for
// int8 pools, converter warps (exact int8 -> f16 into the swizzled operand
// layout, and the tree tile from the node K/V).
#include <cuda_fp16.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common/sm100.cuh"
#include "common/smem_attr.cuh"
#include "common/spec_math.cuh"  // max3
#include "kernels/q4gemm.h"  // make_tmap_f16_2d
#include "kernels/tree_attn.h"

namespace velo {
namespace {

using namespace sm100;

constexpr int D = kAttnHeadDim;        // 128
constexpr int TK = 64;                 // keys per tile
constexpr int BMQ = 128;               // query rows per query tile
constexpr int KV_HALF = TK * 64 * 2;           // 8 KiB: 64 keys x 64 dims
constexpr int KV_STAGE = 4 * KV_HALF;          // K halves + V halves: 32 KiB
constexpr int RAW_KV = TK * D;                 // int8 tile of K (or V): 8 KiB
constexpr int RAW_STAGE = 2 * RAW_KV + 2 * TK * 2;  // K, V, K scales, V scales
constexpr float kRescaleLog2 = 8.0f;           // lazy O rescale threshold

constexpr int kErrPage = 0x5101, kErrWait = 0x5102;

// swizzled byte offset of 16-byte chunk c of row r in a 128-byte-row tile
__device__ __forceinline__ uint32_t sw128(int r, int c) {
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// Four int8 (little-endian in w) -> f16 pairs (b0,b1), (b2,b3), exactly:
// flipping the sign bit gives u = x + 128, 0x6400 | u is 1024 + u in f16, and
// subtracting 1152 leaves x.
// Then times the token's scale sc2 (both halves), rounded to f16 once.
__device__ __forceinline__ void i8x4_to_f16(uint32_t w, __half2 sc2, uint32_t& lo, uint32_t& hi) {
    const uint32_t u = w ^ 0x80808080u;
    const uint32_t r01 = __byte_perm(u, 0x64646464u, 0x5140);
    const uint32_t r23 = __byte_perm(u, 0x64646464u, 0x5342);
    const __half2 k = __half2half2(__ushort_as_half(0x6480));  // 1152
    const __half2 a = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&r01), k), sc2);
    const __half2 c = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&r23), k), sc2);
    lo = *reinterpret_cast<const uint32_t*>(&a);
    hi = *reinterpret_cast<const uint32_t*>(&c);
}

// Maximum of 32 raw scores of a query row.  kMasked: scores of keys without
// a bit in kmask become -inf first (the tree tile and a ragged last tile).
template <bool kMasked>
__device__ __forceinline__ float raw_max32(uint32_t (&x32)[32], uint32_t kmask) {
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

// Producer role (one warp on warp-uniform state; an elected lane issues the
// copies): the K/V tiles of the sequence's pages into the ring -- f16 pools by
// TMA (128-byte swizzle straight into the operand tiles, the tree tile by a
// 3-D TMA of the node rows), int8 pools as raw bulk copies of pages and scales
// for the converters.  Returns early on abort.
template <bool INT8, int KS, int RS>
__device__ __forceinline__ void produce_tiles(const TreeAttnArgs& a, const CUtensorMap* tmk,
                                              const CUtensorMap* tmv, const CUtensorMap* tnk,
                                              const CUtensorMap* tnv, int b, int h, int T_pre, int T,
                                              uint8_t* skv, uint8_t* sraw, uint64_t* kv_full,
                                              uint64_t* kv_empty, uint64_t* raw_full, uint64_t* raw_empty,
                                              volatile int* abort_flag) {
    constexpr int PPT = TK / kKvPage;  // pages per tile
    const uint32_t* pt = a.page_table + (size_t)b * a.max_pages;
    // page ids of the next tile are read one iteration early, so the
    // global-memory latency hides behind the wait for a free slot
    uint32_t pg_next[PPT];
    auto fetch = [&](int j, uint32_t (&dst)[PPT]) {
#pragma unroll
        for (int i = 0; i < PPT; ++i) {
            const int pi = j * PPT + i;
            dst[i] = (j < T_pre && pi < a.max_pages) ? pt[pi] : 0u;
        }
    };
    fetch(0, pg_next);
    for (int j = 0; j < (INT8 ? T_pre : T); ++j) {
        uint32_t pg[PPT];
        bool bad = false;
#pragma unroll
        for (int i = 0; i < PPT; ++i) {
            pg[i] = pg_next[i];
            if (pg[i] >= (uint32_t)a.pool_pages) {
                bad = true;
                pg[i] = 0;
            }
        }
        fetch(j + 1, pg_next);
        if constexpr (!INT8) {
            const int s = j % KS;
            const bool ok = mbar_wait(&kv_empty[s], ((j / KS) & 1) ^ 1, a.err, kErrWait, abort_flag, 64);
            if (!__all_sync(0xffffffffu, ok)) return;
            if (elect_one()) {
                if (bad) atomicCAS(a.err, 0, kErrPage);
                mbar_arrive_expect_tx(&kv_full[s], KV_STAGE);
                uint8_t* st = skv + s * KV_STAGE;
                if (j == T_pre) {
                    // tree tile: node K/V rows b*N .. b*N+63 of KV head h (3-D
                    // maps [B*N][Hkv][128]); rows past this sequence's nodes
                    // are masked, rows past the tensor read as zero
                    for (int dh = 0; dh < 2; ++dh) {
                        tma_load_3d(st + dh * KV_HALF, tnk, &kv_full[s], dh * 64, h, b * a.N);
                        tma_load_3d(st + 2 * KV_HALF + dh * KV_HALF, tnv, &kv_full[s], dh * 64, h, b * a.N);
                    }
                } else {
                    for (int i = 0; i < PPT; ++i) {
                        const int row = (int)((pg[i] * a.Hkv + h) * kKvPage);
                        for (int dh = 0; dh < 2; ++dh) {
                            tma_load_2d(st + dh * KV_HALF + i * 2048, tmk, &kv_full[s], dh * 64, row);
                            tma_load_2d(st + 2 * KV_HALF + dh * KV_HALF + i * 2048, tmv, &kv_full[s], dh * 64,
                                        row);
                        }
                    }
                }
            }
            __syncwarp();
        } else {
            const int r = j % RS;
            const bool ok = mbar_wait(&raw_empty[r], ((j / RS) & 1) ^ 1, a.err, kErrWait, abort_flag, 64);
            if (!__all_sync(0xffffffffu, ok)) return;
            if (elect_one()) {
                if (bad) atomicCAS(a.err, 0, kErrPage);
                mbar_arrive_expect_tx(&raw_full[r], RAW_STAGE);
                uint8_t* st = sraw + r * RAW_STAGE;
                for (int i = 0; i < PPT; ++i) {
                    const size_t blk = (size_t)pg[i] * a.Hkv + h;  // (page, head) block
                    bulk_load(st + i * 2048, static_cast<const int8_t*>(a.k_pool) + blk * 2048, 2048,
                              &raw_full[r]);
                    bulk_load(st + RAW_KV + i * 2048, static_cast<const int8_t*>(a.v_pool) + blk * 2048, 2048,
                              &raw_full[r]);
                    bulk_load(st + 2 * RAW_KV + i * 32, a.k_scale + blk * kKvPage, 32, &raw_full[r]);
                    bulk_load(st + 2 * RAW_KV + TK * 2 + i * 32, a.v_scale + blk * kKvPage, 32, &raw_full[r]);
                }
            }
            __syncwarp();
        }
    }
}

// Converter role (128 threads from conv_base), int8 pools only: every tile of
// the ring -- the cached tokens converted from the raw stage into the
// swizzled f16 operand layout, the tree tile from the node K/V rows -- and
// the per-token scales.  Returns early on abort.
template <bool INT8, int KS, int RS>
__device__ __forceinline__ void convert_tiles(const TreeAttnArgs& a, int conv_base, int b, int h, int T_pre,
                                              int T, uint8_t* skv, const uint8_t* sraw, uint64_t* kv_full,
                                              uint64_t* kv_empty, uint64_t* raw_full, uint64_t* raw_empty,
                                              volatile int* abort_flag) {
    if constexpr (INT8) {
        const int t = threadIdx.x - conv_base;  // 0..127
        const int kr = t >> 1, hh = t & 1;  // key row, 64-dim half
        for (int j = 0; j < T; ++j) {
            const int s = j % KS;
            if (!mbar_wait(&kv_empty[s], ((j / KS) & 1) ^ 1, a.err, kErrWait, abort_flag)) return;
            uint8_t* st = skv + s * KV_STAGE;
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
            } else {
                const int r = j % RS;
                if (!mbar_wait(&raw_full[r], (j / RS) & 1, a.err, kErrWait, abort_flag)) return;
                const uint8_t* rs = sraw + r * RAW_STAGE;
                const __half* sc = reinterpret_cast<const __half*>(rs + 2 * RAW_KV);  // K scales, V scales
#pragma unroll
                for (int kvs = 0; kvs < 2; ++kvs) {
                    const __half2 sc2 = __half2half2(sc[kvs * TK + kr]);  // this key row's scale
                    const uint4* src = reinterpret_cast<const uint4*>(rs + kvs * RAW_KV + kr * D + hh * 64);
                    uint8_t* dst = st + kvs * 2 * KV_HALF + hh * KV_HALF;
#pragma unroll
                    for (int c4 = 0; c4 < 4; ++c4) {
                        // chunks in a per-row rotation: the 16 rows a warp reads
                        // (128 B apart) then spread over all banks
                        const int cc = (c4 + kr) & 3;
                        const uint4 raw = src[cc];  // 16 int8 -> two 16-byte f16 chunks
                        uint32_t o[8];
                        i8x4_to_f16(raw.x, sc2, o[0], o[1]);
                        i8x4_to_f16(raw.y, sc2, o[2], o[3]);
                        i8x4_to_f16(raw.z, sc2, o[4], o[5]);
                        i8x4_to_f16(raw.w, sc2, o[6], o[7]);
                        *reinterpret_cast<uint4*>(dst + sw128(kr, 2 * cc)) = make_uint4(o[0], o[1], o[2], o[3]);
                        *reinterpret_cast<uint4*>(dst + sw128(kr, 2 * cc + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
                    }
                }
                mbar_arrive(&raw_empty[r]);  // after every read of the raw stage
            }
            fence_async_smem();
            mbar_arrive(&kv_full[s]);
        }
    }
}

// ---------------------------------------------------------------- kernel
// Q and P are the A operands of their MMAs straight from tensor memory
// (tcgen05.mma with A in TMEM), so the tensor core reads only K and V from
// shared memory; P_j is written over the first 32 columns of its own S_j.
// QT = 1: per CTA 128 query rows, S/P double-buffered.  QT = 2 (more than 128
// rows per KV head): two query tiles share every K/V tile (fetched, and for
// int8 pools converted, once), one S/P buffer per tile, so S_j of a tile is
// issued only after its PV_{j-1}; the other tile keeps the tensor core busy.
//   warp 0            producer          warp 1  MMA issue     warp 2  TMEM
//   warps 4 .. 4+4QT-1 softmax, one thread per query row (all 64 keys of a
//                     tile; warps 4-7 tile 0, 8-11 tile 1); they also place
//                     the Q rows into TMEM at the start
//   next 4 warps      (int8 pools) converters
template <bool INT8, int QT>
struct TmCfg {
    static_assert(QT == 1 || QT == 2, "one or two query tiles per CTA");
    static constexpr int kThreads = 128 + QT * 128 + 128;
    static constexpr int kConvBase = 128 + QT * 128;
    static constexpr int SB = QT == 1 ? 2 : 1;     // S/P buffers per query tile
    static constexpr int KS = INT8 ? 4 : 6;        // f16 operand ring
    static constexpr int RS = INT8 ? 4 : 0;        // raw int8 ring
    // TMEM columns: Q of tile qt (64 columns of f16 pairs), its S/P buffers
    // (64 each), its O (128); 512 allocated
    static constexpr uint32_t colQ(int qt) { return QT == 1 ? 0u : (uint32_t)qt * 64u; }
    static constexpr uint32_t colS(int qt, int sb) { return QT == 1 ? 64u + (uint32_t)sb * 64u : 128u + (uint32_t)qt * 64u; }
    static constexpr uint32_t colO(int qt) { return 256u + (uint32_t)qt * 128u; }
    static constexpr uint32_t kCols = 512;
    // ring, raw ring, alignment, barriers
    static constexpr size_t kSmem = (size_t)KS * KV_STAGE + (size_t)RS * RAW_STAGE + 1024 + 512;
    static_assert(kSmem <= 232448, "shared memory budget (227 KiB per block)");
};

// Per query tile barriers: s_full[2], p_full[2] (SB used), pv_done (phase j <->
// PV_j done), o_full (the last PV done).
struct TileBars {
    uint64_t* s_full;
    uint64_t* p_full;
    uint64_t* pv_done;
    uint64_t* o_full;
};
__device__ __forceinline__ TileBars tile_bars(uint64_t* qbars, int qt) {
    uint64_t* q = qbars + qt * 6;
    return TileBars{q, q + 2, q + 4, q + 5};
}

// 2^y for y <= 0 on the FMA pipe, two lanes at once: y = j + f with j = rn(y)
// (the 1.5 * 2^23 addition trick), f in [-0.5, 0.5]; 2^f by a cubic fitted for
// minimax relative error on that interval (coefficients from a reweighted
// least-squares / Remez iteration: max relative error 7.5e-5, below the 2^-11
// of the f16 rounding P goes through next); 2^j added to the exponent bits.
// y is clamped at -126, so masked keys (-inf) give ~1e-38, which is 0 in f16
// and nothing in an f32 row sum.  The softmax evaluates a quarter of its
// exponentials this way so that the special-function unit, which takes the
// rest, stops bounding the softmax (it did: 45 % XU against 45 % tensor pipe).
__device__ __forceinline__ float2 exp2_fma2(float2 y) {
    constexpr float kMagic = 12582912.0f;
    y.x = fmaxf(y.x, -126.0f);
    y.y = fmaxf(y.y, -126.0f);
    const float2 t = __fadd2_rn(y, make_float2(kMagic, kMagic));
    const float2 jf = __fadd2_rn(t, make_float2(-kMagic, -kMagic));
    const float2 f = __fadd2_rn(y, make_float2(-jf.x, -jf.y));
    float2 p = __ffma2_rn(make_float2(0.0551705f, 0.0551705f), f, make_float2(0.24260852f, 0.24260852f));
    p = __ffma2_rn(p, f, make_float2(0.69326094f, 0.69326094f));
    p = __ffma2_rn(p, f, make_float2(0.99992824f, 0.99992824f));
    const uint32_t kb = __float_as_uint(kMagic);
    return make_float2(__uint_as_float(__float_as_uint(p.x) + ((__float_as_uint(t.x) - kb) << 23)),
                       __uint_as_float(__float_as_uint(p.y) + ((__float_as_uint(t.y) - kb) << 23)));
}

// 2^(x * sl2 - ms) of 16 keys (one packed FMA per pair), packed as 8 f16
// pairs into pw; returns the pairwise sums.  Pairs 1 and 5 take the FMA-pipe
// exponential, the others the special-function unit.
__device__ __forceinline__ float2 exp_pack16(const uint32_t* x, float sl2, float ms, uint32_t (&pw)[8]) {
    float2 acc = make_float2(0.0f, 0.0f);
    const float2 s2 = make_float2(sl2, sl2), nm = make_float2(-ms, -ms);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float2 y = __ffma2_rn(make_float2(__uint_as_float(x[2 * i]), __uint_as_float(x[2 * i + 1])), s2, nm);
        const float2 pp = (i & 3) == 1 ? exp2_fma2(y)
                                       : make_float2(ex2_approx(y.x), ex2_approx(y.y));  // masked (-inf) -> 0
        acc = __fadd2_rn(acc, pp);
        __half2 hp = __floats2half2_rn(pp.x, pp.y);
        pw[i] = *reinterpret_cast<uint32_t*>(&hp);
    }
    return acc;
}


// Softmax role: thread = query row r of tile qt (TMEM lane r).  Returns
// early (the CTA then exits) when a wait runs out or another role aborted.
template <bool INT8, int QT>
__device__ __forceinline__ void softmax_rows(const TreeAttnArgs& a, int warp, int lane, int mt, int b, int h,
                                             int L, int T_pre, int T, int G, int rows_total, uint32_t tmem,
                                             uint64_t* q_full, const TileBars& tb, volatile int* abort_flag) {
    using C = TmCfg<INT8, QT>;
    constexpr int SB = C::SB;
    const int qt = (warp - 4) >> 2, q = warp & 3;
    const int r = q * 32 + lane;
    const int row = (mt * QT + qt) * BMQ + r;
    const bool row_ok = row < rows_total;
    const int node = row_ok ? row / G : 0, g = row_ok ? row % G : 0;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const uint32_t t_o = tmem + lane_base + C::colO(qt);
    const size_t qo = (((size_t)b * a.N + node) * a.Hq + h * G + g) * D;  // Q / output row
    {
        // the row's Q (128 f16 = 64 columns of pairs) into TMEM; zeros for
        // absent rows, whose S and P then stay zero
        const uint4* src = reinterpret_cast<const uint4*>(a.q + qo);
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            uint32_t qa[32];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint4 v = row_ok ? src[hf * 8 + i] : make_uint4(0, 0, 0, 0);
                qa[4 * i] = v.x; qa[4 * i + 1] = v.y; qa[4 * i + 2] = v.z; qa[4 * i + 3] = v.w;
            }
            tmem_st_32x32b_x32(tmem + lane_base + C::colQ(qt) + hf * 32, qa);
        }
        tmem_st_wait();
    }
    tc_fence_before();
    mbar_arrive(q_full);
    if (!__any_sync(0xffffffffu, row_ok)) {
        // no query row of this warp exists: it only keeps the barrier counts
        // (its lanes' P columns hold S of zero Q rows, i.e. zeros)
        for (int j = 0; j < T; ++j) {
            const int sb = j % SB;
            const bool got = mbar_wait(&tb.s_full[sb], (j / SB) & 1, a.err, kErrWait, abort_flag, 32);
            if (!__all_sync(0xffffffffu, got)) return;
            mbar_arrive(&tb.p_full[sb]);
        }
        return;
    }
    const uint64_t anc = a.anc[(size_t)b * a.N + node];
    float m = -INFINITY, l = 0.0f;
    for (int j = 0; j < T; ++j) {
        const int sb = j % SB;
        bool got = mbar_wait(&tb.s_full[sb], (j / SB) & 1, a.err, kErrWait, abort_flag);
        if (!__all_sync(0xffffffffu, got)) return;
        tc_fence_after();
        const uint32_t sc = tmem + lane_base + C::colS(qt, sb);  // S_j, then P_j
        uint32_t xa[32], xb[32];
        tmem_ld_32x32b_x32(sc, xa);
        tmem_ld_32x32b_x32(sc + 32, xb);
        tmem_ld_wait();
        // maximum of the row's raw scores (scale_log2 > 0 commutes with max):
        // full tiles of cached tokens need no mask; the tree tile keeps the
        // node's ancestors, a ragged last tile the tokens below ctx_len
        float mx;
        if (j < T_pre && L - j * TK >= TK) {
            mx = fmaxf(raw_max32<false>(xa, 0u), raw_max32<false>(xb, 0u));
        } else {
            uint64_t kmask;
            if (j == T_pre) {
                kmask = anc;
            } else {
                const int nvalid = L - j * TK;
                kmask = nvalid <= 0 ? 0ull : (1ull << nvalid) - 1ull;  // nvalid < 64 here
            }
            mx = fmaxf(raw_max32<true>(xa, (uint32_t)kmask), raw_max32<true>(xb, (uint32_t)(kmask >> 32)));
        }
        mx *= a.scale_log2;  // the scaled maximum, exactly (rounding is monotonic)
        // lazy rescale, decided per warp so the TMEM accesses stay convergent
        if (__any_sync(0xffffffffu, mx > m + kRescaleLog2)) {
            const float m_new = fmaxf(m, mx);
            const float f = m == -INFINITY ? 0.0f : ex2_approx(m - m_new);
            l *= f;
            if (j > 0) {
                if constexpr (SB == 2) {
                    // O holds PV_0..PV_{j-1}; wait for PV_{j-1}.  Its phase is
                    // the only one in doubt: S_j was issued after PV_{j-2} (so
                    // phase j-2 is complete) and PV_j needs this tile's P (so
                    // phase j is not), hence a parity wait is exact here.
                    got = mbar_wait(tb.pv_done, (j - 1) & 1, a.err, kErrWait, abort_flag);
                    if (!__all_sync(0xffffffffu, got)) return;
                    tc_fence_after();
                }
                // (one buffer: S_j was issued after PV_{j-1}, which the
                // tensor pipe completed before S_j)
#pragma unroll 1
                for (int c = 0; c < 8; ++c) {
                    uint32_t o[16];
                    tmem_ld_32x32b_x16(t_o + c * 16, o);
                    tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
                    tmem_st_32x32b_x16(t_o + c * 16, o);
                }
            }
            m = m_new;
        }
        // P_j (f16 pairs) over the first 32 columns of S_j, 8 columns at a time
        const float ms = m == -INFINITY ? 0.0f : m;  // all keys masked so far: p = 0
        float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
            uint32_t pw[8];
            const float2 sq = exp_pack16((qq < 2 ? xa : xb) + (qq & 1) * 16, a.scale_log2, ms, pw);
            acc = __fadd2_rn(acc, sq);
            tmem_st_32x32b_x8(sc + qq * 8, pw);
        }
        l += acc.x + acc.y;
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&tb.p_full[sb]);
    }
    // epilogue: O / l after the last PV
    {
        const bool ok = mbar_wait(tb.o_full, 0, a.err, kErrWait, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) return;
    }
    tc_fence_after();
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        const int col = c * 32;
        tmem_ld_32x32b_x32(t_o + col, o);
        tmem_ld_wait();
        if (!row_ok) continue;
        if (a.out_f16) {
            __half* dst = static_cast<__half*>(a.out) + qo + col;
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
            float* dst = static_cast<float*>(a.out) + qo + col;
#pragma unroll
            for (int qq = 0; qq < 8; ++qq)
                reinterpret_cast<float4*>(dst)[qq] =
                    make_float4(__uint_as_float(o[4 * qq]) * inv, __uint_as_float(o[4 * qq + 1]) * inv,
                                __uint_as_float(o[4 * qq + 2]) * inv, __uint_as_float(o[4 * qq + 3]) * inv);
        }
    }
}

template <bool INT8, int QT>
__global__ void __launch_bounds__(TmCfg<INT8, QT>::kThreads, 1)
    tree_attn_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                     const __grid_constant__ CUtensorMap tnk, const __grid_constant__ CUtensorMap tnv,
                     const TreeAttnArgs a) {
    using C = TmCfg<INT8, QT>;
    constexpr int KS = C::KS, RS = C::RS, SB = C::SB;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* skv = base;                               // KS x (K0 K1 V0 V1) 8 KiB each
    uint8_t* sraw = skv + KS * KV_STAGE;               // RS x raw int8 stage
    uint64_t* bars = reinterpret_cast<uint64_t*>(sraw + RS * RAW_STAGE);
    uint64_t* kv_full = bars;
    uint64_t* kv_empty = kv_full + KS;
    uint64_t* raw_full = kv_empty + KS;                // RS entries (int8)
    uint64_t* raw_empty = raw_full + (RS ? RS : 1);
    uint64_t* q_full = raw_empty + (RS ? RS : 1);      // Q rows in TMEM
    uint64_t* qbars = q_full + 1;                      // QT x 6 (tile_bars)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(qbars + QT * 6);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

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
        mbar_init(q_full, QT * BMQ);
        for (int qt = 0; qt < QT; ++qt) {
            const TileBars tb = tile_bars(qbars, qt);
            for (int i = 0; i < 2; ++i) {
                mbar_init(&tb.s_full[i], 1);
                mbar_init(&tb.p_full[i], BMQ);
            }
            mbar_init(tb.pv_done, 1);
            mbar_init(tb.o_full, 1);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 2) {
        tmem_alloc(tmem_slot, C::kCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        produce_tiles<INT8, KS, RS>(a, &tmk, &tmv, &tnk, &tnv, b, h, T_pre, T, skv, sraw, kv_full, kv_empty,
                                    raw_full, raw_empty, abort_flag);
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issue
        // The whole warp runs on warp-uniform state; an elected lane issues
        // each group of MMAs and its commits.  Per query tile, S_j = Q K_j^T
        // (A: Q in TMEM) and PV_j: O += P_j V_j (A: P_j in TMEM, over S_j's
        // columns).  The tensor pipe runs one CTA's MMAs in issue order, so
        // S_j may follow PV_{j-SB} (the last reader of its buffer) at once.
        // Fixed order with blocking waits: after PV_j of a tile comes S_{j+SB}
        // of that tile, and the query tiles take turns, so one tile's MMAs
        // run while the other tile's softmax works.  With two buffers, when
        // S_j completes every PV before j-1 has completed (the softmax waits
        // for PV_{j-1} by parity).  A K/V stage is released after the last
        // query tile's PV of it.
        {
            const uint32_t id_s = idesc_f16_f32(BMQ, TK);
            const uint32_t id_pv = idesc_f16_f32(BMQ, D, /*b_mn_major=*/true);
            bool ok = mbar_wait(q_full, 0, a.err, kErrWait, abort_flag);
            if (!__all_sync(0xffffffffu, ok)) goto done;
            tc_fence_after();
            auto issue_s = [&](int qt, int j) -> bool {  // false: gave up
                const int s = j % KS, sb = j % SB;
                const bool got = mbar_wait(&kv_full[s], (j / KS) & 1, a.err, kErrWait, abort_flag);
                if (!__all_sync(0xffffffffu, got)) return false;
                tc_fence_after();
                const uint32_t k_addr = smem_u32(skv + s * KV_STAGE);
                if (elect_one()) {
#pragma unroll
                    for (int k = 0; k < D / 16; ++k) {
                        const uint64_t bd = desc_kmajor_sw128(k_addr + (k >> 2) * KV_HALF) + (k & 3) * 2;
                        mma_f16_ts(tmem + C::colS(qt, sb), tmem + C::colQ(qt) + k * 8, bd, id_s, k > 0);
                    }
                    mma_commit(&tile_bars(qbars, qt).s_full[sb]);
                }
                __syncwarp();
                return true;
            };
            auto issue_pv = [&](int qt, int j) -> bool {
                const TileBars tb = tile_bars(qbars, qt);
                const int pb = j % SB, sv = j % KS;
                const bool got = mbar_wait(&tb.p_full[pb], (j / SB) & 1, a.err, kErrWait, abort_flag);
                if (!__all_sync(0xffffffffu, got)) return false;
                tc_fence_after();
                const uint32_t v_addr = smem_u32(skv + sv * KV_STAGE + 2 * KV_HALF);
                if (elect_one()) {
#pragma unroll
                    for (int kk = 0; kk < TK / 16; ++kk) {
                        const uint64_t bd = desc_mnmajor_sw128(v_addr + kk * 2048, KV_HALF);
                        mma_f16_ts(tmem + C::colO(qt), tmem + C::colS(qt, pb) + kk * 8, bd, id_pv, (j | kk) != 0);
                    }
                    if (qt == QT - 1) mma_commit(&kv_empty[sv]);  // the stage's last reader
                    mma_commit(tb.pv_done);
                    if (j == T - 1) mma_commit(tb.o_full);
                }
                __syncwarp();
                return true;
            };
            for (int j = 0; j < SB && j < T; ++j)
                for (int qt = 0; qt < QT; ++qt)
                    if (!issue_s(qt, j)) goto done;
            for (int j = 0; j < T; ++j)
                for (int qt = 0; qt < QT; ++qt) {
                    if (!issue_pv(qt, j)) goto done;
                    if (j + SB < T && !issue_s(qt, j + SB)) goto done;
                }
        }
    } else if (warp >= 4 && warp < 4 + 4 * QT) {
        softmax_rows<INT8, QT>(a, warp, lane, mt, b, h, L, T_pre, T, G, rows_total, tmem, q_full,
                               tile_bars(qbars, (warp - 4) >> 2), abort_flag);
    } else if (warp >= 4 + 4 * QT) {
        convert_tiles<INT8, KS, RS>(a, C::kConvBase, b, h, T_pre, T, skv, sraw, kv_full, kv_empty, raw_full,
                                    raw_empty, abort_flag);
    }
done:
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, C::kCols);
    }
}

// Tensor maps of the f16 pools and node K/V (int8 pools use bulk copies).
template <bool INT8>
cudaError_t make_maps(const TreeAttnArgs& a, CUtensorMap* tk, CUtensorMap* tv, CUtensorMap* tnk,
                      CUtensorMap* tnv) {
    if (INT8) return cudaSuccess;
    const uint64_t rows = (uint64_t)a.pool_pages * a.Hkv * kKvPage;
    cudaError_t e = make_tmap_f16_2d(tk, a.k_pool, rows, D, D * 2, kKvPage);
    if (e == cudaSuccess) e = make_tmap_f16_2d(tv, a.v_pool, rows, D, D * 2, kKvPage);
    const uint64_t nodes = (uint64_t)a.B * a.N;
    if (e == cudaSuccess)
        e = make_tmap_f16_3d(tnk, a.node_k, D, a.Hkv, nodes, D * 2, (uint64_t)a.Hkv * D * 2, TK);
    if (e == cudaSuccess)
        e = make_tmap_f16_3d(tnv, a.node_v, D, a.Hkv, nodes, D * 2, (uint64_t)a.Hkv * D * 2, TK);
    return e;
}

template <bool INT8, int QT>
cudaError_t launch_impl(const TreeAttnArgs& a, cudaStream_t stream) {
    using C = TmCfg<INT8, QT>;
    static SmemAttr attr;
    const cudaError_t attr_err = ensure_smem(attr, tree_attn_kernel<INT8, QT>, (int)C::kSmem);
    if (attr_err != cudaSuccess) return attr_err;
    CUtensorMap tk{}, tv{}, tnk{}, tnv{};
    const cudaError_t e = make_maps<INT8>(a, &tk, &tv, &tnk, &tnv);
    if (e != cudaSuccess) return e;
    const int G = a.Hq / a.Hkv;
    const int MT = (a.N * G + QT * BMQ - 1) / (QT * BMQ);
    const long grid = (long)a.B * a.Hkv * MT;
    tree_attn_kernel<INT8, QT><<<(unsigned)grid, C::kThreads, C::kSmem, stream>>>(tk, tv, tnk, tnv, a);
    return cudaGetLastError();
}

// More than 128 query rows per KV head (nodes x group heads) take two query
// tiles per CTA: each K/V tile is then fetched (and converted) once for 256
// rows (config 4: 802 us against 1246 with one tile per CTA; config-5 layer:
// 359 us against 455) -- unless that grid would leave more than half the SMs
// idle: one rank's heads of the config-5 layer at 8 GPUs (64 sequences x 1 KV
// head = 64 CTAs of two tiles) took 84.1 us, as 128 CTAs of one tile 53.6 us
// (at 4 GPUs, 128 CTAs of two tiles 88.3 us against 256 of one 98.7 us).
// VELO_ATTN_QUERY_TILES=1 or 2 in the environment forces one layout (read at
// each launch; for comparisons).
template <bool INT8>
cudaError_t launch_rows(const TreeAttnArgs& a, cudaStream_t stream) {
    const char* e = std::getenv("VELO_ATTN_QUERY_TILES");
    const bool many_rows = a.N * (a.Hq / a.Hkv) > BMQ;
    int qt = many_rows ? 2 : 1;
    if (qt == 2) {
        int dev = 0, sms = 0;
        if (cudaGetDevice(&dev) == cudaSuccess &&
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess) {
            const long rows = (long)a.N * (a.Hq / a.Hkv);
            const long grid2 = (long)a.B * a.Hkv * ((rows + 2 * BMQ - 1) / (2 * BMQ));
            if (2 * grid2 <= sms) qt = 1;
        }
    }
    if (e != nullptr && std::strcmp(e, "1") == 0) qt = 1;
    if (e != nullptr && std::strcmp(e, "2") == 0 && many_rows) qt = 2;
    return qt == 2 ? launch_impl<INT8, 2>(a, stream) : launch_impl<INT8, 1>(a, stream);
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
