// q4gemm.cu -- q4_0 weights x f16 activations on the sm_100a tensor cores.
//
// Replaces the per-token, per-row `matvec_quant` of the reference CPU path
// (src/llama_cpu.rs:75-90, dequant_row src/quant.rs:50-73) for the verify
// step, where all drafted tokens of all sequences form the M side of one GEMM:
//   Y[m][n] = sum_k X[m][k] * W[n][k],   W = q4_0 dequantised (d * (q - 8)).
//
// Two persistent kernels (one CTA per SM):
//  * q4_gemm_ta_kernel (M > 128 activation rows, plain and residual-add
//    stores): the dequantised weights are the A operand straight from tensor
//    memory (the dequant thread of weight row i writes TMEM lane i), the
//    activations the B operand from shared memory; 128 weight rows x 256
//    activation rows per tile.  Per k step the SM's shared memory then carries
//    the activation tile in (TMA) and out (MMA) and the raw q4_0 tile only.
//  * q4_gemm_ta_swiglu_kernel (M > 128, SwiGLU): the same with
//    the gate and the up row of each output in one TMEM lane (two
//    accumulators), so silu(gate) * up needs no exchange between warps.
//  * q4_gemm_kernel (M <= 128): the dequantised weights pass
//    through shared memory as the B operand; 128 (activation rows) x 256 or
//    128 (weight rows) tiles with a double-buffered accumulator, so the
//    epilogue of one tile overlaps the main loop of the next:
//   warp 0      producer: per k step the activation tile (TMA, 64 k, 128-byte
//               swizzle) and the raw q4_0 tiles (bulk copies) on one barrier
//   warp 1      tcgen05.mma (M=128, N=256, K=16) x 4 per step, elected lane
//   warp 2      allocates / frees 512 TMEM columns
//   warps 4-11  dequantise their weight row of each k step into a ring of
//               swizzled f16 operand tiles
//   warps 12-15 epilogue out of TMEM (tcgen05.ld), fused store / residual
//               add / SwiGLU
// Dequantisation: the nibble order chosen at repack time turns a 32-bit word
// into f16 pairs with one LOP3 each (0x6400 | q = 1024 + q), an exact subtract
// (or exact FMA for the high nibbles) gives q - 8, and one HMUL2 by the block
// scale rounds d * (q - 8) once to f16.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common/sm100.cuh"
#include "common/smem_attr.cuh"
#include "kernels/q4gemm.h"

namespace velo {
namespace {

using namespace sm100;

constexpr int BM = 128, BK = kQ4TileK;
constexpr int X_BYTES = BM * BK * 2;      // 16 KiB
constexpr int kEpilogueThreads = 128;     // last four warps, one accumulator lane each

// Per-width configuration: BN weight rows per CTA tile (one or two repacked
// 128-row tiles per k step).
template <int BN>
struct Cfg {
    static constexpr int SUB = BN / kQ4TileN;               // repacked tiles per step
    static constexpr int W_BYTES = BN * BK * 2;             // 32 / 16 KiB
    static constexpr int RAW_BYTES = SUB * kQ4TileBytes;    // 9 / 4.5 KiB
    // input stage: the activation tile and the raw q4_0 tiles of one k step,
    // one transaction barrier (the copy engine completes about one barrier
    // stage per ~240 ns per SM, whatever its size, so both share one)
    static constexpr int IN_BYTES = ((X_BYTES + RAW_BYTES) + 1023) / 1024 * 1024;
    static constexpr int ISTAGES = BN == 256 ? 6 : 8;       // input ring
    static constexpr int WSTAGES = BN == 256 ? 2 : 3;       // dequantised f16 weight ring
    static constexpr int kDequantThreads = BN;              // warps 4.. : one weight row each
    static constexpr int kThreads = 128 + BN + kEpilogueThreads;
    static constexpr int kEpiWarp0 = (128 + BN) / 32;
    static constexpr int kTmemCols = 2 * BN;                // double-buffered accumulator
    static constexpr size_t kSmemBytes = (size_t)ISTAGES * IN_BYTES + (size_t)WSTAGES * W_BYTES + 1024 + 512;
    static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

// error codes written to Q4GemmArgs::err when a wait gives up
constexpr int kErrWaitEmpty = 0x4101, kErrWaitReady = 0x4102, kErrWaitFull = 0x4103,
              kErrWaitAccum = 0x4104, kErrWaitAccEmpty = 0x4105, kErrWaitWEmpty = 0x4106;

// ---------------------------------------------------------------- repack
__global__ void q4_repack_kernel(const uint8_t* __restrict__ a, const uint8_t* __restrict__ b,
                                 int pair, int N, int K, uint8_t* __restrict__ dst, int n_rows,
                                 int kblocks) {
    const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long)n_rows * kblocks) return;
    const int r = (int)(idx % n_rows);  // row fastest: coalesced 16-byte writes
    const int kb = (int)(idx / n_rows);
    const int t = r / kQ4TileN, l = r % kQ4TileN;
    const int nb = K / 32;
    const uint8_t* src;
    int srow;
    bool valid;
    if (pair) {
        srow = (kQ4TileN / 2) * t + (l % (kQ4TileN / 2));
        src = l < kQ4TileN / 2 ? a : b;
        valid = srow < N / 2;
    } else {
        srow = r;
        src = a;
        valid = srow < N;
    }
    uint8_t q[32];
    uint16_t d = 0;
    if (valid && kb < nb) {
        const uint8_t* p = src + ((size_t)srow * nb + kb) * 18;
        d = (uint16_t)(p[0] | (p[1] << 8));
        for (int i = 0; i < 16; ++i) {
            q[2 * i] = p[2 + i] & 15;
            q[2 * i + 1] = p[2 + i] >> 4;
        }
    } else {
        for (int i = 0; i < 32; ++i) q[i] = 8;
    }
    uint32_t w[4];
    for (int g = 0; g < 4; ++g) {
        const uint8_t* e = q + 8 * g;
        w[g] = (uint32_t)(e[0] | (e[2] << 4)) | ((uint32_t)(e[4] | (e[6] << 4)) << 8) |
               ((uint32_t)(e[1] | (e[3] << 4)) << 16) | ((uint32_t)(e[5] | (e[7] << 4)) << 24);
    }
    const int k_tiles = (kblocks + 1) / 2;
    uint8_t* tile = dst + ((size_t)t * k_tiles + kb / 2) * kQ4TileBytes;
    *reinterpret_cast<uint4*>(tile + (kb & 1) * kQ4Block1Off + l * 16) =
        make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint16_t*>(tile + kQ4ScaleOff + l * 4 + (kb & 1) * 2) = d;
}

// ---------------------------------------------------------------- dequant
// Eight elements (one 32-bit word of the repacked block) -> 16 bytes of f16.
__device__ __forceinline__ uint4 dequant8(uint32_t w, __half2 d2) {
    const uint32_t kMagic = 0x64006400u;
    uint32_t p01, p23, p45, p67;
    // (w & mask) | magic as a single LOP3 each
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(p01) : "r"(w), "r"(0x000F000Fu), "r"(kMagic));
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(p23) : "r"(w), "r"(0x00F000F0u), "r"(kMagic));
    const uint32_t w2 = w >> 8;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(p45) : "r"(w2), "r"(0x000F000Fu), "r"(kMagic));
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(p67) : "r"(w2), "r"(0x00F000F0u), "r"(kMagic));
    const __half2 k1032 = __half2half2(__ushort_as_half(0x6408));  // 1032
    const __half2 k1_16 = __half2half2(__ushort_as_half(0x2C00));  // 1/16
    const __half2 km72 = __half2half2(__ushort_as_half(0xD480));   // -72
    __half2 v01 = __hsub2(*reinterpret_cast<__half2*>(&p01), k1032);
    __half2 v23 = __hfma2(*reinterpret_cast<__half2*>(&p23), k1_16, km72);
    __half2 v45 = __hsub2(*reinterpret_cast<__half2*>(&p45), k1032);
    __half2 v67 = __hfma2(*reinterpret_cast<__half2*>(&p67), k1_16, km72);
    v01 = __hmul2(v01, d2);
    v23 = __hmul2(v23, d2);
    v45 = __hmul2(v45, d2);
    v67 = __hmul2(v67, d2);
    uint4 o;
    o.x = *reinterpret_cast<uint32_t*>(&v01);
    o.y = *reinterpret_cast<uint32_t*>(&v23);
    o.z = *reinterpret_cast<uint32_t*>(&v45);
    o.w = *reinterpret_cast<uint32_t*>(&v67);
    return o;
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

// Row `row` of a repacked q4_0 tile (k 0..63) as 32 f16 pairs, lower k in the low half.
__device__ __forceinline__ void dequant_row64(const uint8_t* tile, int row, uint32_t (&r)[32]) {
    const uint4 c0 = *reinterpret_cast<const uint4*>(tile + row * 16);
    const uint4 c1 = *reinterpret_cast<const uint4*>(tile + kQ4Block1Off + row * 16);
    const uint32_t sc = *reinterpret_cast<const uint32_t*>(tile + kQ4ScaleOff + row * 4);
    const __half2 d0 = __half2half2(__ushort_as_half((uint16_t)(sc & 0xFFFF)));
    const __half2 d1 = __half2half2(__ushort_as_half((uint16_t)(sc >> 16)));
    const uint32_t w0[4] = {c0.x, c0.y, c0.z, c0.w};
    const uint32_t w1[4] = {c1.x, c1.y, c1.z, c1.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const uint4 v = dequant8(w0[q], d0);
        r[4 * q] = v.x; r[4 * q + 1] = v.y; r[4 * q + 2] = v.z; r[4 * q + 3] = v.w;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const uint4 v = dequant8(w1[q], d1);
        r[16 + 4 * q] = v.x; r[16 + 4 * q + 1] = v.y; r[16 + 4 * q + 2] = v.z; r[16 + 4 * q + 3] = v.w;
    }
}

// ---------------------------------------------------------------- epilogue
__device__ __forceinline__ void store_row32(const Q4GemmArgs& a, int m, int n, const uint32_t (&r)[32]) {
    if (a.mode == kEpiPeerBF16) {  // 32 columns of one owner (peer_cols % 32 == 0, n % 32 == 0)
        const int o = n / a.peer_cols;
        uint4* y = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.peer_y[o]) + (size_t)m * a.peer_cols +
                                            (n - o * a.peer_cols));
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            uint4 v;
            uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const __nv_bfloat162 h =
                    __floats2bfloat162_rn(__uint_as_float(r[8 * c + 2 * i]), __uint_as_float(r[8 * c + 2 * i + 1]));
                w[i] = *reinterpret_cast<const uint32_t*>(&h);
            }
            y[c] = v;
        }
        return;
    }
    if (a.mode == kEpiStoreBF16) {
        __nv_bfloat16* y = static_cast<__nv_bfloat16*>(a.y) + (size_t)m * a.ldy + n;
#pragma unroll
        for (int e = 0; e < 32; ++e)
            if (n + e < a.N) y[e] = __float2bfloat16_rn(__uint_as_float(r[e]));
        return;
    }
    if (a.mode == kEpiStoreF16) {
        __half* y = static_cast<__half*>(a.y) + (size_t)m * a.ldy + n;
        if (n + 32 <= a.N && (a.ldy % 8) == 0 && ((uintptr_t)a.y % 16) == 0) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint4 v;
                __half2 h0 = __floats2half2_rn(__uint_as_float(r[8 * c + 0]), __uint_as_float(r[8 * c + 1]));
                __half2 h1 = __floats2half2_rn(__uint_as_float(r[8 * c + 2]), __uint_as_float(r[8 * c + 3]));
                __half2 h2 = __floats2half2_rn(__uint_as_float(r[8 * c + 4]), __uint_as_float(r[8 * c + 5]));
                __half2 h3 = __floats2half2_rn(__uint_as_float(r[8 * c + 6]), __uint_as_float(r[8 * c + 7]));
                v.x = *reinterpret_cast<uint32_t*>(&h0);
                v.y = *reinterpret_cast<uint32_t*>(&h1);
                v.z = *reinterpret_cast<uint32_t*>(&h2);
                v.w = *reinterpret_cast<uint32_t*>(&h3);
                reinterpret_cast<uint4*>(y)[c] = v;
            }
        } else {
#pragma unroll
            for (int e = 0; e < 32; ++e)
                if (n + e < a.N) y[e] = __float2half_rn(__uint_as_float(r[e]));
        }
        return;
    }
    float* y = static_cast<float*>(a.y) + (size_t)m * a.ldy + n;
    const bool add = a.mode == kEpiAddF32;
    if (n + 32 <= a.N && (a.ldy % 4) == 0 && ((uintptr_t)a.y % 16) == 0) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            float4 v = make_float4(__uint_as_float(r[4 * c]), __uint_as_float(r[4 * c + 1]),
                                   __uint_as_float(r[4 * c + 2]), __uint_as_float(r[4 * c + 3]));
            if (add) {
                const float4 o = reinterpret_cast<float4*>(y)[c];
                v.x += o.x;
                v.y += o.y;
                v.z += o.z;
                v.w += o.w;
            }
            reinterpret_cast<float4*>(y)[c] = v;
        }
    } else {
#pragma unroll
        for (int e = 0; e < 32; ++e)
            if (n + e < a.N) y[e] = add ? y[e] + __uint_as_float(r[e]) : __uint_as_float(r[e]);
    }
}

// ---------------------------------------------------------------- GEMM
// Persistent: CTA c takes output tiles c, c + grid, ... (activation-row tile
// fastest, so the CTAs sharing a weight tile run together and read it from
// HBM once).  The k-step counter g runs on across tiles, so every ring keeps
// its phase from one tile to the next.  Two rings:
//   in  (ISTAGES x (16 KiB activations + 9 / 4.5 KiB raw q4_0)) TMA + bulk
//        copies on one barrier -> MMA (activations) and dequant (raw); freed
//        when the MMA commit and every dequant thread have arrived
//   W   (WSTAGES x 32 / 16 KiB)  dequant -> MMA; freed by the MMA commit
// Each CTA walks the k steps of a tile starting at its own offset kt0: all
// CTAs read the same few activation tiles otherwise, and those L2 lines turn
// into a hot spot that stretches the TMA latency to ~2 us.
template <int BN>
__global__ void __launch_bounds__(Cfg<BN>::kThreads, 1)
    q4_gemm_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ Q4GemmArgs a) {
    using C = Cfg<BN>;
    constexpr int ISTAGES = C::ISTAGES, WSTAGES = C::WSTAGES, IN_BYTES = C::IN_BYTES;
    constexpr int W_BYTES = C::W_BYTES, RAW_BYTES = C::RAW_BYTES;
    constexpr int kDequantThreads = C::kDequantThreads, kTmemCols = C::kTmemCols;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sin = base;                             // ISTAGES x (X tile | raw tiles), 1024-aligned
    uint8_t* sw = sin + ISTAGES * IN_BYTES;          // 1024-aligned tiles
    uint64_t* bars = reinterpret_cast<uint64_t*>(sw + WSTAGES * W_BYTES);
    uint64_t* ifull = bars;                          // X and raw tiles landed (tx bytes)
    uint64_t* iempty = ifull + ISTAGES;              // MMAs and dequant done with them
    uint64_t* wfull = iempty + ISTAGES;              // f16 weight tile written
    uint64_t* wempty = wfull + WSTAGES;              // MMAs reading it done
    uint64_t* afull = wempty + WSTAGES;              // accumulator b complete
    uint64_t* aempty = afull + 2;                    // accumulator b drained
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(aempty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KT = (a.K + BK - 1) / BK;
    const int MT = (a.M + BM - 1) / BM;
    const int n_tiles = MT * (q4_n_tiles(a.N) / C::SUB);
    const int kt0 = a.krot ? (int)((blockIdx.x * 5u) % (unsigned)KT) : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < ISTAGES; ++s) {
            mbar_init(&ifull[s], 1);
            mbar_init(&iempty[s], 1 + kDequantThreads);  // the MMA commit + every dequant thread
        }
        for (int s = 0; s < WSTAGES; ++s) {
            mbar_init(&wfull[s], kDequantThreads);
            mbar_init(&wempty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&afull[b], 1);
            mbar_init(&aempty[b], kEpilogueThreads);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 2) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) prefetch_tmap(&tmx);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // producer (whole warp on warp-uniform state; an elected lane issues):
        // the activation tile by TMA and the raw q4_0 tiles by bulk copies, one
        // barrier per stage
        uint32_t g = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
            const int mt = tile % MT, nt = tile / MT;
            const uint8_t* wt = a.w + (size_t)nt * C::SUB * KT * kQ4TileBytes;
            for (int kt = 0; kt < KT; ++kt, ++g) {
                const int s = g % ISTAGES;
                const bool ok = mbar_wait(&iempty[s], ((g / ISTAGES) & 1) ^ 1, a.err, kErrWaitEmpty, abort_flag);
                if (!__all_sync(0xffffffffu, ok)) goto done;
                const int kk = kt + kt0 < KT ? kt + kt0 : kt + kt0 - KT;
                if (elect_one()) {
                    uint8_t* st = sin + s * IN_BYTES;
                    mbar_arrive_expect_tx(&ifull[s], X_BYTES + RAW_BYTES);
                    tma_load_2d(st, &tmx, &ifull[s], kk * BK, mt * BM);
#pragma unroll
                    for (int sub = 0; sub < C::SUB; ++sub)
                        bulk_load(st + X_BYTES + sub * kQ4TileBytes, wt + ((size_t)sub * KT + kk) * kQ4TileBytes,
                                  kQ4TileBytes, &ifull[s]);
                }
                __syncwarp();
            }
        }
    } else if (warp == 1) {
        // MMA issue: the whole warp runs the loop on warp-uniform state (so it
        // stays in uniform registers); one elected lane issues the MMAs and
        // their commits
        const uint32_t idesc = idesc_f16_f32(BM, BN);
        uint32_t g = 0, it = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
            const int b = it & 1;
            const uint32_t aph = (it >> 1) & 1;
            const bool ok = mbar_wait(&aempty[b], aph ^ 1, a.err, kErrWaitAccEmpty, abort_flag);
            if (!__all_sync(0xffffffffu, ok)) goto done;
            tc_fence_after();
            const uint32_t d = tmem + b * BN;
            for (int kt = 0; kt < KT; ++kt, ++g) {
                const int s = g % ISTAGES, ws = g % WSTAGES;
                const bool ready = mbar_wait(&ifull[s], (g / ISTAGES) & 1, a.err, kErrWaitFull, abort_flag) &&
                                   mbar_wait(&wfull[ws], (g / WSTAGES) & 1, a.err, kErrWaitReady, abort_flag);
                if (!__all_sync(0xffffffffu, ready)) goto done;
                tc_fence_after();
                const uint64_t ad = desc_kmajor_sw128(smem_u32(sin + s * IN_BYTES));
                const uint64_t bd = desc_kmajor_sw128(smem_u32(sw + ws * W_BYTES));
                if (elect_one()) {
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)
                        mma_f16_ss(d, ad + 2 * k, bd + 2 * k, idesc, (kt | k) != 0);
                    mma_commit(&iempty[s]);
                    mma_commit(&wempty[ws]);
                }
                __syncwarp();
            }
            if (elect_one()) mma_commit(&afull[b]);
            __syncwarp();
        }
    } else if (warp >= 4 && warp < C::kEpiWarp0) {
        // dequantisation: thread i owns weight row i of every tile
        const int i = threadIdx.x - 128;
        const int rsub = (i / kQ4TileN) * kQ4TileBytes + (i % kQ4TileN) * 16;  // raw offset
        const int rsc = (i / kQ4TileN) * kQ4TileBytes + kQ4ScaleOff + (i % kQ4TileN) * 4;
        const int sx7 = i & 7;
        uint8_t* wrow_base = sw + (i >> 3) * 1024 + (i & 7) * 128;
        uint32_t g = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
            for (int kt = 0; kt < KT; ++kt, ++g) {
                const int s = g % ISTAGES, ws = g % WSTAGES;
                if (!mbar_wait(&ifull[s], (g / ISTAGES) & 1, a.err, kErrWaitFull, abort_flag)) goto done;
                const uint8_t* raw = sin + s * IN_BYTES + X_BYTES;
                const uint4 c0 = *reinterpret_cast<const uint4*>(raw + rsub);
                const uint4 c1 = *reinterpret_cast<const uint4*>(raw + rsub + kQ4Block1Off);
                const uint32_t sc = *reinterpret_cast<const uint32_t*>(raw + rsc);
                if (!mbar_wait(&wempty[ws], ((g / WSTAGES) & 1) ^ 1, a.err, kErrWaitWEmpty, abort_flag))
                    goto done;
                const __half2 d0 = __half2half2(__ushort_as_half((uint16_t)(sc & 0xFFFF)));
                const __half2 d1 = __half2half2(__ushort_as_half((uint16_t)(sc >> 16)));
                uint8_t* wrow = wrow_base + ws * W_BYTES;
                const uint32_t w0[4] = {c0.x, c0.y, c0.z, c0.w};
                const uint32_t w1[4] = {c1.x, c1.y, c1.z, c1.w};
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    *reinterpret_cast<uint4*>(wrow + ((q ^ sx7) << 4)) = dequant8(w0[q], d0);
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    *reinterpret_cast<uint4*>(wrow + (((4 + q) ^ sx7) << 4)) = dequant8(w1[q], d1);
                // the input slot is released only now: the shared loads above have
                // returned (their values were consumed), so the next bulk copy into
                // it (async proxy) cannot overtake them
                mbar_arrive(&iempty[s]);
                fence_async_smem();
                mbar_arrive(&wfull[ws]);
            }
        }
    } else if (warp >= C::kEpiWarp0) {
        // epilogue: the last four warps; warp with (warp % 4) == q drains TMEM
        // lanes 32q .. 32q + 31
        const int q = warp & 3;
        uint32_t it = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
            const int mt = tile % MT, nt = tile / MT;
            const int b = it & 1;
            const bool ok = mbar_wait(&afull[b], (it >> 1) & 1, a.err, kErrWaitAccum, abort_flag);
            __syncwarp();
            if (!__all_sync(0xffffffffu, ok)) goto done;
            tc_fence_after();
            const int m = mt * BM + q * 32 + lane;
            const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + b * BN;
            if (a.mode != kEpiSwiGLU) {
#pragma unroll 1
                for (int j = 0; j < BN / 32; ++j) {
                    const int col = j * 32;
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(trow + col, r);
                    tmem_ld_wait();
                    const int n = nt * BN + col;
                    if (m < a.M && n < a.N) store_row32(a, m, n, r);
                }
            } else {
                // each repacked 128-row tile holds 64 gate rows then 64 up rows
                const int F = a.N / 2;
#pragma unroll 1
                for (int j = 0; j < BN / 64; ++j) {
                    const int col = (j >> 1) * kQ4TileN + (j & 1) * 32;
                    uint32_t gt[32], up[32];
                    tmem_ld_32x32b_x32(trow + col, gt);
                    tmem_ld_32x32b_x32(trow + col + kQ4TileN / 2, up);
                    tmem_ld_wait();
                    const int n = nt * (BN / 2) + j * 32;
                    if (m < a.M && n < F) {
                        __half* y = static_cast<__half*>(a.y) + (size_t)m * a.ldy + n;
#pragma unroll
                        for (int e = 0; e < 32; e += 2) {
                            if (n + e >= F) break;
                            const float v0 = silu(__uint_as_float(gt[e])) * __uint_as_float(up[e]);
                            const float v1 = silu(__uint_as_float(gt[e + 1])) * __uint_as_float(up[e + 1]);
                            if (n + e + 1 < F && ((a.ldy | n) & 1) == 0 && ((uintptr_t)a.y & 3) == 0) {
                                *reinterpret_cast<__half2*>(y + e) = __floats2half2_rn(v0, v1);
                            } else {
                                y[e] = __float2half_rn(v0);
                                if (n + e + 1 < F) y[e + 1] = __float2half_rn(v1);
                            }
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&aempty[b]);
        }
    }
done:
    // peer stores: performed at system scope before the kernel ends, so that the sum
    // kernel's cross-rank release that follows on this stream covers them
    if (a.mode == kEpiPeerBF16) __threadfence_system();
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ---------------------------------------------------------------- host
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

}  // namespace

cudaError_t make_tmap_f16_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                             uint64_t row_stride_bytes, uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    if (((uintptr_t)base & 15) || (row_stride_bytes & 15)) return cudaErrorMisalignedAddress;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {row_stride_bytes};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t make_tmap_f16_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1,
                             uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes,
                             uint32_t box2) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    if (((uintptr_t)base & 15) || (stride1_bytes & 15) || (stride2_bytes & 15))
        return cudaErrorMisalignedAddress;
    const cuuint64_t dims[3] = {d0, d1, d2};
    const cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
    const cuuint32_t box[3] = {64, 1, box2};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t launch_q4_repack(const uint8_t* src_a, const uint8_t* src_b, bool pair, int N, int K,
                             uint8_t* dst, cudaStream_t stream) {
    const int n_rows = q4_n_tiles(N) * kQ4TileN;
    const int kblocks = q4_k_tiles(K) * 2;
    const long total = (long)n_rows * kblocks;
    const int threads = 256;
    q4_repack_kernel<<<(unsigned)((total + threads - 1) / threads), threads, 0, stream>>>(
        src_a, src_b, pair ? 1 : 0, N, K, dst, n_rows, kblocks);
    return cudaGetLastError();
}

namespace {

__device__ __forceinline__ void red_add_f32(float* p, float v) {
    asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

// ---------------------------------------------------------------- GEMM, weights in TMEM
// Variant for M > 128, plain and residual-add stores: the dequantised weights
// are the A operand straight from tensor memory.  D[128 weight rows][BNT
// activation rows] += W . X^T per tile, tcgen05.mma (M=128, N=BNT, K=16) with
// A = W in TMEM (the dequant thread of weight row i writes its row into TMEM
// lane i with one 32-column tcgen05.st per k step) and B = X from shared
// memory.  The f16 weight tile then never passes through shared memory: per k
// step the SM's shared memory sees the activation tile in (TMA) and out (MMA)
// plus the 4.5 KiB raw tile, against 48 KiB of operand reads and 32 KiB of
// dequantised stores with the weights as the B operand.  8 weight slots of 32
// columns fill the 256 columns after the accumulator(s).
//   warp 0      producer: per k step one input stage (128-row activation
//               boxes by TMA + the raw q4_0 tile by bulk copy, one barrier)
//   warp 1      MMA issue (warp-uniform loop, elected lane)
//   warp 2      TMEM allocation (512 columns)
//   warps 4-7   dequantisation, thread = weight row of the tile = TMEM lane
//   warps 8-15  epilogue out of TMEM in two groups (8-11: the first half of
//               the tile's activation rows, 12-15: the second): thread =
//               weight row, 16 activation rows per tcgen05.ld, coalesced
//               across the warp
// BNT activation rows per tile (the MMA N): 256 with one accumulator, or 128
// with two, so that the epilogue of a tile overlaps the next tile's main loop.
// A pipeline step covers KSUB = 2 k tiles of 64 (k 128): one stage holds the
// activation boxes and the raw q4_0 tiles of both, one weight slot their 64
// dequantised columns, and the MMA warp waits once and commits twice per 16
// MMAs instead of per 8, which halves the per-step barrier round trips that
// leave the tensor pipe idle between steps.  An odd k-tile count ends with a
// one-tile step.
constexpr int KSUB = 2;

template <int BNT>
struct TaCfg {
    static_assert(BNT == 128 || BNT == 256, "activation tile");
    static constexpr int ACC = BNT == 128 ? 2 : 1;      // accumulator buffers
    static constexpr int X2_BYTES = BNT * BK * 2;       // one k tile of 128-row TMA boxes
    static constexpr int IN_BYTES = ((KSUB * (X2_BYTES + kQ4TileBytes)) + 1023) / 1024 * 1024;
    static constexpr int ISTAGES = BNT == 128 ? 5 : 3;
    static constexpr int WSLOTS = (512 - ACC * BNT) / (32 * KSUB);  // TMEM weight slots (4)
    static constexpr uint32_t kColW = ACC * BNT;        // first weight slot column (256)
    static constexpr int kThreads = 512;                 // two epilogue groups (warps 8-11, 12-15)
    static constexpr size_t kSmemBytes = (size_t)ISTAGES * IN_BYTES + 1024 + 512;
    static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

template <int BNT>
__global__ void __launch_bounds__(512, 1)
    q4_gemm_ta_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ Q4GemmArgs a) {
    using C = TaCfg<BNT>;
    constexpr int ACC = C::ACC, X2_BYTES = C::X2_BYTES, IN_BYTES = C::IN_BYTES, ISTAGES = C::ISTAGES;
    constexpr int WSLOTS = C::WSLOTS;
    constexpr uint32_t kColW = C::kColW;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sin = base;                                   // ISTAGES x (X 256 rows | raw tile)
    uint64_t* bars = reinterpret_cast<uint64_t*>(sin + ISTAGES * IN_BYTES);
    uint64_t* ifull = bars;                                // X and raw landed (tx bytes)
    uint64_t* iempty = ifull + ISTAGES;                    // MMA commit + 128 dequant threads
    uint64_t* wfull = iempty + ISTAGES;                    // weight slot written (128 threads)
    uint64_t* wempty = wfull + WSLOTS;                     // MMAs reading the slot done
    uint64_t* afull = wempty + WSLOTS;                     // ACC: accumulator complete
    uint64_t* aempty = afull + ACC;                        // ACC: accumulator drained (128 threads)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(aempty + ACC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KT = (a.K + BK - 1) / BK;                 // k tiles of 64
    const int KS = (KT + KSUB - 1) / KSUB;               // pipeline steps
    const int MT = (a.M + BNT - 1) / BNT;
    const int n_tiles = MT * q4_n_tiles(a.N);
    const int ks0 = a.krot ? (int)((blockIdx.x * 5u) % (unsigned)KS) : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < ISTAGES; ++s) {
            mbar_init(&ifull[s], 1);
            mbar_init(&iempty[s], 1 + kQ4TileN);
        }
        for (int s = 0; s < WSLOTS; ++s) {
            mbar_init(&wfull[s], kQ4TileN);
            mbar_init(&wempty[s], 1);
        }
        for (int b = 0; b < ACC; ++b) {
            mbar_init(&afull[b], 1);
            mbar_init(&aempty[b], 2 * kEpilogueThreads);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 2) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) prefetch_tmap(&tmx);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // producer (warp-uniform; an elected lane issues)
        uint32_t g = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
            const int mt = tile % MT, nt = tile / MT;
            const uint8_t* wt = a.w + (size_t)nt * KT * kQ4TileBytes;
            for (int ks = 0; ks < KS; ++ks, ++g) {
                const int s = g % ISTAGES;
                const bool ok = mbar_wait(&iempty[s], ((g / ISTAGES) & 1) ^ 1, a.err, kErrWaitEmpty, abort_flag);
                if (!__all_sync(0xffffffffu, ok)) goto done;
                const int kj = ks + ks0 < KS ? ks + ks0 : ks + ks0 - KS;
                const int kk = kj * KSUB, nsub = kk + 1 < KT ? KSUB : 1;
                if (elect_one()) {
                    // stage: [k tile kk boxes | k tile kk + 1 boxes | raw tiles kk, kk + 1]
                    uint8_t* st = sin + s * IN_BYTES;
                    mbar_arrive_expect_tx(&ifull[s], nsub * (X2_BYTES + kQ4TileBytes));
                    for (int sub = 0; sub < nsub; ++sub)
#pragma unroll
                        for (int xb = 0; xb < BNT / BM; ++xb)
                            tma_load_2d(st + sub * X2_BYTES + xb * X_BYTES, &tmx, &ifull[s], (kk + sub) * BK,
                                        mt * BNT + xb * BM);
                    bulk_load(st + KSUB * X2_BYTES, wt + (size_t)kk * kQ4TileBytes, nsub * kQ4TileBytes,
                              &ifull[s]);
                }
                __syncwarp();
            }
        }
    } else if (warp == 1) {
        // MMA issue (warp-uniform; an elected lane issues the MMAs and commits)
        const uint32_t idesc = idesc_f16_f32(kQ4TileN, BNT);
        uint32_t g = 0, it = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
            const int b = it % ACC;
            const bool ok = mbar_wait(&aempty[b], ((it / ACC) & 1) ^ 1, a.err, kErrWaitAccEmpty, abort_flag);
            if (!__all_sync(0xffffffffu, ok)) goto done;
            tc_fence_after();
            const uint32_t d = tmem + b * BNT;
            for (int ks = 0; ks < KS; ++ks, ++g) {
                const int s = g % ISTAGES, ws = g % WSLOTS;
                const int kj = ks + ks0 < KS ? ks + ks0 : ks + ks0 - KS;
                const int nsub = kj * KSUB + 1 < KT ? KSUB : 1;
                // wfull implies ifull: the dequantisation threads arrive on
                // wfull[ws] only after they observed ifull[s] (the stage's
                // activation boxes and raw tiles landed) and consumed it, so the
                // acquire on wfull orders the activation reads too
                const bool ready = mbar_wait_hot(&wfull[ws], (g / WSLOTS) & 1, a.err, kErrWaitReady, abort_flag);
                if (!__all_sync(0xffffffffu, ready)) goto done;
                tc_fence_after();
                if (elect_one()) {
                    for (int sub = 0; sub < nsub; ++sub) {
                        const uint64_t bd = desc_kmajor_sw128(smem_u32(sin + s * IN_BYTES + sub * X2_BYTES));
#pragma unroll
                        for (int k = 0; k < BK / 16; ++k)
                            mma_f16_ts(d, tmem + kColW + ws * (32 * KSUB) + sub * 32 + k * 8, bd + 2 * k, idesc,
                                       (ks | sub | k) != 0);
                    }
                    mma_commit(&iempty[s]);
                    mma_commit(&wempty[ws]);
                }
                __syncwarp();
            }
            if (elect_one()) mma_commit(&afull[b]);
            __syncwarp();
        }
    } else if (warp >= 4 && warp < 8) {
        // dequantisation: thread i = weight row i of the tile = TMEM lane i
        const int i = threadIdx.x - 128;
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        uint32_t g = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
            for (int ks = 0; ks < KS; ++ks, ++g) {
                const int s = g % ISTAGES, ws = g % WSLOTS;
                const int kj = ks + ks0 < KS ? ks + ks0 : ks + ks0 - KS;
                const int nsub = kj * KSUB + 1 < KT ? KSUB : 1;
                bool ok = mbar_wait(&ifull[s], (g / ISTAGES) & 1, a.err, kErrWaitFull, abort_flag);
                if (!__all_sync(0xffffffffu, ok)) goto done;
                for (int sub = 0; sub < nsub; ++sub) {
                    uint32_t r[32];  // k 0..63 of the sub tile as 32 f16 pairs (lower k in the low half)
                    dequant_row64(sin + s * IN_BYTES + KSUB * X2_BYTES + sub * kQ4TileBytes, i, r);
                    if (sub == 0) {  // dequantise first: only the TMEM store waits for the slot
                        ok = mbar_wait(&wempty[ws], ((g / WSLOTS) & 1) ^ 1, a.err, kErrWaitWEmpty, abort_flag);
                        if (!__all_sync(0xffffffffu, ok)) goto done;
                        tc_fence_after();
                    }
                    tmem_st_32x32b_x32(tmem + lane_base + kColW + ws * (32 * KSUB) + sub * 32, r);
                }
                // the input slot is released once the raw values were consumed
                mbar_arrive(&iempty[s]);
                tmem_st_wait();
                tc_fence_before();
                mbar_arrive(&wfull[ws]);
            }
        }
    } else if (warp >= 8) {
        // epilogue, two groups (warps 8-11 and 12-15) of one thread per weight
        // row (TMEM lane), each draining half of the tile's activation rows
        const int q = warp & 3;
        const int c0 = warp >= 12 ? BNT / 32 : 0;
        const int l = q * 32 + lane;  // weight row within the tile
        const uint32_t lane_base = (uint32_t)(q * 32) << 16;
        uint32_t it = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
            const int mt = tile % MT, nt = tile / MT;
            const int b = it % ACC;
            const bool ok = mbar_wait(&afull[b], (it / ACC) & 1, a.err, kErrWaitAccum, abort_flag);
            if (!__all_sync(0xffffffffu, ok)) goto done;
            tc_fence_after();
#pragma unroll 1
            for (int c = c0; c < c0 + BNT / 32; ++c) {
                uint32_t v[16];
                tmem_ld_32x32b_x16(tmem + lane_base + b * BNT + c * 16, v);
                tmem_ld_wait();
                const int m0 = mt * BNT + c * 16;
                const int mcount = a.M - m0 < 16 ? a.M - m0 : 16;  // rows of this chunk that exist
                const int n = nt * kQ4TileN + l;
                if (n < a.N && mcount > 0) {
                    if (a.mode == kEpiStoreF32 || a.mode == kEpiAddF32) {
                        float* p = static_cast<float*>(a.y) + (size_t)m0 * a.ldy + n;
                        if (a.mode == kEpiAddF32) {
                            // one reduction per element (no other adder): the same
                            // value as a load-add-store, without waiting on the load
#pragma unroll
                            for (int j = 0; j < 16; ++j, p += a.ldy)
                                if (j < mcount) red_add_f32(p, __uint_as_float(v[j]));
                        } else {
#pragma unroll
                            for (int j = 0; j < 16; ++j, p += a.ldy)
                                if (j < mcount) *p = __uint_as_float(v[j]);
                        }
                    } else if (a.mode == kEpiStoreBF16) {
                        __nv_bfloat16* p = static_cast<__nv_bfloat16*>(a.y) + (size_t)m0 * a.ldy + n;
#pragma unroll
                        for (int j = 0; j < 16; ++j, p += a.ldy)
                            if (j < mcount) *p = __float2bfloat16_rn(__uint_as_float(v[j]));
                    } else if (a.mode == kEpiPeerBF16) {
                        // the owner's receive area, row stride peer_cols (a warp's 32
                        // columns belong to one owner: 64 contiguous bytes per row)
                        const int o = n / a.peer_cols;
                        __nv_bfloat16* p = static_cast<__nv_bfloat16*>(a.peer_y[o]) + (size_t)m0 * a.peer_cols +
                                           (n - o * a.peer_cols);
#pragma unroll
                        for (int j = 0; j < 16; ++j, p += a.peer_cols)
                            if (j < mcount) *p = __float2bfloat16_rn(__uint_as_float(v[j]));
                    } else {
                        __half* p = static_cast<__half*>(a.y) + (size_t)m0 * a.ldy + n;
#pragma unroll
                        for (int j = 0; j < 16; ++j, p += a.ldy)
                            if (j < mcount) *p = __float2half_rn(__uint_as_float(v[j]));
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&aempty[b]);
        }
    }
done:
    // peer stores: performed at system scope before the kernel ends, so that the sum
    // kernel's cross-rank release that follows on this stream covers them
    if (a.mode == kEpiPeerBF16) __threadfence_system();
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------------- SwiGLU GEMM, weights in TMEM
// y[m][j] = f16(silu(gate_j . x_m) * (up_j . x_m)) with both weight rows of output j as
// TMEM A operands in the same lane: per tile 128 outputs x 128 activation rows, two
// accumulators (gate: columns 0..127, up: 128..255) written by two tcgen05.mma
// (M=128, N=128, K=16) per K16 step that share the activation tile.  The pair-repacked
// weight holds outputs 64t..64t+63 of tile t as gate rows 0..63 then up rows 64..127,
// so for output 128u + l the dequant threads of lane l (one for the gate row,
// one for the up row) read row (l & 63), resp. 64 + (l & 63), of tile 2u + (l >> 6).  With both values in one thread the epilogue
// needs no exchange between warps.  The accumulator pair is single-buffered (2 weight
// slots of KSUB x 2 x 32 columns fill the other 256 of the 512 columns).
namespace swi {
constexpr int BNT = 128;                                // activation rows per tile
constexpr int RAW2 = 2 * kQ4TileBytes;                  // the two repacked tiles of 128 outputs
// stage: [k tile kk boxes | k tile kk + 1 boxes | raw tile 2u: kk, kk + 1 | raw tile 2u + 1: kk, kk + 1]
constexpr int IN_BYTES = ((KSUB * (X_BYTES + RAW2)) + 1023) / 1024 * 1024;
constexpr int ISTAGES = 4;
constexpr int WSLOTS = 2;                               // 128 columns each: per k tile gate 32 | up 32
constexpr uint32_t kColUp = 128, kColW = 256;           // up accumulator, first weight slot
constexpr int kThreads = 640;                           // warps 4-7 gate rows, 12-15 up rows,
                                                        // 8-11 and 16-19 the epilogue
constexpr size_t kSmemBytes = (size_t)ISTAGES * IN_BYTES + 1024 + 512;
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
}  // namespace swi

__device__ __forceinline__ float silu_fast(float g) { return __fdividef(g, 1.0f + __expf(-g)); }


__global__ void __launch_bounds__(swi::kThreads, 1)
    q4_gemm_ta_swiglu_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ Q4GemmArgs a) {
    using namespace swi;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sin = base;                                   // ISTAGES x (X 128 rows | 2 raw tiles)
    uint64_t* bars = reinterpret_cast<uint64_t*>(sin + ISTAGES * IN_BYTES);
    uint64_t* ifull = bars;                                // X and raw landed (tx bytes)
    uint64_t* iempty = ifull + ISTAGES;                    // MMA commit + 128 dequant threads
    uint64_t* wfull = iempty + ISTAGES;                    // weight slot pair written (128 threads)
    uint64_t* wempty = wfull + WSLOTS;                     // MMAs reading the slots done
    uint64_t* afull = wempty + WSLOTS;                     // accumulators complete
    uint64_t* aempty = afull + 1;                          // accumulators drained (128 threads)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(aempty + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KT = (a.K + BK - 1) / BK;                 // k tiles of 64
    const int KS = (KT + KSUB - 1) / KSUB;               // pipeline steps
    const int MT = (a.M + BNT - 1) / BNT;
    const int n_tiles = MT * (q4_n_tiles(a.N) / 2);       // 128 outputs per tile
    const int ks0 = a.krot ? (int)((blockIdx.x * 5u) % (unsigned)KS) : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < ISTAGES; ++s) {
            mbar_init(&ifull[s], 1);
            mbar_init(&iempty[s], 1 + 2 * kQ4TileN);
        }
        for (int s = 0; s < WSLOTS; ++s) {
            mbar_init(&wfull[s], 2 * kQ4TileN);
            mbar_init(&wempty[s], 1);
        }
        mbar_init(afull, 1);
        mbar_init(aempty, 2 * kEpilogueThreads);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 2) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    if (warp == 0 && lane == 0) prefetch_tmap(&tmx);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // producer (warp-uniform; an elected lane issues)
        uint32_t g = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
            const int mt = tile % MT, u = tile / MT;
            const uint8_t* wt = a.w + (size_t)(2 * u) * KT * kQ4TileBytes;
            for (int ks = 0; ks < KS; ++ks, ++g) {
                const int s = g % ISTAGES;
                const bool ok = mbar_wait(&iempty[s], ((g / ISTAGES) & 1) ^ 1, a.err, kErrWaitEmpty, abort_flag);
                if (!__all_sync(0xffffffffu, ok)) goto done;
                const int kj = ks + ks0 < KS ? ks + ks0 : ks + ks0 - KS;
                const int kk = kj * KSUB, nsub = kk + 1 < KT ? KSUB : 1;
                if (elect_one()) {
                    uint8_t* st = sin + s * IN_BYTES;
                    mbar_arrive_expect_tx(&ifull[s], nsub * (X_BYTES + RAW2));
                    for (int sub = 0; sub < nsub; ++sub)
                        tma_load_2d(st + sub * X_BYTES, &tmx, &ifull[s], (kk + sub) * BK, mt * BNT);
#pragma unroll
                    for (int sel = 0; sel < 2; ++sel)
                        bulk_load(st + KSUB * X_BYTES + sel * KSUB * kQ4TileBytes,
                                  wt + ((size_t)sel * KT + kk) * kQ4TileBytes, nsub * kQ4TileBytes, &ifull[s]);
                }
                __syncwarp();
            }
        }
    } else if (warp == 1) {
        // MMA issue (warp-uniform; an elected lane issues the MMAs and commits)
        const uint32_t idesc = idesc_f16_f32(kQ4TileN, BNT);
        uint32_t g = 0, it = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
            const bool ok = mbar_wait(aempty, (it & 1) ^ 1, a.err, kErrWaitAccEmpty, abort_flag);
            if (!__all_sync(0xffffffffu, ok)) goto done;
            tc_fence_after();
            for (int ks = 0; ks < KS; ++ks, ++g) {
                const int s = g % ISTAGES, ws = g % WSLOTS;
                const int kj = ks + ks0 < KS ? ks + ks0 : ks + ks0 - KS;
                const int nsub = kj * KSUB + 1 < KT ? KSUB : 1;
                // wfull implies ifull (see q4_gemm_ta_kernel)
                const bool ready = mbar_wait_hot(&wfull[ws], (g / WSLOTS) & 1, a.err, kErrWaitReady, abort_flag);
                if (!__all_sync(0xffffffffu, ready)) goto done;
                tc_fence_after();
                if (elect_one()) {
                    for (int sub = 0; sub < nsub; ++sub) {
                        const uint64_t bd = desc_kmajor_sw128(smem_u32(sin + s * IN_BYTES + sub * X_BYTES));
                        const uint32_t wg = tmem + kColW + ws * 128 + sub * 64;  // gate rows, up rows at +32
#pragma unroll
                        for (int k = 0; k < BK / 16; ++k) {
                            const uint32_t acc = (ks | sub | k) != 0;
                            mma_f16_ts(tmem, wg + k * 8, bd + 2 * k, idesc, acc);
                            mma_f16_ts(tmem + kColUp, wg + 32 + k * 8, bd + 2 * k, idesc, acc);
                        }
                    }
                    mma_commit(&iempty[s]);
                    mma_commit(&wempty[ws]);
                }
                __syncwarp();
            }
            if (elect_one()) mma_commit(afull);
            __syncwarp();
        }
    } else if ((warp >= 4 && warp < 8) || (warp >= 12 && warp < 16)) {
        // dequantisation: warps 4-7 the gate rows, warps 12-15 the up rows; thread
        // l = output 128u + l = TMEM lane l
        const int l = (warp & 3) * 32 + lane;
        const int up = warp >= 12 ? 1 : 0;
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        const int sel = l >> 6, r = (l & 63) + 64 * up;  // row r of repacked tile 2u + sel
        uint32_t g = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
            for (int ks = 0; ks < KS; ++ks, ++g) {
                const int s = g % ISTAGES, ws = g % WSLOTS;
                const int kj = ks + ks0 < KS ? ks + ks0 : ks + ks0 - KS;
                const int nsub = kj * KSUB + 1 < KT ? KSUB : 1;
                bool ok = mbar_wait(&ifull[s], (g / ISTAGES) & 1, a.err, kErrWaitFull, abort_flag);
                if (!__all_sync(0xffffffffu, ok)) goto done;
                const uint8_t* raw = sin + s * IN_BYTES + KSUB * X_BYTES + sel * KSUB * kQ4TileBytes;
                for (int sub = 0; sub < nsub; ++sub) {
                    uint32_t w[32];
                    dequant_row64(raw + sub * kQ4TileBytes, r, w);
                    if (sub == 0) {  // dequantise first: only the TMEM store waits for the slot
                        ok = mbar_wait(&wempty[ws], ((g / WSLOTS) & 1) ^ 1, a.err, kErrWaitWEmpty, abort_flag);
                        if (!__all_sync(0xffffffffu, ok)) goto done;
                        tc_fence_after();
                    }
                    tmem_st_32x32b_x32(tmem + lane_base + kColW + ws * 128 + sub * 64 + 32 * up, w);
                }
                // the input slot is released once the raw values were consumed
                mbar_arrive(&iempty[s]);
                tmem_st_wait();
                tc_fence_before();
                mbar_arrive(&wfull[ws]);
            }
        }
    } else if ((warp >= 8 && warp < 12) || warp >= 16) {
        // epilogue, two groups (warps 8-11 and 16-19) of one thread per output
        // column 128u + l, each draining half of the tile's activation rows,
        // 16 rows per load
        const int q = warp & 3;
        const int c0 = warp >= 16 ? BNT / 32 : 0;
        const int l = q * 32 + lane;
        const uint32_t lane_base = (uint32_t)(q * 32) << 16;
        const int F = a.N / 2;
        uint32_t it = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
            const int mt = tile % MT, u = tile / MT;
            const bool ok = mbar_wait(afull, it & 1, a.err, kErrWaitAccum, abort_flag);
            if (!__all_sync(0xffffffffu, ok)) goto done;
            tc_fence_after();
            const int n = u * 128 + l;
#pragma unroll 1
            for (int c = c0; c < c0 + BNT / 32; ++c) {
                uint32_t gv[16], uv[16];
                tmem_ld_32x32b_x16(tmem + lane_base + c * 16, gv);
                tmem_ld_32x32b_x16(tmem + lane_base + kColUp + c * 16, uv);
                tmem_ld_wait();
                const int m0 = mt * BNT + c * 16;
                const int mcount = a.M - m0 < 16 ? a.M - m0 : 16;
                if (n < F && mcount > 0) {
                    __half* p = static_cast<__half*>(a.y) + (size_t)m0 * a.ldy + n;
#pragma unroll
                    for (int j = 0; j < 16; ++j, p += a.ldy)
                        if (j < mcount)
                            *p = __float2half_rn(silu_fast(__uint_as_float(gv[j])) * __uint_as_float(uv[j]));
                }
            }
            tc_fence_before();
            mbar_arrive(aempty);
        }
    }
done:
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

template <int BNT>
cudaError_t launch_ta(const Q4GemmArgs& a, const CUtensorMap& map, int tiles, int sm_count,
                      cudaStream_t stream) {
    using C = TaCfg<BNT>;
    static SmemAttr attr;
    const cudaError_t attr_err = ensure_smem(attr, q4_gemm_ta_kernel<BNT>, (int)C::kSmemBytes);
    if (attr_err != cudaSuccess) return attr_err;
    const int grid = tiles < sm_count ? tiles : sm_count;
    q4_gemm_ta_kernel<BNT><<<grid, C::kThreads, C::kSmemBytes, stream>>>(map, a);
    return cudaGetLastError();
}

}  // namespace

template <int BN>
cudaError_t launch_width(const Q4GemmArgs& a, const CUtensorMap& map, int tiles, int sm_count,
                         cudaStream_t stream) {
    using C = Cfg<BN>;
    static SmemAttr attr;
    const cudaError_t attr_err = ensure_smem(attr, q4_gemm_kernel<BN>, (int)C::kSmemBytes);
    if (attr_err != cudaSuccess) return attr_err;
    const int grid = tiles < sm_count ? tiles : sm_count;
    q4_gemm_kernel<BN><<<grid, C::kThreads, C::kSmemBytes, stream>>>(map, a);
    return cudaGetLastError();
}

cudaError_t launch_q4_gemm(const Q4GemmArgs& args, const __half* x, int sm_count,
                           cudaStream_t stream) {
    Q4GemmArgs a = args;
    {
        // Staggered k starts spread the CTAs sharing a weight tile over its k range, which
        // helps while the whole activation matrix stays in L2; beyond half the L2 they scatter
        // the CTAs' live activation windows and L2 misses: the config-5 w2 GEMM (M 2048, K 28672,
        // 117 MB of activations) read 4.8 GB from DRAM and took 957 us staggered, 798 us aligned
        // (the K = 8192 GEMMs are ~3 % faster staggered).  VELO_Q4_KROT=0/1 forces either.
        const char* kr = std::getenv("VELO_Q4_KROT");
        const size_t act_bytes = (size_t)a.M * a.K * 2;
        a.krot = kr ? std::atoi(kr) : (act_bytes <= (size_t(64) << 20) ? 1 : 0);
    }
    CUtensorMap map;
    cudaError_t e = make_tmap_f16_2d(&map, x, (uint64_t)a.M, (uint64_t)a.K, (uint64_t)a.K * 2, BM);
    if (e != cudaSuccess) return e;
    // More than 128 activation rows: the kernel with the weights in TMEM
    // (VELO_Q4_GEMM=smem / tmem / tmem128 / tmem256 in the environment forces
    // a kernel and tile width, for comparisons).
    // Plain and residual-add stores take the TMEM-weight kernel with 128- or
    // 256-row activation tiles.
    const char* env = std::getenv("VELO_Q4_GEMM");
    const bool force_smem = env != nullptr && std::strcmp(env, "smem") == 0;
    // SwiGLU: the paired-accumulator kernel (config-3 w1/w3 130 us against 146
    // on the shared-memory-weight kernel; config 5 1830 against 1838)
    if (a.M > BM && !force_smem && a.mode == kEpiSwiGLU) {
        static SmemAttr attr;
        const cudaError_t attr_err = ensure_smem(attr, q4_gemm_ta_swiglu_kernel, (int)swi::kSmemBytes);
        if (attr_err != cudaSuccess) return attr_err;
        const int tiles = ((a.M + swi::BNT - 1) / swi::BNT) * (q4_n_tiles(a.N) / 2);
        const int grid = tiles < sm_count ? tiles : sm_count;
        q4_gemm_ta_swiglu_kernel<<<grid, swi::kThreads, swi::kSmemBytes, stream>>>(map, a);
        return cudaGetLastError();
    }
    if (a.M > BM && !force_smem && a.mode != kEpiSwiGLU) {
        // 256 activation rows per tile unless 128-row tiles (two accumulators;
        // measured at about 0.78 of the time of a 256-row tile on config-3
        // shapes) finish the waves sooner
        const int nq = q4_n_tiles(a.N);
        const int t256 = ((a.M + 255) / 256) * nq, t128 = ((a.M + 127) / 128) * nq;
        const double c256 = (double)((t256 + sm_count - 1) / sm_count);
        const double c128 = 0.78 * (double)((t128 + sm_count - 1) / sm_count);
        bool narrow = c128 < c256;
        if (env != nullptr && std::strcmp(env, "tmem128") == 0) narrow = true;
        if (env != nullptr && std::strcmp(env, "tmem256") == 0) narrow = false;
        return narrow ? launch_ta<128>(a, map, t128, sm_count, stream)
                      : launch_ta<256>(a, map, t256, sm_count, stream);
    }
    // 256-row tiles halve the activation traffic per MMA; 128-row tiles when
    // 256-row ones would leave SMs idle.
    const int mt = (a.M + BM - 1) / BM;
    const int t256 = mt * (q4_n_tiles(a.N) / 2);
    if (t256 >= sm_count) return launch_width<256>(a, map, t256, sm_count, stream);
    return launch_width<128>(a, map, mt * q4_n_tiles(a.N), sm_count, stream);
}

}  // namespace velo
