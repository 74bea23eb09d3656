// q4gemm.cu -- q4_0 weights x f16 activations on the sm_100a tensor cores.
//
// Replaces the per-token, per-row `matvec_quant` of the reference CPU path
// (src/llama_cpu.rs:75-90, dequant_row src/quant.rs:50-73) for the verify
// step, where all drafted tokens of all sequences form the M side of one GEMM:
//   Y[m][n] = sum_k X[m][k] * W[n][k],   W = q4_0 dequantised (d * (q - 8)).
//
// One CTA computes a 128 (activation rows) x 256 (weight rows) tile with the
// accumulator in tensor memory:
//   warp 0      TMA producer: X tile (64 k, 128-byte swizzle) + the raw q4_0
//               tile (one 9216-byte bulk copy) per k step into a 3-stage ring
//   warp 1      one thread issues tcgen05.mma (M=128, N=256, K=16) x 4 per stage
//   warp 2      allocates / frees 256 TMEM columns
//   warps 4-11  dequantise their weight row of each stage into the swizzled
//               f16 operand tile, then run the fused epilogue out of TMEM
// Dequantisation: the nibble order chosen at repack time turns a 32-bit word
// into f16 pairs with one LOP3 each (0x6400 | q = 1024 + q), an exact subtract
// (or exact FMA for the high nibbles) gives q - 8, and one HMUL2 by the block
// scale rounds d * (q - 8) once to f16.
#include <cuda.h>
#include <cuda_fp16.h>

#include <mutex>

#include "common/sm100.cuh"
#include "kernels/q4gemm.h"

namespace velo {
namespace {

using namespace sm100;

constexpr int BM = 128, BN = kQ4TileN, BK = kQ4TileK, STAGES = 3;
constexpr int X_BYTES = BM * BK * 2;      // 16 KiB
constexpr int W_BYTES = BN * BK * 2;      // 32 KiB
constexpr int RAW_BYTES = kQ4TileBytes;   // 9 KiB
constexpr int kThreads = 384;
constexpr int kDequantThreads = 256;      // warps 4..11, one weight row each
constexpr int kTmemCols = 256;
constexpr size_t kSmemBytes = (size_t)STAGES * (X_BYTES + W_BYTES + RAW_BYTES) + 1024 + 256;

// error codes written to Q4GemmArgs::err when a wait gives up
constexpr int kErrWaitEmpty = 0x4101, kErrWaitReady = 0x4102, kErrWaitFull = 0x4103,
              kErrWaitAccum = 0x4104;

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
    *reinterpret_cast<uint4*>(tile + (kb & 1) * 4096 + l * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint16_t*>(tile + 8192 + l * 4 + (kb & 1) * 2) = d;
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

// ---------------------------------------------------------------- epilogue
__device__ __forceinline__ void store_row32(const Q4GemmArgs& a, int m, int n, const uint32_t (&r)[32]) {
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
__global__ void __launch_bounds__(kThreads, 1)
    q4_gemm_kernel(const __grid_constant__ CUtensorMap tmx, const Q4GemmArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* sx = base;
    uint8_t* sw = sx + STAGES * X_BYTES;
    uint8_t* sr = sw + STAGES * W_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sr + STAGES * RAW_BYTES);
    uint64_t* full = bars;
    uint64_t* wready = bars + STAGES;
    uint64_t* empty = bars + 2 * STAGES;
    uint64_t* accum = bars + 3 * STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * STAGES + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * BM;
    const int nt = blockIdx.y;
    const int KT = (a.K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&wready[s], kDequantThreads);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accum, 1);
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
        if (lane == 0) {
            const uint8_t* wt = a.w + (size_t)nt * KT * RAW_BYTES;
            for (int kt = 0; kt < KT; ++kt) {
                const int s = kt % STAGES;
                const uint32_t ph = (kt / STAGES) & 1;
                if (!mbar_wait(&empty[s], ph ^ 1, a.err, kErrWaitEmpty, abort_flag)) break;
                mbar_arrive_expect_tx(&full[s], X_BYTES + RAW_BYTES);
                tma_load_2d(sx + s * X_BYTES, &tmx, &full[s], kt * BK, m0);
                bulk_load(sr + s * RAW_BYTES, wt + (size_t)kt * RAW_BYTES, RAW_BYTES, &full[s]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = idesc_f16_f32(BM, BN);
            bool ok = true;
            for (int kt = 0; kt < KT; ++kt) {
                const int s = kt % STAGES;
                const uint32_t ph = (kt / STAGES) & 1;
                if (!mbar_wait(&wready[s], ph, a.err, kErrWaitReady, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint64_t ad = desc_kmajor_sw128(smem_u32(sx + s * X_BYTES));
                const uint64_t bd = desc_kmajor_sw128(smem_u32(sw + s * W_BYTES));
#pragma unroll
                for (int k = 0; k < BK / 16; ++k)
                    mma_f16_ss(tmem, ad + 2 * k, bd + 2 * k, idesc, (kt | k) != 0);
                mma_commit(&empty[s]);
            }
            if (ok) mma_commit(accum);
        }
    } else if (warp >= 4) {
        const int i = threadIdx.x - 128;  // weight row within the tile
        uint8_t* wrow_base = sw + (i >> 3) * 1024 + (i & 7) * 128;
        const int sx7 = i & 7;
        bool ok = true;
        for (int kt = 0; kt < KT; ++kt) {
            const int s = kt % STAGES;
            const uint32_t ph = (kt / STAGES) & 1;
            if (!mbar_wait(&full[s], ph, a.err, kErrWaitFull, abort_flag)) {
                ok = false;
                break;
            }
            const uint8_t* raw = sr + s * RAW_BYTES;
            const uint4 c0 = *reinterpret_cast<const uint4*>(raw + i * 16);
            const uint4 c1 = *reinterpret_cast<const uint4*>(raw + 4096 + i * 16);
            const uint32_t sc = *reinterpret_cast<const uint32_t*>(raw + 8192 + i * 4);
            const __half2 d0 = __half2half2(__ushort_as_half((uint16_t)(sc & 0xFFFF)));
            const __half2 d1 = __half2half2(__ushort_as_half((uint16_t)(sc >> 16)));
            uint8_t* wrow = wrow_base + s * W_BYTES;
            const uint32_t w0[4] = {c0.x, c0.y, c0.z, c0.w};
            const uint32_t w1[4] = {c1.x, c1.y, c1.z, c1.w};
#pragma unroll
            for (int g = 0; g < 4; ++g)
                *reinterpret_cast<uint4*>(wrow + ((g ^ sx7) << 4)) = dequant8(w0[g], d0);
#pragma unroll
            for (int g = 0; g < 4; ++g)
                *reinterpret_cast<uint4*>(wrow + (((4 + g) ^ sx7) << 4)) = dequant8(w1[g], d1);
            fence_async_smem();
            mbar_arrive(&wready[s]);
        }
        if (ok) ok = mbar_wait(accum, 0, a.err, kErrWaitAccum, abort_flag);
        __syncwarp();
        if (__all_sync(0xffffffffu, ok)) {
            tc_fence_after();
            const int q = warp & 3, h = (warp - 4) >> 2;
            const int m = m0 + q * 32 + lane;
            const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
            if (a.mode != kEpiSwiGLU) {
#pragma unroll 1
                for (int j = 0; j < 4; ++j) {
                    const int col = h * 128 + j * 32;
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(trow + col, r);
                    tmem_ld_wait();
                    const int n = nt * BN + col;
                    if (m < a.M && n < a.N) store_row32(a, m, n, r);
                }
            } else {
                const int F = a.N / 2;
#pragma unroll 1
                for (int j = 0; j < 2; ++j) {
                    const int col = h * 64 + j * 32;
                    uint32_t g[32], u[32];
                    tmem_ld_32x32b_x32(trow + col, g);
                    tmem_ld_32x32b_x32(trow + BN / 2 + col, u);
                    tmem_ld_wait();
                    const int n = nt * (BN / 2) + col;
                    if (m < a.M && n < F) {
                        __half* y = static_cast<__half*>(a.y) + (size_t)m * a.ldy + n;
#pragma unroll
                        for (int e = 0; e < 32; e += 2) {
                            if (n + e >= F) break;
                            const float v0 = silu(__uint_as_float(g[e])) * __uint_as_float(u[e]);
                            const float v1 = silu(__uint_as_float(g[e + 1])) * __uint_as_float(u[e + 1]);
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
        }
    }
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

cudaError_t launch_q4_gemm(const Q4GemmArgs& a, const __half* x, cudaStream_t stream) {
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(once, [] {
        attr_err = cudaFuncSetAttribute(q4_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)kSmemBytes);
    });
    if (attr_err != cudaSuccess) return attr_err;
    CUtensorMap map;
    cudaError_t e = make_tmap_f16_2d(&map, x, (uint64_t)a.M, (uint64_t)a.K, (uint64_t)a.K * 2, BM);
    if (e != cudaSuccess) return e;
    dim3 grid((a.M + BM - 1) / BM, q4_n_tiles(a.N));
    q4_gemm_kernel<<<grid, kThreads, kSmemBytes, stream>>>(map, a);
    return cudaGetLastError();
}

}  // namespace velo
