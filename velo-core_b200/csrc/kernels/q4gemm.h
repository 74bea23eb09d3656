// q4gemm.h -- q4_0 weight repack and the tcgen05 dequant-fused GEMM (q4gemm.cu).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace velo {

// Repacked q4_0 weight: tiles of kQ4TileN weight rows x kQ4TileK elements,
// ordered [n_tile][k_tile], each kQ4TileBytes contiguous bytes:
//   [0, 2048)     block 0 (k 0..31 of the tile) of rows 0..127, 16 B per row
//   [2048, 4096)  block 1 (k 32..63), 16 B per row
//   [4096, 4608)  fp16 scales [row][2] (block 0, block 1)
// Inside a row's 16 bytes, 32-bit word g carries elements 8g..8g+7 of the
// block as nibbles e0 e2 | e4 e6 | e1 e3 | e5 e7 (byte 0 .. byte 3, low nibble
// first), so that two masks and a shift yield f16 pairs in element order.
// Rows past N and blocks past K hold weight 0 (nibble 8, scale 0); the row
// count is padded to a multiple of 256 so a GEMM may take tiles in pairs.
constexpr int kQ4TileN = 128;
constexpr int kQ4TileK = 64;
constexpr int kQ4TileBytes = kQ4TileN * 36;             // 4608
constexpr int kQ4ScaleOff = kQ4TileN * 32;              // 4096
constexpr int kQ4Block1Off = kQ4TileN * 16;             // 2048

__host__ __device__ inline int q4_n_tiles(int N) { return 2 * ((N + 255) / 256); }
__host__ __device__ inline int q4_k_tiles(int K) { return (K + kQ4TileK - 1) / kQ4TileK; }
inline size_t q4_repacked_bytes(int N, int K) {
    return (size_t)q4_n_tiles(N) * q4_k_tiles(K) * kQ4TileBytes;
}

// Repacks GGUF/velo-core q4_0 rows ([rows][K/32] blocks of 18 B: fp16 d then
// 16 bytes, element 2i = low nibble of byte i, 2i+1 = high nibble;
// src/quant.rs:50-64).  pair == false: src_a is [N][K], out row r = src_a row r.
// pair == true (SwiGLU gate/up): src_a, src_b are [N/2][K] each; in out tile t
// rows 0..63 are src_a rows 64t.. and rows 64..127 are src_b rows 64t..
cudaError_t launch_q4_repack(const uint8_t* src_a, const uint8_t* src_b, bool pair, int N, int K,
                             uint8_t* dst, cudaStream_t stream);

enum Q4Epilogue : int {
    kEpiStoreF32 = 0,  // y[m][n] = acc                       (f32)
    kEpiStoreF16 = 1,  // y[m][n] = f16(acc)                  (f16)
    kEpiAddF32 = 2,    // y[m][n] += acc                      (f32, residual stream)
    kEpiSwiGLU = 3,    // y[m][j] = f16(silu(gate) * up)      (f16, pair-repacked weight)
    kEpiStoreBF16 = 4, // y[m][n] = bf16(acc)                 (bf16: tensor-parallel partials)
    // bf16(acc) pushed to the rank that owns output column n: element (m, n) goes to
    // peer_y[o][m * peer_cols + n - o * peer_cols], o = n / peer_cols (the first half of a
    // tensor-parallel sum, fused into the row-split GEMM; peer_y are NVLink peer mappings)
    kEpiPeerBF16 = 5,
};

struct Q4GemmArgs {
    const uint8_t* w;  // repacked weight
    int N, K, M;       // weight rows (pair: 2 x F), reduction length, activation rows
    void* y;           // output, row stride ldy elements
    int ldy;
    int mode;          // Q4Epilogue
    int* err;          // device error word (a barrier wait gave up)
    int krot;          // set by launch_q4_gemm: CTAs start their k loops at staggered offsets
    void* peer_y[8];   // kEpiPeerBF16: per owner rank, its receive area for this rank's rows
    int peer_cols;     // kEpiPeerBF16: output columns per owner (a multiple of 32)
};

// X: f16 [M][K] row-major device buffer (K % 8 == 0, 16-byte aligned base).
// Persistent launch: min(output tiles, sm_count) CTAs.
cudaError_t launch_q4_gemm(const Q4GemmArgs& a, const __half* x, int sm_count,
                           cudaStream_t stream);

// Builds the 2-D TMA descriptor of an f16 [rows][cols] row-major matrix with a
// box of 64 x box_rows elements and 128-byte swizzle.
cudaError_t make_tmap_f16_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                             uint64_t row_stride_bytes, uint32_t box_rows);

// 3-D f16 tensor [d2][d1][d0] (d0 contiguous) with a box of 64 x 1 x box2
// elements and 128-byte swizzle (one 128-byte row per (d1, d2) index).
cudaError_t make_tmap_f16_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1,
                             uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes,
                             uint32_t box2);

}  // namespace velo
