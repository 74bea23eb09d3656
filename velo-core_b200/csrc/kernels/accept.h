// accept.h -- launch interface of the fused acceptance kernel (accept.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace velo {

constexpr int kAcceptMaxK = 64;                     // draft positions per sequence
constexpr int kAcceptMaxRows = 2 * kAcceptMaxK + 1; // target k+1 rows + draft k rows
constexpr int kAcceptMaxTiles = 256;                // vocabulary <= 256 * 1024
constexpr int kAcceptMaxV = kAcceptMaxTiles * 1024;

struct AcceptParams {
    const float* tgt;       // [B][k+1][V]
    const float* drf;       // [B][k][V] (sampling only)
    const uint32_t* tok;    // [B][k]
    const float* u;         // [B][k+1]
    int32_t* acc_len;       // [B]
    uint32_t* bonus;        // [B]
    float2* part;           // workspace: [B][nrows][ntiles] tile statistics
    unsigned* counters;     // [B] completion tickets, zero between launches
    int* err_flag;          // device flag: bad draft token seen
    int B, k, V;
    float inv_t;
    bool vec4;              // rows are 16-byte aligned (V % 4 == 0, aligned bases)
    // filled by launch_accept
    int ntiles, nrows, ctas_per_seq;
};

// Bytes of the tile-statistics workspace for one launch.
size_t accept_workspace_bytes(int B, int k, int V, bool greedy);

cudaError_t launch_accept(const AcceptParams& p, bool greedy, cudaStream_t stream);

}  // namespace velo
