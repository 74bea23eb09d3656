// accept.h -- launch interface of the fused acceptance kernels (accept.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace velo {

constexpr int kAcceptMaxK = 64;                     // draft positions per sequence
constexpr int kAcceptMaxRows = 2 * kAcceptMaxK + 1; // target k+1 rows + draft k rows
constexpr int kAcceptMaxTiles = 128;                // vocabulary <= 128 * 1024
constexpr int kAcceptMaxV = kAcceptMaxTiles * 1024;

struct AcceptParams {
    const float* tgt;       // [B][k+1][V]
    const float* drf;       // [B][k][V] (sampling only)
    const uint32_t* tok;    // [B][k]
    const float* u;         // [B][k+1]
    int32_t* acc_len;       // [B]
    uint32_t* bonus;        // [B]
    // workspace (per launch; contents need no initialisation)
    float2* part;           // [B][nrows][ntiles] tile statistics
    float* tokval;          // [B][nrows] logit of row i at its draft token (rows != k)
    float* lane_w;          // [B][ntiles][32] draw lane weights
    float* tile_w;          // [B][ntiles] draw tile weights
    // per-sequence ticket of the finish CTAs; zeroed at allocation, reset by
    // the CTA that takes the last ticket, so it is zero between launches
    unsigned* done;         // [B]
    int* err_flag;          // device flag: bad draft token seen
    int B, k, V;
    float inv_t;
    bool vec4;              // rows are 16-byte aligned (V % 4 == 0, aligned bases)
    int grid;               // stream CTAs (0: 4 per SM)
    // filled by launch_accept
    int ntiles, nrows;
};

// Bytes of the per-launch workspace.
size_t accept_workspace_bytes(int B, int k, int V, bool greedy);
// Bytes of the ticket block (must be zero before the first launch).
size_t accept_counter_bytes(int B);
// Carve `ws` (workspace) and `cnt` (tickets) into the params' pointers.
void accept_bind_buffers(AcceptParams& p, void* ws, void* cnt, bool greedy);

cudaError_t launch_accept(const AcceptParams& p, bool greedy, int sm_count, cudaStream_t stream);

// Rejection sampling over draft trees (sampling only, temperature > 0).
struct AcceptTreeParams {
    const float* tgt;       // [B][N][V]: row n = target logits after node n
    const float* drf;       // [B][N-1][V]: row n = draft distribution of node n's children
    const uint32_t* tok;    // [B][N], node 0 = the root (its token is not tested)
    const int32_t* par;     // [B][N], -1 for node 0, parents[n] < n
    const float* u;         // [B][N]: u[c-1] tests child c, u[N-1] draws the bonus
    int32_t* path;          // [B][N] out: accepted nodes, root first, -1 padded
    int32_t* path_len;      // [B] out: nodes on the path (root included)
    uint32_t* bonus;        // [B] out
    int* err_flag;          // device flag: a token >= V (counted as a rejection)
    int B, N, V;
    float inv_t;
    bool vec4;              // rows are 16-byte aligned
};
cudaError_t launch_accept_tree(const AcceptTreeParams& p, cudaStream_t stream);

}  // namespace velo
