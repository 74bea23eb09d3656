// context.h -- internal definition of velo_cuda_ctx and runtime helpers.
#pragma once
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstddef>
#include <cstdint>
#include <string>

#include <nvtx3/nvToolsExt.h>

#include "velo_cuda.h"

namespace velo {

// NVTX range over a scope (header-only NVTX v3: a no-op unless a profiler
// is attached), so a timeline shows each C ABI call and its phases.
struct Range {
    explicit Range(const char* name) { nvtxRangePushA(name); }
    ~Range() { nvtxRangePop(); }
    Range(const Range&) = delete;
    Range& operator=(const Range&) = delete;
};

// Thread-local last-error message (velo_cuda_last_error).
void set_last_error(const char* fmt, ...);
void clear_last_error();

// Records a message and returns `st`.
int32_t fail(int32_t st, const char* fmt, ...);

// CUDA error -> VELO_ERR_CUDA with the call site.
#define VELO_CUDA_TRY(expr)                                                              \
    do {                                                                                 \
        cudaError_t _e = (expr);                                                         \
        if (_e != cudaSuccess)                                                           \
            return ::velo::fail(_e == cudaErrorMemoryAllocation ? VELO_ERR_OUT_OF_MEMORY \
                                                                : VELO_ERR_CUDA,         \
                                "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e),  \
                                __FILE__, __LINE__);                                     \
    } while (0)

// A device buffer that only grows.  Growing waits for `stream` first.
struct DeviceBuffer {
    void* ptr = nullptr;
    size_t bytes = 0;
    int32_t ensure(size_t need, cudaStream_t stream, bool zero_new = false);
    void release();
};

}  // namespace velo

struct velo_cuda_ctx;
namespace velo {
struct Model;
// Device-buffer acceptance on the context stream (velo_cuda_accept_device
// without the argument checks).
int32_t run_accept(velo_cuda_ctx* c, const float* tgt, const float* drf, const uint32_t* tok,
                   const float* u, int32_t B, int32_t k, int32_t V, float temperature,
                   int32_t* acc, uint32_t* bonus);
void destroy_model(Model* m);
}  // namespace velo

struct velo_cuda_ctx {
    int device = 0;
    int tp_rank = 0, tp_size = 1;
    velo_cuda_config cfg{};
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    int sm_count = 0;

    velo::DeviceBuffer workspace;  // per-launch scratch (tile statistics, partials)
    velo::DeviceBuffer counters;   // completion tickets, zero between launches
    velo::DeviceBuffer io;         // device copies for the host-buffer entries
    velo::DeviceBuffer attn_ws;    // tree attention: ancestor masks
    int* err_flag = nullptr;       // device-side input flag
    int* err_host = nullptr;       // pinned host copy of err_flag (read at sync)
    velo::Model* model = nullptr;  // weights, KV pool and verify buffers (velo_cuda_load_model)
    void* nccl_comm = nullptr;     // ncclComm_t of the tensor-parallel group (tp_size > 1)
    void* nccl_comm2 = nullptr;    // a second communicator of the group (ncclCommSplit), so
                                   // two halves of a batch reduce on two streams at once
};
