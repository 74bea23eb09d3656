// accept_static.cu -- velo_cuda_accept_static: the acceptance step for
// callers that must not allocate device memory.
//
// Some hosts of this library cannot call cudaMalloc on the verify path: a
// serving engine that carves all of HBM into its own pools at start-up and
// forbids further allocations, code that runs while another component holds
// the allocator, or latency-critical loops where cudaMalloc / cudaFree would
// synchronise the device.  This entry point takes only caller-provided input
// and output buffers and keeps its intermediate statistics in a fixed block of
// device memory that is part of the loaded library itself.
//
// The scratch block is a file-scope `__device__` array of kStaticScratchBytes
// (4 MiB).  Every GPU that loads the library holds one copy of it until the
// process exits.  Host code cannot use the array's name as a device address
// (in host code it names a host-side stand-in), so the device address is
// looked up once per device with cudaGetSymbolAddress, with that device
// current, on the first call made on that device; make that first call before
// any stream capture.  All calls on a device share the one block, and it keeps
// the contents of the last call: calls whose work overlaps on the GPU (two
// streams, or two host threads) race on it and must be serialised by the
// caller.  The completion tickets that must start at zero, and the error word,
// are cleared on the caller's stream before each launch.
//
// The error word sits at a fixed place (the last 256 bytes of the block): a
// draft token >= V is counted as a rejection and raises it, and
// velo_cuda_accept_static_error copies it out, so a caller that cannot trust
// its tokens can check each call without a context.  The block's address is
// kept for the life of the process: do not use these entry points after a
// cudaDeviceReset.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <mutex>

#include "kernels/accept.h"
#include "runtime/context.h"

namespace velo {
namespace {

constexpr size_t kStaticScratchBytes = size_t(4) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_accept_scratch[kStaticScratchBytes];

std::mutex g_setup_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_accept_scratch on the current device (looked up once).
int32_t scratch_address(int device, void** out) {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch_addr[device]) {
        void* ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_accept_scratch);
        if (e != cudaSuccess || !ptr)
            return fail(VELO_ERR_CUDA, "cudaGetSymbolAddress(g_accept_scratch) failed: %s",
                        cudaGetErrorString(e));
        g_scratch_addr[device] = ptr;
    }
    *out = g_scratch_addr[device];
    return VELO_OK;
}

size_t up256(size_t x) { return (x + 255) & ~(size_t)255; }

constexpr size_t kErrWordOffset = kStaticScratchBytes - 256;  // the error word's place

int32_t current_block(char** base) {
    int device = 0;
    VELO_CUDA_TRY(cudaGetDevice(&device));
    if (device < 0 || device >= kMaxDevices) return fail(VELO_ERR_INVALID_ARGUMENT, "device %d unsupported", device);
    void* p = nullptr;
    const int32_t st = scratch_address(device, &p);
    *base = static_cast<char*>(p);
    return st;
}

}  // namespace
}  // namespace velo

using velo::fail;

extern "C" int32_t velo_cuda_accept_static(const float* target_logits, const float* draft_logits,
                                           const uint32_t* draft_tokens, const float* uniforms,
                                           int32_t B, int32_t k, int32_t V, float temperature,
                                           int32_t* accepted_len, uint32_t* bonus_token,
                                           void* stream) {
    velo::clear_last_error();
    if (B < 0) return fail(VELO_ERR_INVALID_ARGUMENT, "B = %d < 0", B);
    if (k < 0 || k > velo::kAcceptMaxK)
        return fail(VELO_ERR_INVALID_ARGUMENT, "k = %d outside [0, %d]", k, velo::kAcceptMaxK);
    if (V < 1 || V > velo::kAcceptMaxV)
        return fail(VELO_ERR_INVALID_ARGUMENT, "V = %d outside [1, %d]", V, velo::kAcceptMaxV);
    if (!(temperature >= 0.0f) || std::isinf(temperature))
        return fail(VELO_ERR_INVALID_ARGUMENT, "temperature must be finite and >= 0");
    if (B == 0) return VELO_OK;
    const bool greedy = temperature == 0.0f;
    if (!target_logits || !accepted_len || !bonus_token || (k > 0 && !draft_tokens))
        return fail(VELO_ERR_INVALID_ARGUMENT, "NULL target_logits / draft_tokens / outputs");
    if (!greedy && ((k > 0 && !draft_logits) || !uniforms))
        return fail(VELO_ERR_INVALID_ARGUMENT, "sampling needs draft_logits and uniforms");

    // scratch layout: [workspace | tickets | ... | error word (last 256 bytes)]
    const size_t ws = velo::up256(velo::accept_workspace_bytes(B, k, V, greedy));
    const size_t tk = velo::up256(velo::accept_counter_bytes(B));
    const size_t need = ws + tk + 256;
    if (need > velo::kStaticScratchBytes)
        return fail(VELO_ERR_INVALID_ARGUMENT,
                    "velo_cuda_accept_static: B=%d k=%d V=%d needs %zu bytes of scratch, more than "
                    "the fixed %zu; use velo_cuda_accept_device",
                    B, k, V, need, velo::kStaticScratchBytes);

    int device = 0;
    VELO_CUDA_TRY(cudaGetDevice(&device));
    if (device < 0 || device >= velo::kMaxDevices)
        return fail(VELO_ERR_INVALID_ARGUMENT, "device %d unsupported", device);
    int sm_count = 0;
    VELO_CUDA_TRY(cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, device));
    void* base = nullptr;
    int32_t st = velo::scratch_address(device, &base);
    if (st) return st;

    cudaStream_t s = (cudaStream_t)stream;
    char* b = (char*)base;
    // tickets and the error word must be zero at launch; clearing them is a
    // memset, not an allocation
    VELO_CUDA_TRY(cudaMemsetAsync(b + ws, 0, tk, s));
    VELO_CUDA_TRY(cudaMemsetAsync(b + velo::kErrWordOffset, 0, sizeof(int), s));

    velo::AcceptParams p{};
    p.tgt = target_logits;
    p.drf = draft_logits;
    p.tok = draft_tokens;
    p.u = uniforms;
    p.acc_len = accepted_len;
    p.bonus = bonus_token;
    p.err_flag = (int*)(b + velo::kErrWordOffset);
    p.B = B;
    p.k = k;
    p.V = V;
    p.inv_t = greedy ? 0.0f : 1.0f / temperature;
    p.vec4 = (V % 4 == 0) && ((uintptr_t)target_logits % 16 == 0) &&
             (greedy || k == 0 || (uintptr_t)draft_logits % 16 == 0);
    velo::accept_bind_buffers(p, b, b + ws, greedy);
    VELO_CUDA_TRY(velo::launch_accept(p, greedy, sm_count, s));
    return VELO_OK;
}

extern "C" int32_t velo_cuda_accept_static_error(int32_t* flag_out, void* stream) {
    velo::clear_last_error();
    if (!flag_out) return fail(VELO_ERR_INVALID_ARGUMENT, "flag_out is NULL");
    char* b = nullptr;
    const int32_t st = velo::current_block(&b);
    if (st) return st;
    VELO_CUDA_TRY(cudaMemcpyAsync(flag_out, b + velo::kErrWordOffset, sizeof(int32_t),
                                  cudaMemcpyDeviceToDevice, (cudaStream_t)stream));
    return VELO_OK;
}
