// context.cu -- lifecycle, errors, workspace and the acceptance entry points
// of the C ABI (include/velo_cuda.h).
#include "runtime/context.h"

#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <new>
#include <thread>

#include "kernels/accept.h"
#include "runtime/nccl_dyn.h"

namespace velo {

static thread_local std::string g_last_error;

void set_last_error(const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
}

void clear_last_error() { g_last_error.clear(); }

int32_t fail(int32_t st, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return st;
}

int32_t DeviceBuffer::ensure(size_t need, cudaStream_t stream, bool zero_new) {
    if (need <= bytes) return VELO_OK;
    size_t want = need + need / 4;  // headroom so small growth does not thrash
    if (ptr) {
        VELO_CUDA_TRY(cudaStreamSynchronize(stream));
        VELO_CUDA_TRY(cudaFree(ptr));
        ptr = nullptr;
        bytes = 0;
    }
    VELO_CUDA_TRY(cudaMalloc(&ptr, want));
    if (zero_new) VELO_CUDA_TRY(cudaMemsetAsync(ptr, 0, want, stream));
    bytes = want;
    return VELO_OK;
}

void DeviceBuffer::release() {
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    bytes = 0;
}

}  // namespace velo

namespace velo {

int32_t run_accept(velo_cuda_ctx* c, const float* tgt, const float* drf,
                          const uint32_t* tok, const float* u, int32_t B, int32_t k, int32_t V,
                          float temperature, int32_t* acc, uint32_t* bonus) {
    const bool greedy = temperature == 0.0f;
    int32_t st = c->workspace.ensure(velo::accept_workspace_bytes(B, k, V, greedy), c->stream);
    if (st) return st;
    // ticket block: zeroed when (re)allocated, then kept at zero by the kernel
    st = c->counters.ensure(velo::accept_counter_bytes(B), c->stream, /*zero_new=*/true);
    if (st) return st;
    velo::AcceptParams p{};
    p.tgt = tgt;
    p.drf = drf;
    p.tok = tok;
    p.u = u;
    p.acc_len = acc;
    p.bonus = bonus;
    p.err_flag = c->err_flag;
    p.B = B;
    p.k = k;
    p.V = V;
    p.inv_t = greedy ? 0.0f : 1.0f / temperature;
    p.vec4 = (V % 4 == 0) && ((uintptr_t)tgt % 16 == 0) && (greedy || k == 0 || (uintptr_t)drf % 16 == 0);
    velo::accept_bind_buffers(p, c->workspace.ptr, c->counters.ptr, greedy);
    VELO_CUDA_TRY(velo::launch_accept(p, greedy, c->sm_count, c->stream));
    return VELO_OK;
}

}  // namespace velo

using velo::fail;

extern "C" {

int32_t velo_cuda_abi_version(void) { return VELO_CUDA_ABI_VERSION; }

const char* velo_cuda_last_error(void) { return velo::g_last_error.c_str(); }

int32_t velo_cuda_create(const velo_cuda_config* cfg, int32_t device, int32_t tp_rank,
                         int32_t tp_size, const void* nccl_unique_id, velo_cuda_ctx** out) {
    velo::clear_last_error();
    if (!out) return fail(VELO_ERR_INVALID_ARGUMENT, "velo_cuda_create: out is NULL");
    *out = nullptr;
    if (tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size)
        return fail(VELO_ERR_INVALID_ARGUMENT, "tp_rank %d / tp_size %d invalid", tp_rank, tp_size);
    if (tp_size > 1 && !nccl_unique_id)
        return fail(VELO_ERR_INVALID_ARGUMENT, "tp_size > 1 needs an NCCL unique id");
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(VELO_ERR_NO_DEVICE, "no CUDA device available");
    }
    if (device < 0 || device >= n)
        return fail(VELO_ERR_INVALID_ARGUMENT, "device %d out of range (%d devices)", device, n);
    cudaDeviceProp prop;
    VELO_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        return fail(VELO_ERR_NO_DEVICE, "device %d is sm_%d%d; this build is sm_100a only", device,
                    prop.major, prop.minor);
    velo_cuda_ctx* c = new (std::nothrow) velo_cuda_ctx();
    if (!c) return fail(VELO_ERR_OUT_OF_MEMORY, "host allocation failed");
    c->device = device;
    c->tp_rank = tp_rank;
    c->tp_size = tp_size;
    c->sm_count = prop.multiProcessorCount;
    if (cfg) {
        if (cfg->struct_size != 0 && cfg->struct_size != sizeof(velo_cuda_config)) {
            delete c;
            return fail(VELO_ERR_INVALID_ARGUMENT, "velo_cuda_config.struct_size %u != %zu",
                        cfg->struct_size, sizeof(velo_cuda_config));
        }
        c->cfg = *cfg;
    }
    c->cfg.struct_size = sizeof(velo_cuda_config);
    if (c->cfg.page_size == 0) c->cfg.page_size = 16;
    if (c->cfg.max_slots == 0) c->cfg.max_slots = 1;
    if (c->cfg.max_pages_per_slot == 0) c->cfg.max_pages_per_slot = c->cfg.total_pages;
    if (c->cfg.kv_dtype > VELO_KV_F32) {
        const unsigned kd = c->cfg.kv_dtype;
        delete c;
        return fail(VELO_ERR_INVALID_ARGUMENT, "kv_dtype %u unknown", kd);
    }
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&c->err_flag, sizeof(int));
    if (e == cudaSuccess) e = cudaMallocHost(&c->err_host, sizeof(int));
    if (e == cudaSuccess) *c->err_host = 0;
    if (e == cudaSuccess) e = cudaMemsetAsync(c->err_flag, 0, sizeof(int), c->own_stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->own_stream);
    if (e != cudaSuccess) {
        int32_t st = fail(VELO_ERR_CUDA, "context setup failed: %s", cudaGetErrorString(e));
        velo_cuda_destroy(c);
        return st;
    }
    c->stream = c->own_stream;
    if (tp_size > 1) {
        // tensor-parallel group: every rank calls velo_cuda_create with the
        // same id at the same time (ncclCommInitRank is collective)
        const velo::NcclApi* nc = velo::nccl_api();
        if (!nc) {
            velo_cuda_destroy(c);
            return VELO_ERR_NCCL;
        }
        ncclUniqueId id;
        std::memcpy(&id, nccl_unique_id, sizeof(id));
        ncclComm_t comm = nullptr;
        ncclResult_t r = nc->CommInitRank(&comm, tp_size, id, tp_rank);
        if (r != ncclSuccess) {
            const char* msg = nc->GetErrorString(r);
            velo_cuda_destroy(c);
            return fail(VELO_ERR_NCCL, "ncclCommInitRank(rank %d of %d) failed: %s", tp_rank, tp_size, msg);
        }
        c->nccl_comm = comm;
        // a second communicator over the same ranks (collective, same order
        // on every rank); without ncclCommSplit the steps use one stream
        if (nc->CommSplit) {
            ncclComm_t comm2 = nullptr;
            if (nc->CommSplit(comm, 0, tp_rank, &comm2, nullptr) == ncclSuccess) c->nccl_comm2 = comm2;
        }
    }
    *out = c;
    return VELO_OK;
}

int32_t velo_cuda_nccl_unique_id(void* out) {
    velo::clear_last_error();
    if (!out) return fail(VELO_ERR_INVALID_ARGUMENT, "out is NULL");
    const velo::NcclApi* nc = velo::nccl_api();
    if (!nc) return VELO_ERR_NCCL;
    ncclUniqueId id;
    ncclResult_t r = nc->GetUniqueId(&id);
    if (r != ncclSuccess) return fail(VELO_ERR_NCCL, "ncclGetUniqueId failed: %s", nc->GetErrorString(r));
    std::memcpy(out, &id, sizeof(id));
    return VELO_OK;
}

void velo_cuda_destroy(velo_cuda_ctx* c) {
    if (!c) return;
    cudaSetDevice(c->device);
    if (c->own_stream) cudaStreamSynchronize(c->own_stream);
    if (c->stream && c->stream != c->own_stream) cudaStreamSynchronize(c->stream);
    c->workspace.release();
    c->counters.release();
    c->io.release();
    c->attn_ws.release();
    velo::destroy_model(c->model);
    c->model = nullptr;
    if (c->nccl_comm2) {
        if (const velo::NcclApi* nc = velo::nccl_api()) nc->CommDestroy(static_cast<ncclComm_t>(c->nccl_comm2));
        c->nccl_comm2 = nullptr;
    }
    if (c->nccl_comm) {
        if (const velo::NcclApi* nc = velo::nccl_api()) nc->CommDestroy(static_cast<ncclComm_t>(c->nccl_comm));
        c->nccl_comm = nullptr;
    }
    if (c->err_flag) cudaFree(c->err_flag);
    if (c->err_host) cudaFreeHost(c->err_host);
    if (c->own_stream) cudaStreamDestroy(c->own_stream);
    delete c;
}

int32_t velo_cuda_set_stream(velo_cuda_ctx* c, void* stream) {
    if (!c) return fail(VELO_ERR_INVALID_ARGUMENT, "ctx is NULL");
    c->stream = stream ? (cudaStream_t)stream : c->own_stream;
    return VELO_OK;
}

int32_t velo_cuda_sync(velo_cuda_ctx* c, int64_t timeout_ns) {
    if (!c) return fail(VELO_ERR_INVALID_ARGUMENT, "ctx is NULL");
    cudaSetDevice(c->device);
    // the device error word rides along with the stream's work
    VELO_CUDA_TRY(cudaMemcpyAsync(c->err_host, c->err_flag, sizeof(int), cudaMemcpyDeviceToHost,
                                  c->stream));
    if (timeout_ns < 0) {
        cudaError_t e = cudaStreamSynchronize(c->stream);
        if (e != cudaSuccess) return fail(VELO_ERR_CUDA, "stream error: %s", cudaGetErrorString(e));
    } else {
        // poll: yield for the first 200 us (short steps finish here), then sleep
        const auto start = std::chrono::steady_clock::now();
        for (;;) {
            cudaError_t e = cudaStreamQuery(c->stream);
            if (e == cudaSuccess) break;
            if (e != cudaErrorNotReady)
                return fail(VELO_ERR_CUDA, "stream error: %s", cudaGetErrorString(e));
            auto el = std::chrono::duration_cast<std::chrono::nanoseconds>(
                          std::chrono::steady_clock::now() - start).count();
            if (el > timeout_ns)
                return fail(VELO_ERR_TIMEOUT, "velo_cuda_sync: work still running after %lld ns",
                            (long long)timeout_ns);
            if (el < 200000)
                std::this_thread::yield();
            else
                std::this_thread::sleep_for(std::chrono::microseconds(20));
        }
    }
    const int flag = *c->err_host;
    if (flag) {
        *c->err_host = 0;
        VELO_CUDA_TRY(cudaMemset(c->err_flag, 0, sizeof(int)));
        return fail(VELO_ERR_DEVICE_FLAG, "a kernel flagged invalid input (code %d)", flag);
    }
    return VELO_OK;
}

// ---------------------------------------------------------------- acceptance

static int32_t check_accept_args(int32_t B, int32_t k, int32_t V, float temperature,
                                 const void* tgt, const void* drf, const void* tok,
                                 const void* u, const void* acc, const void* bonus) {
    if (B < 0) return fail(VELO_ERR_INVALID_ARGUMENT, "B = %d < 0", B);
    if (k < 0 || k > velo::kAcceptMaxK)
        return fail(VELO_ERR_INVALID_ARGUMENT, "k = %d outside [0, %d]", k, velo::kAcceptMaxK);
    if (V < 1 || V > velo::kAcceptMaxV)
        return fail(VELO_ERR_INVALID_ARGUMENT, "V = %d outside [1, %d]", V, velo::kAcceptMaxV);
    if (!(temperature >= 0.0f) || std::isinf(temperature))
        return fail(VELO_ERR_INVALID_ARGUMENT, "temperature must be finite and >= 0");
    if (B == 0) return VELO_OK;
    if (!tgt || !acc || !bonus || (k > 0 && !tok))
        return fail(VELO_ERR_INVALID_ARGUMENT, "NULL target_logits / draft_tokens / outputs");
    if (temperature > 0.0f && ((k > 0 && !drf) || !u))
        return fail(VELO_ERR_INVALID_ARGUMENT, "sampling needs draft_logits and uniforms");
    return VELO_OK;
}

int32_t velo_cuda_accept_device(velo_cuda_ctx* c, const float* tgt, const float* drf,
                                const uint32_t* tok, const float* u, int32_t B, int32_t k,
                                int32_t V, float temperature, int32_t* acc, uint32_t* bonus) {
    velo::Range nvtx_range("velo.accept_device");
    velo::clear_last_error();
    if (!c) return fail(VELO_ERR_INVALID_ARGUMENT, "ctx is NULL");
    int32_t st = check_accept_args(B, k, V, temperature, tgt, drf, tok, u, acc, bonus);
    if (st || B == 0) return st;
    VELO_CUDA_TRY(cudaSetDevice(c->device));
    return velo::run_accept(c, tgt, drf, tok, u, B, k, V, temperature, acc, bonus);
}

int32_t velo_cuda_accept(velo_cuda_ctx* c, const float* tgt, const float* drf,
                         const uint32_t* tok, const float* u, int32_t B, int32_t k, int32_t V,
                         float temperature, int32_t* acc, uint32_t* bonus) {
    velo::Range nvtx_range("velo.accept");
    velo::clear_last_error();
    if (!c) return fail(VELO_ERR_INVALID_ARGUMENT, "ctx is NULL");
    int32_t st = check_accept_args(B, k, V, temperature, tgt, drf, tok, u, acc, bonus);
    if (st || B == 0) return st;
    for (size_t i = 0; i < (size_t)B * k; ++i)
        if (tok[i] >= (uint32_t)V)
            return fail(VELO_ERR_INVALID_ARGUMENT, "draft token %u at %zu is >= V = %d", tok[i], i, V);
    VELO_CUDA_TRY(cudaSetDevice(c->device));
    const bool greedy = temperature == 0.0f;
    const size_t n_t = (size_t)B * (k + 1) * V * sizeof(float);
    const size_t n_d = greedy ? 0 : (size_t)B * k * V * sizeof(float);
    const size_t n_tok = (size_t)B * k * sizeof(uint32_t);
    const size_t n_u = greedy ? 0 : (size_t)B * (k + 1) * sizeof(float);
    auto up16 = [](size_t x) { return (x + 255) & ~(size_t)255; };
    const size_t off_d = up16(n_t), off_tok = off_d + up16(n_d), off_u = off_tok + up16(n_tok);
    const size_t off_acc = off_u + up16(n_u), off_bonus = off_acc + up16((size_t)B * 4);
    const size_t total = off_bonus + up16((size_t)B * 4);
    st = c->io.ensure(total, c->stream);
    if (st) return st;
    char* base = (char*)c->io.ptr;
    float* d_t = (float*)base;
    float* d_d = greedy ? nullptr : (float*)(base + off_d);
    uint32_t* d_tok = (uint32_t*)(base + off_tok);
    float* d_u = greedy ? nullptr : (float*)(base + off_u);
    int32_t* d_acc = (int32_t*)(base + off_acc);
    uint32_t* d_bonus = (uint32_t*)(base + off_bonus);
    VELO_CUDA_TRY(cudaMemcpyAsync(d_t, tgt, n_t, cudaMemcpyHostToDevice, c->stream));
    if (n_d) VELO_CUDA_TRY(cudaMemcpyAsync(d_d, drf, n_d, cudaMemcpyHostToDevice, c->stream));
    if (n_tok) VELO_CUDA_TRY(cudaMemcpyAsync(d_tok, tok, n_tok, cudaMemcpyHostToDevice, c->stream));
    if (n_u) VELO_CUDA_TRY(cudaMemcpyAsync(d_u, u, n_u, cudaMemcpyHostToDevice, c->stream));
    st = velo::run_accept(c, d_t, d_d, d_tok, d_u, B, k, V, temperature, d_acc, d_bonus);
    if (st) return st;
    VELO_CUDA_TRY(cudaMemcpyAsync(acc, d_acc, (size_t)B * 4, cudaMemcpyDeviceToHost, c->stream));
    VELO_CUDA_TRY(cudaMemcpyAsync(bonus, d_bonus, (size_t)B * 4, cudaMemcpyDeviceToHost, c->stream));
    return velo_cuda_sync(c, -1);
}

// ---------------------------------------------------------------- tree acceptance

static int32_t check_tree_args(int32_t B, int32_t N, int32_t V, float temperature, const void* tgt,
                               const void* drf, const void* tok, const void* par, const void* u,
                               const void* path, const void* plen, const void* bonus) {
    if (B < 0) return fail(VELO_ERR_INVALID_ARGUMENT, "B = %d < 0", B);
    if (N < 1) return fail(VELO_ERR_EMPTY_DRAFT_WINDOW, "n_nodes = %d: the tree needs its root", N);
    if (N > velo::kAcceptMaxK) return fail(VELO_ERR_DRAFT_TOO_MANY, "n_nodes = %d > %d", N, velo::kAcceptMaxK);
    if (V < 1 || V > velo::kAcceptMaxV)
        return fail(VELO_ERR_INVALID_ARGUMENT, "V = %d outside [1, %d]", V, velo::kAcceptMaxV);
    if (!(temperature > 0.0f) || std::isinf(temperature))
        return fail(VELO_ERR_INVALID_ARGUMENT, "tree sampling needs a finite temperature > 0");
    if (B == 0) return VELO_OK;
    if (!tgt || !tok || !par || !u || !path || !plen || !bonus || (N > 1 && !drf))
        return fail(VELO_ERR_INVALID_ARGUMENT, "NULL input / output buffer");
    return VELO_OK;
}

static int32_t launch_tree(velo_cuda_ctx* c, const float* tgt, const float* drf, const uint32_t* tok,
                           const int32_t* par, const float* u, int32_t B, int32_t N, int32_t V, float temperature,
                           int32_t* path, int32_t* plen, uint32_t* bonus) {
    velo::AcceptTreeParams p{};
    p.tgt = tgt;
    p.drf = drf;
    p.tok = tok;
    p.par = par;
    p.u = u;
    p.path = path;
    p.path_len = plen;
    p.bonus = bonus;
    p.err_flag = c->err_flag;
    p.B = B;
    p.N = N;
    p.V = V;
    p.inv_t = 1.0f / temperature;
    p.vec4 = (V % 4 == 0) && ((uintptr_t)tgt % 16 == 0) && (N == 1 || (uintptr_t)drf % 16 == 0);
    VELO_CUDA_TRY(velo::launch_accept_tree(p, c->stream));
    return VELO_OK;
}

int32_t velo_cuda_accept_tree_device(velo_cuda_ctx* c, const float* tgt, const float* drf,
                                     const uint32_t* tok, const int32_t* par, const float* u, int32_t B,
                                     int32_t N, int32_t V, float temperature, int32_t* path,
                                     int32_t* path_len, uint32_t* bonus) {
    velo::Range nvtx_range("velo.accept_tree_device");
    velo::clear_last_error();
    if (!c) return fail(VELO_ERR_INVALID_ARGUMENT, "ctx is NULL");
    int32_t st = check_tree_args(B, N, V, temperature, tgt, drf, tok, par, u, path, path_len, bonus);
    if (st || B == 0) return st;
    VELO_CUDA_TRY(cudaSetDevice(c->device));
    return launch_tree(c, tgt, drf, tok, par, u, B, N, V, temperature, path, path_len, bonus);
}

int32_t velo_cuda_accept_tree(velo_cuda_ctx* c, const float* tgt, const float* drf, const uint32_t* tok,
                              const int32_t* par, const float* u, int32_t B, int32_t N, int32_t V,
                              float temperature, int32_t* path, int32_t* path_len, uint32_t* bonus) {
    velo::Range nvtx_range("velo.accept_tree");
    velo::clear_last_error();
    if (!c) return fail(VELO_ERR_INVALID_ARGUMENT, "ctx is NULL");
    int32_t st = check_tree_args(B, N, V, temperature, tgt, drf, tok, par, u, path, path_len, bonus);
    if (st || B == 0) return st;
    for (int32_t b = 0; b < B; ++b) {
        if (par[(size_t)b * N] != -1)
            return fail(VELO_ERR_INVALID_ARGUMENT, "node 0 of sequence %d must be the root (parent -1)", b);
        for (int32_t n = 1; n < N; ++n) {
            const int32_t q = par[(size_t)b * N + n];
            if (q < 0 || q >= n) return fail(VELO_ERR_INVALID_ARGUMENT, "parents[%d][%d] = %d", b, n, q);
            if (tok[(size_t)b * N + n] >= (uint32_t)V)
                return fail(VELO_ERR_INVALID_ARGUMENT, "token %u >= V = %d", tok[(size_t)b * N + n], V);
        }
    }
    VELO_CUDA_TRY(cudaSetDevice(c->device));
    const size_t n_t = (size_t)B * N * V * 4, n_d = (size_t)B * (N - 1) * V * 4;
    const size_t n_i = (size_t)B * N * 4;
    auto up = [](size_t x) { return (x + 255) & ~(size_t)255; };
    const size_t o_d = up(n_t), o_tok = o_d + up(n_d), o_par = o_tok + up(n_i), o_u = o_par + up(n_i);
    const size_t o_path = o_u + up(n_i), o_len = o_path + up(n_i), o_bonus = o_len + up((size_t)B * 4);
    st = c->io.ensure(o_bonus + up((size_t)B * 4), c->stream);
    if (st) return st;
    char* base = (char*)c->io.ptr;
    VELO_CUDA_TRY(cudaMemcpyAsync(base, tgt, n_t, cudaMemcpyHostToDevice, c->stream));
    if (n_d) VELO_CUDA_TRY(cudaMemcpyAsync(base + o_d, drf, n_d, cudaMemcpyHostToDevice, c->stream));
    VELO_CUDA_TRY(cudaMemcpyAsync(base + o_tok, tok, n_i, cudaMemcpyHostToDevice, c->stream));
    VELO_CUDA_TRY(cudaMemcpyAsync(base + o_par, par, n_i, cudaMemcpyHostToDevice, c->stream));
    VELO_CUDA_TRY(cudaMemcpyAsync(base + o_u, u, n_i, cudaMemcpyHostToDevice, c->stream));
    st = launch_tree(c, (const float*)base, (const float*)(base + o_d), (const uint32_t*)(base + o_tok),
                     (const int32_t*)(base + o_par), (const float*)(base + o_u), B, N, V, temperature,
                     (int32_t*)(base + o_path), (int32_t*)(base + o_len), (uint32_t*)(base + o_bonus));
    if (st) return st;
    VELO_CUDA_TRY(cudaMemcpyAsync(path, base + o_path, n_i, cudaMemcpyDeviceToHost, c->stream));
    VELO_CUDA_TRY(cudaMemcpyAsync(path_len, base + o_len, (size_t)B * 4, cudaMemcpyDeviceToHost, c->stream));
    VELO_CUDA_TRY(cudaMemcpyAsync(bonus, base + o_bonus, (size_t)B * 4, cudaMemcpyDeviceToHost, c->stream));
    return velo_cuda_sync(c, -1);
}

}  // extern "C"
