// model.cu -- the target model on the device and the verify step of the C ABI
// (include/velo_cuda.h): weight upload / repack, the paged KV pool and page
// table, and the per-step launch sequence
//   embed -> L x [rmsnorm -> QKV GEMM -> RoPE + split -> tree attention ->
//   o_proj GEMM (+residual) -> rmsnorm -> w1/w3 GEMM (SwiGLU) -> w2 GEMM
//   (+residual)] -> rmsnorm -> LM head GEMM -> acceptance -> KV commit,
// all on the context stream.  The per-token loop of the reference
// (LlamaCpuModel::forward_one, src/llama_cpu.rs:191-358, called k times by
// verify_logits :401-419) becomes one pass over all B x N tree nodes.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "kernels/accept.h"
#include "kernels/f32_path.h"
#include "kernels/q4gemm.h"
#include "kernels/tp_allreduce.h"
#include "kernels/tree_attn.h"
#include "kernels/verify_ops.h"
#include "runtime/context.h"
#include "runtime/nccl_dyn.h"
#include "runtime/page_alloc.h"
#include "runtime/shard.h"

#include <deque>

namespace velo {

// Matrices are repacked q4_0 (the tensor-core path) or, on the fp32 path, f32
// rows (cast from the same pointers).
struct Layer {
    uint8_t* wqkv = nullptr;  // [(Hq + 2 Hkv) D][H]
    uint8_t* wo = nullptr;    // [H][Hq D]
    uint8_t* w13 = nullptr;   // SwiGLU pair [2F][H] (f32: w1 rows, then w3 rows)
    uint8_t* w2 = nullptr;    // [H][F]
    float* attn_norm = nullptr;
    float* ffn_norm = nullptr;
};

struct Model {
    velo_model_desc meta{};    // head / kv-head / ffn counts of this rank's shard
    int tp = 1, rank = 0;      // tensor-parallel position
    // fp32 path (f32 KV pool): weights dequantised to f32 at load (dequant_row,
    // quant.rs:181-191) and every op in f32 on the CUDA cores, the precision of
    // LlamaCpuModel; otherwise q4_0 weights on the tensor cores, f16 / int8 pages
    bool f32 = false;
    int D = 128;               // head_dim
    int V_loc = 0, v_ofs = 0;  // this rank's vocabulary shard of the LM head
    float* emb = nullptr;      // [V][H] f32
    float* out_norm = nullptr; // [H]
    uint8_t* lm_head = nullptr;
    std::vector<Layer> layers;
    std::vector<void*> allocs;
    // KV pool [L][pages][Hkv][16][D] and page table [slots][max_pages]
    void* k_pool = nullptr;
    void* v_pool = nullptr;
    __half* k_scale = nullptr;
    __half* v_scale = nullptr;
    int pool_pages = 0, kv_int8 = 0, max_slots = 0, max_pages = 0;  // kv_int8: int8 pages
    uint32_t* page_table = nullptr;
    std::vector<uint32_t> page_table_host;
    velo::PageAllocator* allocator = nullptr;  // velo_cuda_slot_allocate / _release
    // per-step buffers, sized for cap_M rows
    int cap_M = 0, cap_B = 0;
    std::vector<void*> work;
    float* x = nullptr;
    __half* xn = nullptr;
    float* qkv = nullptr;
    __half* q = nullptr;
    __half* nk = nullptr;  // [L][M][Hkv][D]
    __half* nv = nullptr;
    __half* attn = nullptr;
    __half* hbuf = nullptr;
    float* xn32 = nullptr;     // fp32 path: normed rows / SwiGLU rows [M][max(H, F)]
    float* q32 = nullptr;      // [M][Hq][D]
    float* nk32 = nullptr;     // [L][M][Hkv][D]
    float* nv32 = nullptr;
    float* attn32 = nullptr;   // [M][Hq D]
    float* h32 = nullptr;      // [M][F]
    float* logits = nullptr;   // [M][V_loc]
    float* y = nullptr;        // [M][H] partial of a row-split GEMM (tp > 1, fp32 path)
    __nv_bfloat16* ybf = nullptr;  // [M][H] bf16 partial of a row-split GEMM (tp > 1)
    // tensor parallelism: two halves of the batch on two streams (one NCCL
    // communicator each) so that one half's all-reduce overlaps the other's GEMMs
    cudaStream_t half_stream[2] = {nullptr, nullptr};
    cudaEvent_t half_fork = nullptr, half_join[2] = {nullptr, nullptr};
    // tensor parallelism over NVLink peer memory: this rank's flag block and every
    // rank's flag block and partial buffer (ybf) mapped by CUDA IPC
    unsigned long long* ar_flags = nullptr;
    uint8_t* ipc_stage = nullptr;  // [tp][128] handles and device UUIDs for the all-gather
    unsigned long long* peer_flags[kPeerMaxRanks] = {};
    __nv_bfloat16* peer_ybf[kPeerMaxRanks] = {};
    // receive area of the fused sum: [tp][cap_M][H / tp], slab s = rank s's partial
    // of this rank's column block, written by rank s's GEMM epilogue
    __nv_bfloat16* stage = nullptr;
    __nv_bfloat16* peer_stage[kPeerMaxRanks] = {};
    // copy-engine sum: this rank's partial, column-blocked [tp][cap_M][H / tp] (local)
    __nv_bfloat16* part = nullptr;
    bool peer_flags_ok = false, peer_ybf_ok = false, peer_stage_ok = false;
    // step profile (velo_cuda_profile): an event at the start of every phase
    bool profile = false;
    std::vector<cudaEvent_t> prof_ev;
    std::vector<int> prof_cls;
    size_t prof_n = 0;
    double prof_ms[VELO_PHASE_COUNT] = {};
    int prof_steps = 0;
    int2* pairs = nullptr;     // [M] this shard's argmax
    int2* pairs_all = nullptr; // [tp][M]
    float* logits_all = nullptr;  // [tp][M][V_loc] gathered shards (tp > 1)
    size_t logits_all_cap = 0;
    float* logits_full = nullptr;  // [M][V] reassembled rows (tp > 1, sampling)
    size_t logits_full_cap = 0;
    // per-step inputs, one device block filled by one copy from a pinned
    // host mirror: tokens [M] | parents [M] | ctxlen [B] | slots [B] | pt_batch [B][max_pages]
    uint8_t* din = nullptr;
    uint8_t* hin = nullptr;
    size_t in_bytes = 0;
    uint32_t* tokens = nullptr;
    int32_t* parents = nullptr;
    int32_t* ctxlen = nullptr;
    uint32_t* slots = nullptr;
    uint32_t* pt_batch = nullptr;  // [B][max_pages] gathered rows
    // per-step outputs, one device block read back by one copy into pinned
    // memory: path_len [B] | bonus [B] | path [M] | expected [M]
    uint8_t* dout = nullptr;
    uint8_t* hout = nullptr;
    bool staging_busy = false;  // a step's copies may still use hin / hout
    // CUDA graphs of the step's launch sequence, one per (B, N, commit mode),
    // valid while the work buffers keep their addresses
    std::map<uint64_t, cudaGraphExec_t> graphs;
    bool graphs_off = false;    // capture refused on the stream in use
    uint64_t* anc = nullptr;
    uint32_t* expected = nullptr;
    int32_t* path = nullptr;
    int32_t* path_len = nullptr;
    uint32_t* bonus = nullptr;
    int32_t* acc = nullptr;
    float* drf = nullptr;
    float* uni = nullptr;
    uint32_t* dtok = nullptr;
    size_t drf_cap = 0;

    int H() const { return (int)meta.n_embd; }
    int Hq() const { return (int)meta.n_head; }
    int Hkv() const { return (int)meta.n_head_kv; }
    int F() const { return (int)meta.n_ff; }
    int V() const { return (int)meta.n_vocab; }
    int L() const { return (int)meta.n_layer; }
    size_t kv_elt() const { return f32 ? 4 : kv_int8 ? 1 : 2; }
    size_t layer_pool_elems() const { return (size_t)pool_pages * Hkv() * 16 * D; }
    size_t layer_scale_elems() const { return (size_t)pool_pages * Hkv() * 16; }
};

void close_peers(Model* m, void** peers) {
    for (int p = 0; p < m->tp && p < kPeerMaxRanks; ++p) {
        if (p != m->rank && peers[p]) cudaIpcCloseMemHandle(peers[p]);
        peers[p] = nullptr;
    }
}

void destroy_model(Model* m) {
    if (!m) return;
    close_peers(m, reinterpret_cast<void**>(m->peer_ybf));
    close_peers(m, reinterpret_cast<void**>(m->peer_stage));
    close_peers(m, reinterpret_cast<void**>(m->peer_flags));
    for (void* p : m->allocs) cudaFree(p);
    for (void* p : m->work) cudaFree(p);
    if (m->hin) cudaFreeHost(m->hin);
    if (m->hout) cudaFreeHost(m->hout);
    for (auto& g : m->graphs) cudaGraphExecDestroy(g.second);
    for (cudaEvent_t e : m->prof_ev) cudaEventDestroy(e);
    for (int h = 0; h < 2; ++h) {
        if (m->half_stream[h]) cudaStreamDestroy(m->half_stream[h]);
        if (m->half_join[h]) cudaEventDestroy(m->half_join[h]);
    }
    if (m->half_fork) cudaEventDestroy(m->half_fork);
    if (m->drf) cudaFree(m->drf);
    if (m->logits_all) cudaFree(m->logits_all);
    if (m->logits_full) cudaFree(m->logits_full);
    delete m->allocator;
    delete m;
}

namespace {

float h2f(uint16_t h) {
    __half_raw r;
    r.x = h;
    return __half2float(__half(r));
}

// dequant_row (src/quant.rs:181-191) for the dtypes accepted here
void host_dequant_row(int dt, const uint8_t* src, float* out, size_t n) {
    if (dt == VELO_DT_F32) {
        std::memcpy(out, src, n * 4);
    } else if (dt == VELO_DT_F16) {
        for (size_t i = 0; i < n; ++i) out[i] = h2f((uint16_t)(src[2 * i] | (src[2 * i + 1] << 8)));
    } else {  // q4_0, interleaved nibbles (quant.rs:50-64)
        for (size_t b = 0; b < n / 32; ++b) {
            const uint8_t* blk = src + b * 18;
            const float d = h2f((uint16_t)(blk[0] | (blk[1] << 8)));
            for (int i = 0; i < 16; ++i) {
                out[b * 32 + 2 * i] = d * (float)((int)(blk[2 + i] & 15) - 8);
                out[b * 32 + 2 * i + 1] = d * (float)((int)(blk[2 + i] >> 4) - 8);
            }
        }
    }
}

size_t row_bytes(int dt, size_t cols) {
    return dt == VELO_DT_F32 ? cols * 4 : dt == VELO_DT_F16 ? cols * 2 : cols / 32 * 18;
}

template <class T>
int32_t dev_alloc(Model* m, T** p, size_t bytes, bool work = false) {
    void* q = nullptr;
    cudaError_t e = cudaMalloc(&q, bytes ? bytes : 16);
    if (e != cudaSuccess)
        return fail(e == cudaErrorMemoryAllocation ? VELO_ERR_OUT_OF_MEMORY : VELO_ERR_CUDA,
                    "cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(e));
    (work ? m->work : m->allocs).push_back(q);
    *p = static_cast<T*>(q);
    return VELO_OK;
}

using Index = std::map<std::string, const velo_weight_desc*>;

const velo_weight_desc* find(const Index& ix, const std::string& name) {
    auto it = ix.find(name);
    return it == ix.end() ? nullptr : it->second;
}

bool on_device(const velo_weight_desc* w) { return (w->flags & VELO_WEIGHT_DEVICE) != 0; }

// A tensor's bytes in host memory: the caller's buffer, or a copy of a device
// tensor in `tmp`.  Null (error recorded) when the copy fails.
const uint8_t* host_view(const velo_weight_desc* w, size_t bytes, std::vector<uint8_t>& tmp) {
    if (!on_device(w)) return static_cast<const uint8_t*>(w->data);
    tmp.resize(bytes);
    const cudaError_t e = cudaMemcpy(tmp.data(), w->data, bytes, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
        fail(VELO_ERR_CUDA, "reading device tensor %s: %s", w->name, cudaGetErrorString(e));
        return nullptr;
    }
    return tmp.data();
}

// f32 vector (norm weight / embedding table) of rows x cols on the device
int32_t upload_f32(Model* m, const velo_weight_desc* w, size_t rows, size_t cols, float** out,
                   cudaStream_t s) {
    if (!w) return fail(VELO_ERR_INVALID_ARGUMENT, "missing tensor");
    if (w->rows * w->cols != rows * cols)
        return fail(VELO_ERR_INVALID_ARGUMENT, "tensor %s has %llu x %llu elements, expected %zu x %zu",
                    w->name, (unsigned long long)w->rows, (unsigned long long)w->cols, rows, cols);
    if (w->dtype < VELO_DT_F32 || w->dtype > VELO_DT_Q4_0 || !w->data ||
        (w->dtype == VELO_DT_Q4_0 && cols % 32))
        return fail(VELO_ERR_INVALID_ARGUMENT, "tensor %s: bad dtype / data", w->name);
    if (on_device(w) && w->dtype == VELO_DT_F32) {  // device f32: a device copy
        int32_t st = dev_alloc(m, out, rows * cols * 4);
        if (st) return st;
        VELO_CUDA_TRY(cudaMemcpyAsync(*out, w->data, rows * cols * 4, cudaMemcpyDeviceToDevice, s));
        VELO_CUDA_TRY(cudaStreamSynchronize(s));
        return VELO_OK;
    }
    std::vector<float> host(rows * cols);
    const size_t rb = row_bytes(w->dtype, cols);
    std::vector<uint8_t> tmp;
    const uint8_t* src = host_view(w, rows * rb, tmp);
    if (!src) return VELO_ERR_CUDA;
    for (size_t r = 0; r < rows; ++r) host_dequant_row(w->dtype, src + r * rb, host.data() + r * cols, cols);
    int32_t st = dev_alloc(m, out, host.size() * 4);
    if (st) return st;
    VELO_CUDA_TRY(cudaMemcpyAsync(*out, host.data(), host.size() * 4, cudaMemcpyHostToDevice, s));
    VELO_CUDA_TRY(cudaStreamSynchronize(s));
    return VELO_OK;
}

// fp32 path: matrices of any dtype (concatenated by rows) dequantised to f32
// rows on the device, as LlamaCpuModel reads them (matvec_quant over
// dequant_row, llama_cpu.rs:75-90)
int32_t upload_f32_rows(Model* m, const std::vector<const velo_weight_desc*>& parts, size_t cols,
                        uint8_t** out, cudaStream_t s) {
    size_t rows = 0;
    for (auto* w : parts) {
        if (!w) return fail(VELO_ERR_INVALID_ARGUMENT, "missing matrix");
        if (w->dtype < VELO_DT_F32 || w->dtype > VELO_DT_Q4_0 || !w->data)
            return fail(VELO_ERR_INVALID_ARGUMENT, "matrix %s: bad dtype / data", w->name);
        if (w->cols != cols || (w->dtype == VELO_DT_Q4_0 && cols % 32))
            return fail(VELO_ERR_INVALID_ARGUMENT, "matrix %s: %llu columns, expected %zu", w->name,
                        (unsigned long long)w->cols, cols);
        rows += w->rows;
    }
    std::vector<float> host(rows * cols);
    size_t r0 = 0;
    for (auto* w : parts) {
        const size_t rb = row_bytes(w->dtype, cols);
        std::vector<uint8_t> tmp;
        const uint8_t* src = host_view(w, w->rows * rb, tmp);
        if (!src) return VELO_ERR_CUDA;
        for (size_t r = 0; r < w->rows; ++r) host_dequant_row(w->dtype, src + r * rb, host.data() + (r0 + r) * cols, cols);
        r0 += w->rows;
    }
    int32_t st = dev_alloc(m, out, host.size() * 4);
    if (st) return st;
    VELO_CUDA_TRY(cudaMemcpyAsync(*out, host.data(), host.size() * 4, cudaMemcpyHostToDevice, s));
    VELO_CUDA_TRY(cudaStreamSynchronize(s));
    return VELO_OK;
}

// q4_0 matrices (concatenated by rows, or a gate/up pair) -> repacked device weight
int32_t upload_q4(Model* m, const std::vector<const velo_weight_desc*>& parts, size_t cols, bool pair,
                  uint8_t** out, cudaStream_t s) {
    size_t rows = 0;
    for (auto* w : parts) {
        if (!w) return fail(VELO_ERR_INVALID_ARGUMENT, "missing matrix");
        if (w->dtype != VELO_DT_Q4_0 || !w->data)
            return fail(VELO_ERR_INVALID_ARGUMENT, "matrix %s must be q4_0 (dtype %d)", w->name, w->dtype);
        if (w->cols != cols || cols % 32)
            return fail(VELO_ERR_INVALID_ARGUMENT, "matrix %s: %llu columns, expected %zu", w->name,
                        (unsigned long long)w->cols, cols);
        rows += w->rows;
    }
    const size_t rb = cols / 32 * 18;
    uint8_t* raw = nullptr;
    VELO_CUDA_TRY(cudaMalloc(&raw, rows * rb));
    size_t off = 0;
    for (auto* w : parts) {
        cudaError_t e = cudaMemcpy(raw + off, w->data, w->rows * rb,
                                   on_device(w) ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            cudaFree(raw);
            return fail(VELO_ERR_CUDA, "weight upload failed: %s", cudaGetErrorString(e));
        }
        off += w->rows * rb;
    }
    int32_t st = dev_alloc(m, out, q4_repacked_bytes((int)rows, (int)cols));
    if (st) {
        cudaFree(raw);
        return st;
    }
    cudaError_t e = launch_q4_repack(raw, pair ? raw + parts[0]->rows * rb : nullptr, pair, (int)rows,
                                     (int)cols, *out, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    cudaFree(raw);
    if (e != cudaSuccess) return fail(VELO_ERR_CUDA, "q4_0 repack failed: %s", cudaGetErrorString(e));
    return VELO_OK;
}

int32_t nccl_check(ncclResult_t r, const NcclApi* nc, const char* what);

// Map every rank's `local` allocation (cudaMalloc base) into this process: the
// CUDA IPC handles are all-gathered over the group's NCCL communicator (every
// rank calls this at the same point), then opened.  peers[rank] = local.
// Returns false (and leaves peers null) when IPC is unavailable or two ranks share
// a GPU (their sum kernels would wait on one another on one device); the callers
// then keep NCCL for the sums.
bool ipc_exchange(velo_cuda_ctx* c, Model* m, void* local, void** peers) {
    constexpr size_t kRec = 128;  // per rank: IPC handle (64 bytes), device UUID (16)
    close_peers(m, peers);
    const NcclApi* nc = nccl_api();
    if (!nc || !m->ipc_stage || m->tp > kPeerMaxRanks) return false;
    uint8_t rec[kRec] = {};
    cudaIpcMemHandle_t h;
    cudaDeviceProp prop;
    bool ok = cudaIpcGetMemHandle(&h, local) == cudaSuccess && cudaGetDeviceProperties(&prop, c->device) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
    } else {
        std::memcpy(rec, &h, 64);
        std::memcpy(rec + 64, &prop.uuid, 16);
    }
    std::vector<uint8_t> all(kRec * m->tp);
    // the all-gather runs on every rank even when this rank's handle failed, so the
    // collective stays matched; a zero handle then fails the open on the others
    cudaStream_t s = c->stream;
    if (cudaMemcpyAsync(m->ipc_stage + kRec * m->rank, rec, kRec, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        nc->AllGather(m->ipc_stage + kRec * m->rank, m->ipc_stage, kRec, ncclUint8,
                      static_cast<ncclComm_t>(c->nccl_comm), s) != ncclSuccess ||
        cudaMemcpyAsync(all.data(), m->ipc_stage, all.size(), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    for (int p = 0; p < m->tp && ok; ++p)
        if (p != m->rank && std::memcmp(all.data() + kRec * p + 64, rec + 64, 16) == 0) ok = false;
    for (int p = 0; p < m->tp && ok; ++p) {
        if (p == m->rank) {
            peers[p] = local;
            continue;
        }
        cudaIpcMemHandle_t hp;
        std::memcpy(&hp, all.data() + kRec * p, 64);
        void* ptr = nullptr;
        if (cudaIpcOpenMemHandle(&ptr, hp, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            ok = false;
            continue;
        }
        peers[p] = ptr;
    }
    if (!ok) close_peers(m, peers);
    return ok;
}

// true only if `ok` holds on every rank (a min all-reduce over the group), so that
// all ranks take the same path for their sums
bool group_all_ok(velo_cuda_ctx* c, Model* m, bool ok) {
    const NcclApi* nc = nccl_api();
    if (!nc || !m->ipc_stage) return false;
    int v = ok ? 1 : 0;
    cudaStream_t s = c->stream;
    int32_t* d = reinterpret_cast<int32_t*>(m->ipc_stage);
    if (cudaMemcpyAsync(d, &v, 4, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        nc->AllReduce(d, d, 1, ncclInt32, ncclMin, static_cast<ncclComm_t>(c->nccl_comm), s) != ncclSuccess ||
        cudaMemcpyAsync(&v, d, 4, cudaMemcpyDeviceToHost, s) != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return v == 1;
}

int32_t ensure_work(velo_cuda_ctx* c, Model* m, int B, int N) {
    const int M = B * N;
    if (M <= m->cap_M && B <= m->cap_B) return VELO_OK;
    VELO_CUDA_TRY(cudaStreamSynchronize(c->stream));
    for (auto& g : m->graphs) cudaGraphExecDestroy(g.second);  // they name the old buffers
    m->graphs.clear();
    for (void* p : m->work) cudaFree(p);
    m->work.clear();
    const int cM = M > m->cap_M ? M : m->cap_M, cB = B > m->cap_B ? B : m->cap_B;
    const size_t H = m->H(), D = m->D, Hq = m->Hq(), Hkv = m->Hkv(), F = m->F();
    const size_t L = m->L();
    int32_t st = VELO_OK;
    if (!st) st = dev_alloc(m, &m->x, (size_t)cM * H * 4, true);
    if (!st) st = dev_alloc(m, &m->qkv, (size_t)cM * (Hq + 2 * Hkv) * D * 4, true);
    if (m->f32) {
        if (!st) st = dev_alloc(m, &m->xn32, (size_t)cM * H * 4, true);
        if (!st) st = dev_alloc(m, &m->q32, (size_t)cM * Hq * D * 4, true);
        if (!st) st = dev_alloc(m, &m->nk32, L * cM * Hkv * D * 4, true);
        if (!st) st = dev_alloc(m, &m->nv32, L * cM * Hkv * D * 4, true);
        if (!st) st = dev_alloc(m, &m->attn32, (size_t)cM * Hq * D * 4, true);
        if (!st) st = dev_alloc(m, &m->h32, (size_t)cM * F * 4, true);
    } else {
        if (!st) st = dev_alloc(m, &m->xn, (size_t)cM * (H > F ? H : F) * 2, true);
        if (!st) st = dev_alloc(m, &m->q, (size_t)cM * Hq * D * 2, true);
        if (!st) st = dev_alloc(m, &m->nk, L * cM * Hkv * D * 2, true);
        if (!st) st = dev_alloc(m, &m->nv, L * cM * Hkv * D * 2, true);
        if (!st) st = dev_alloc(m, &m->attn, (size_t)cM * Hq * D * 2, true);
        if (!st) st = dev_alloc(m, &m->hbuf, (size_t)cM * F * 2, true);
    }
    if (!st) st = dev_alloc(m, &m->logits, (size_t)cM * m->V_loc * 4, true);
    if (!st && m->tp > 1 && m->f32) st = dev_alloc(m, &m->y, (size_t)cM * H * 4, true);
    if (!st && m->tp > 1 && !m->f32) {
        st = dev_alloc(m, &m->ybf, (size_t)cM * H * 2, true);
        // every rank maps every rank's flag block (once) and partial buffer (whenever it
        // grows); all ranks grow their buffers in the same step, so the exchanges match
        if (!st && !m->ar_flags) {
            st = dev_alloc(m, &m->ar_flags, kPeerFlagBytes);
            if (!st) st = dev_alloc(m, &m->ipc_stage, (size_t)128 * kPeerMaxRanks);
            if (!st && cudaMemset(m->ar_flags, 0, kPeerFlagBytes) != cudaSuccess)
                st = fail(VELO_ERR_CUDA, "peer flag block: cudaMemset failed");
            if (!st) m->peer_flags_ok = ipc_exchange(c, m, m->ar_flags, reinterpret_cast<void**>(m->peer_flags));
        }
        if (!st) m->peer_ybf_ok = ipc_exchange(c, m, m->ybf, reinterpret_cast<void**>(m->peer_ybf));
        if (!st) st = dev_alloc(m, &m->stage, (size_t)cM * H * 2, true);
        if (!st) st = dev_alloc(m, &m->part, (size_t)cM * H * 2, true);
        if (!st) m->peer_stage_ok = ipc_exchange(c, m, m->stage, reinterpret_cast<void**>(m->peer_stage));
        if (!st) {
            const bool all = group_all_ok(c, m, m->peer_flags_ok && m->peer_ybf_ok);
            m->peer_flags_ok = m->peer_ybf_ok = all;
            m->peer_stage_ok = group_all_ok(c, m, all && m->peer_stage_ok);
        }
    }
    if (!st) st = dev_alloc(m, &m->pairs, (size_t)cM * 8, true);
    if (!st) st = dev_alloc(m, &m->pairs_all, (size_t)cM * 8 * m->tp, true);

    if (!st) st = dev_alloc(m, &m->anc, (size_t)cM * 8, true);


    if (!st) st = dev_alloc(m, &m->dtok, (size_t)cM * 4, true);
    if (!st) st = dev_alloc(m, &m->uni, (size_t)cM * 4, true);
    // packed step I/O (4-byte words)
    const size_t mp = m->max_pages ? m->max_pages : 1;
    m->in_bytes = ((size_t)2 * cM + 2 * cB + cB * mp) * 4;
    const size_t out_bytes = ((size_t)2 * cB + 2 * cM) * 4;
    if (!st) st = dev_alloc(m, &m->din, m->in_bytes, true);
    if (!st) st = dev_alloc(m, &m->dout, out_bytes, true);
    if (!st) {
        if (m->hin) cudaFreeHost(m->hin);
        if (m->hout) cudaFreeHost(m->hout);
        m->hin = m->hout = nullptr;
        cudaError_t e = cudaMallocHost(&m->hin, m->in_bytes);
        if (e == cudaSuccess) e = cudaMallocHost(&m->hout, out_bytes);
        if (e != cudaSuccess) st = fail(VELO_ERR_OUT_OF_MEMORY, "pinned staging: %s", cudaGetErrorString(e));
    }
    if (!st) st = dev_alloc(m, &m->acc, (size_t)cB * 4, true);
    if (st) {
        m->cap_M = m->cap_B = 0;
        return st;
    }
    m->cap_M = cM;
    m->cap_B = cB;
    return VELO_OK;
}

int32_t gemm_on(velo_cuda_ctx* c, cudaStream_t s, const uint8_t* w, const __half* x, int M, int N, int K,
                void* y, int ldy, int mode) {
    Q4GemmArgs a{};
    a.w = w;
    a.N = N;
    a.K = K;
    a.M = M;
    a.y = y;
    a.ldy = ldy;
    a.mode = mode;
    a.err = c->err_flag;
    VELO_CUDA_TRY(launch_q4_gemm(a, x, c->sm_count, s));
    return VELO_OK;
}

int32_t gemm(velo_cuda_ctx* c, const uint8_t* w, const __half* x, int M, int N, int K, void* y,
             int ldy, int mode) {
    Q4GemmArgs a{};
    a.w = w;
    a.N = N;
    a.K = K;
    a.M = M;
    a.y = y;
    a.ldy = ldy;
    a.mode = mode;
    a.err = c->err_flag;
    VELO_CUDA_TRY(launch_q4_gemm(a, x, c->sm_count, c->stream));
    return VELO_OK;
}

int32_t nccl_check(ncclResult_t r, const NcclApi* nc, const char* what) {
    if (r == ncclSuccess) return VELO_OK;
    return fail(VELO_ERR_NCCL, "%s failed: %s", what, nc->GetErrorString(r));
}

// y (the partial of this rank's row-split GEMM) summed over the group, added to x
int32_t allreduce_add(velo_cuda_ctx* c, Model* m, int M) {
    const NcclApi* nc = nccl_api();
    if (!nc) return VELO_ERR_NCCL;
    const size_t n = (size_t)M * m->H();
    int32_t st = nccl_check(nc->AllReduce(m->y, m->y, n, ncclFloat32, ncclSum,
                                          static_cast<ncclComm_t>(c->nccl_comm), c->stream),
                            nc, "ncclAllReduce");
    if (st) return st;
    VELO_CUDA_TRY(launch_add_f32(m->x, m->y, n, c->stream));
    return VELO_OK;
}

// ybf (bf16 partials of this rank's row-split GEMM) summed over the group in
// place; the RMSNorm that follows adds the sum to the residual
// (launch_add_rmsnorm_f16).  A 16-bit sum moves half the bytes of an f32 one
// over NVLink (33.5 MB instead of 67 MB per call at M = 2048, H = 8192).
// The sum over NVLink peer memory (launch_peer_allreduce) when every rank's
// buffers are mapped, else NCCL; VELO_TP_AR=nccl forces NCCL.
bool use_peer_sum(const Model* m) {
    const char* e = std::getenv("VELO_TP_AR");
    const bool want = e ? std::strcmp(e, "nccl") != 0 : m->tp >= 4;
    return want && m->peer_flags_ok && m->peer_ybf_ok && peer_tp_supported(m->tp);
}

// The fused sum (the GEMM epilogue pushes each column block to its owner, a
// gather kernel adds and broadcasts) when the receive areas are mapped and the
// column blocks are whole 32-column groups, by default from 4 ranks on.  At 2
// ranks the sums are a small share of the step and two streams already hide
// NCCL's; the epilogue's NVLink stores then cost the GEMMs more than the gather
// saves (config 5: 157.6 ms per step with NCCL against 164.2 fused; at 4 ranks
// 95.5 against 89.2).  VELO_TP_AR=fused / peer / nccl chooses explicitly.
bool use_fused_sum(const Model* m) {
    const char* e = std::getenv("VELO_TP_AR");
    const bool want = e ? std::strcmp(e, "fused") == 0 : m->tp >= 4;
    return want && use_peer_sum(m) && m->peer_stage_ok && m->H() % (32 * m->tp) == 0;
}

// The copy-engine sum (VELO_TP_AR=ce): the GEMM stores its partial locally in
// column blocks, each block crosses NVLink as one cudaMemcpyAsync to its owner,
// the owner adds the tp blocks and copies its block of the sum to every rank;
// one-warp kernels publish and await the copies' completion.
bool use_ce_sum(const Model* m) {
    const char* e = std::getenv("VELO_TP_AR");
    return e && std::strcmp(e, "ce") == 0 && m->peer_flags_ok && m->peer_ybf_ok && m->peer_stage_ok &&
           peer_tp_supported(m->tp) && m->H() % (32 * m->tp) == 0;
}

PeerSync peer_sync(velo_cuda_ctx* c, const Model* m, int slot) {
    PeerSync y{};
    for (int p = 0; p < m->tp; ++p) y.flags[p] = m->peer_flags[p];
    y.rank = m->rank;
    y.tp = m->tp;
    y.slot = slot;
    y.err = c->err_flag;
    return y;
}

int32_t peer_sum(velo_cuda_ctx* c, Model* m, size_t offset, size_t n, int slot, cudaStream_t s) {
    PeerAllReduceArgs a{};
    a.sync = peer_sync(c, m, slot);
    for (int p = 0; p < m->tp; ++p) a.buf[p] = m->peer_ybf[p];
    a.offset = offset;
    a.n = n;
    VELO_CUDA_TRY(launch_peer_allreduce(a, s));
    return VELO_OK;
}

// Row-split GEMM (o_proj, down_proj) of `rows` rows from row0 with the
// tensor-parallel sum fused in: the epilogue stores column block o of the bf16
// partial into rank o's receive area (slab `rank`; gemm_push), then the gather
// kernel of this rank adds its block's tp slabs and stores the sum into every
// rank's ybf (gather_sum).
int32_t gemm_push(velo_cuda_ctx* c, Model* m, cudaStream_t s, const uint8_t* w, const __half* x, int rows, int K,
                  size_t row0) {
    const int H = m->H(), tp = m->tp, Hc = H / tp;
    Q4GemmArgs a{};
    a.w = w;
    a.N = H;
    a.K = K;
    a.M = rows;
    a.y = nullptr;
    a.ldy = H;
    a.mode = kEpiPeerBF16;
    a.err = c->err_flag;
    a.peer_cols = Hc;
    for (int o = 0; o < tp; ++o) a.peer_y[o] = m->peer_stage[o] + ((size_t)m->rank * m->cap_M + row0) * Hc;
    VELO_CUDA_TRY(launch_q4_gemm(a, x, c->sm_count, s));
    return VELO_OK;
}

int32_t gather_sum(velo_cuda_ctx* c, Model* m, cudaStream_t s, int rows, size_t row0, int slot) {
    const int H = m->H(), tp = m->tp, Hc = H / tp;
    PeerGatherArgs g{};
    g.sync = peer_sync(c, m, slot);
    g.stage = m->stage + row0 * Hc;
    g.slab = (size_t)m->cap_M * Hc;
    for (int p = 0; p < tp; ++p) g.out[p] = m->peer_ybf[p] + row0 * H + (size_t)m->rank * Hc;
    g.rows = rows;
    g.cols = Hc;
    g.ld = H;
    VELO_CUDA_TRY(launch_peer_gather(g, s));
    return VELO_OK;
}

// Copy-engine form of gemm_fused_sum (use_ce_sum).  Leaves this call's rows of
// the sum in ybf, column-blocked: block o at ybf + o * cap_M * (H / tp).
int32_t ce_gemm(velo_cuda_ctx* c, Model* m, cudaStream_t s, const uint8_t* w, const __half* x, int rows, int K,
                size_t row0) {
    const int H = m->H(), tp = m->tp, Hc = H / tp;
    Q4GemmArgs a{};
    a.w = w;
    a.N = H;
    a.K = K;
    a.M = rows;
    a.y = nullptr;
    a.ldy = H;
    a.mode = kEpiPeerBF16;  // to this rank's own column-blocked buffer: local stores
    a.err = c->err_flag;
    a.peer_cols = Hc;
    for (int o = 0; o < tp; ++o) a.peer_y[o] = m->part + ((size_t)o * m->cap_M + row0) * Hc;
    VELO_CUDA_TRY(launch_q4_gemm(a, x, c->sm_count, s));
    return VELO_OK;
}

int32_t ce_sum(velo_cuda_ctx* c, Model* m, cudaStream_t s, int rows, size_t row0, int slot) {
    const int tp = m->tp, r = m->rank, Hc = m->H() / tp;
    const size_t bytes = (size_t)rows * Hc * 2, blk = (size_t)m->cap_M * Hc;
    const PeerSync y = peer_sync(c, m, slot);
    for (int o = 0; o < tp; ++o)
        if (o != r)
            VELO_CUDA_TRY(cudaMemcpyAsync(m->peer_stage[o] + r * blk + row0 * Hc, m->part + o * blk + row0 * Hc, bytes,
                                          cudaMemcpyDeviceToDevice, s));
    VELO_CUDA_TRY(launch_ce_signal(y, kCePhaseSlabs, s));
    VELO_CUDA_TRY(launch_ce_wait(y, kCePhaseSlabs, s));
    CeSumArgs g{};
    g.own = m->part + r * blk + row0 * Hc;
    g.stage = m->stage + row0 * Hc;
    g.slab = blk;
    g.out = m->ybf + r * blk + row0 * Hc;
    g.n = (size_t)rows * Hc;
    g.rank = r;
    g.tp = tp;
    VELO_CUDA_TRY(launch_ce_sum(g, c->sm_count, s));
    for (int o = 0; o < tp; ++o)
        if (o != r)
            VELO_CUDA_TRY(cudaMemcpyAsync(m->peer_ybf[o] + r * blk + row0 * Hc, m->ybf + r * blk + row0 * Hc, bytes,
                                          cudaMemcpyDeviceToDevice, s));
    VELO_CUDA_TRY(launch_ce_signal(y, kCePhaseSums, s));
    VELO_CUDA_TRY(launch_ce_wait(y, kCePhaseSums, s));
    return VELO_OK;
}

int32_t gemm_fused_sum(velo_cuda_ctx* c, Model* m, cudaStream_t s, const uint8_t* w, const __half* x, int rows,
                       int K, size_t row0, int slot) {
    if (use_ce_sum(m)) {
        int32_t st = ce_gemm(c, m, s, w, x, rows, K, row0);
        return st ? st : ce_sum(c, m, s, rows, row0, slot);
    }
    int32_t st = gemm_push(c, m, s, w, x, rows, K, row0);
    return st ? st : gather_sum(c, m, s, rows, row0, slot);
}

int32_t allreduce_bf16(velo_cuda_ctx* c, Model* m, int M) {
    const size_t n = (size_t)M * m->H();
    if (use_peer_sum(m)) return peer_sum(c, m, 0, n, 0, c->stream);
    const NcclApi* nc = nccl_api();
    if (!nc) return VELO_ERR_NCCL;
    return nccl_check(nc->AllReduce(m->ybf, m->ybf, n, ncclBfloat16, ncclSum,
                                    static_cast<ncclComm_t>(c->nccl_comm), c->stream),
                      nc, "ncclAllReduce");
}

// Tensor-parallel layer loop with the batch cut in two halves, sequences
// [0, B0) and [B0, B), each on its own stream with its own NCCL communicator:
// the layer's work is issued half by half, so while one half's bf16
// all-reduce after o_proj or down_proj crosses NVLink the other half's GEMMs
// and attention keep the SMs busy.  Every row op is row-local (attention
// reads only its own sequence), so each half runs the same kernels on its
// row range; the results equal the single-stream loop's up to the order of
// the GEMMs' f32 k-sums (tiles land on other CTAs, which start their k loops
// at other offsets).  On return the context stream has joined both halves;
// x holds the residual rows with the last sums added, xn the final RMSNorm.
int32_t forward_tp_halves(velo_cuda_ctx* c, Model* m, int B, int N) {
    const int H = m->H(), Hq = m->Hq(), Hkv = m->Hkv(), F = m->F(), L = m->L();
    const int M = B * N, Nqkv = (Hq + 2 * Hkv) * 128;
    const float eps = m->meta.norm_eps;
    const NcclApi* nc = nccl_api();
    if (!nc) return VELO_ERR_NCCL;
    for (int h = 0; h < 2; ++h) {
        if (!m->half_stream[h]) VELO_CUDA_TRY(cudaStreamCreateWithFlags(&m->half_stream[h], cudaStreamNonBlocking));
        if (!m->half_join[h]) VELO_CUDA_TRY(cudaEventCreateWithFlags(&m->half_join[h], cudaEventDisableTiming));
    }
    if (!m->half_fork) VELO_CUDA_TRY(cudaEventCreateWithFlags(&m->half_fork, cudaEventDisableTiming));
    const int bh[2] = {B / 2, B - B / 2}, b0[2] = {0, B / 2};
    void* comm[2] = {c->nccl_comm, c->nccl_comm2};
    VELO_CUDA_TRY(cudaEventRecord(m->half_fork, c->stream));
    for (int h = 0; h < 2; ++h) VELO_CUDA_TRY(cudaStreamWaitEvent(m->half_stream[h], m->half_fork, 0));
    bool pending[2] = {false, false};
    const bool ce = use_ce_sum(m);
    auto rows = [&](int h) { return bh[h] * N; };
    auto r0 = [&](int h) { return (size_t)b0[h] * N; };
    auto norm = [&](int h, const float* w) -> cudaError_t {
        const size_t o = r0(h) * H;
        if (!pending[h]) return launch_rmsnorm_f16(m->x + o, w, rows(h), H, eps, m->xn + o, m->half_stream[h]);
        pending[h] = false;
        if (ce)
            return launch_add_rmsnorm_blocked_f16(m->x + o, m->ybf + r0(h) * (H / m->tp), H / m->tp,
                                                  (size_t)m->cap_M * (H / m->tp), w, rows(h), H, eps, m->xn + o,
                                                  m->half_stream[h]);
        return launch_add_rmsnorm_f16(m->x + o, m->ybf + o, w, rows(h), H, eps, m->xn + o, m->half_stream[h]);
    };
    auto reduce = [&](int h) -> int32_t {
        pending[h] = true;
        if (use_peer_sum(m)) return peer_sum(c, m, r0(h) * H, (size_t)rows(h) * H, h, m->half_stream[h]);
        return nccl_check(nc->AllReduce(m->ybf + r0(h) * H, m->ybf + r0(h) * H, (size_t)rows(h) * H, ncclBfloat16,
                                        ncclSum, static_cast<ncclComm_t>(comm[h]), m->half_stream[h]),
                          nc, "ncclAllReduce");
    };
    const bool fused = ce || use_fused_sum(m);
    int32_t st = VELO_OK;
    for (int l = 0; l < L; ++l) {
        const Layer& ly = m->layers[l];
        for (int h = 0; h < 2 && !st; ++h) {  // attention block
            if (!bh[h]) continue;
            cudaStream_t s = m->half_stream[h];
            const size_t o = r0(h);
            __half* nk = m->nk + (size_t)l * M * Hkv * 128 + o * Hkv * 128;
            __half* nv = m->nv + (size_t)l * M * Hkv * 128 + o * Hkv * 128;
            VELO_CUDA_TRY(norm(h, ly.attn_norm));
            st = gemm_on(c, s, ly.wqkv, m->xn + o * H, rows(h), Nqkv, H, m->qkv + o * Nqkv, Nqkv, kEpiStoreF32);
            if (st) return st;
            VELO_CUDA_TRY(launch_rope_split(m->qkv + o * Nqkv, m->anc + o, m->ctxlen + b0[h], bh[h], N, Hq, Hkv,
                                            m->meta.rope_freq_base, m->q + o * Hq * 128, nk, nv, s));
            TreeAttnArgs a{};
            const size_t lo = (size_t)l * m->layer_pool_elems() * m->kv_elt();
            a.q = m->q + o * Hq * 128;
            a.k_pool = static_cast<uint8_t*>(m->k_pool) + lo;
            a.v_pool = static_cast<uint8_t*>(m->v_pool) + lo;
            a.k_scale = m->kv_int8 ? m->k_scale + (size_t)l * m->layer_scale_elems() : nullptr;
            a.v_scale = m->kv_int8 ? m->v_scale + (size_t)l * m->layer_scale_elems() : nullptr;
            a.page_table = m->pt_batch + (size_t)b0[h] * m->max_pages;
            a.ctx_len = m->ctxlen + b0[h];
            a.node_k = nk;
            a.node_v = nv;
            a.anc = m->anc + o;
            a.out = m->attn + o * Hq * 128;
            a.out_f16 = 1;
            a.B = bh[h];
            a.N = N;
            a.Hq = Hq;
            a.Hkv = Hkv;
            a.max_pages = m->max_pages;
            a.pool_pages = m->pool_pages;
            a.scale_log2 = (float)(1.4426950408889634 / std::sqrt(128.0));
            a.err = c->err_flag;
            VELO_CUDA_TRY(launch_tree_attention(a, m->kv_int8 != 0, s));
            if (fused) {
                pending[h] = true;
                st = gemm_fused_sum(c, m, s, ly.wo, m->attn + o * Hq * 128, rows(h), Hq * 128, o, h);
            } else {
                st = gemm_on(c, s, ly.wo, m->attn + o * Hq * 128, rows(h), H, Hq * 128, m->ybf + o * H, H,
                             kEpiStoreBF16);
                if (!st) st = reduce(h);
            }
        }
        for (int h = 0; h < 2 && !st; ++h) {  // feed-forward block
            if (!bh[h]) continue;
            cudaStream_t s = m->half_stream[h];
            const size_t o = r0(h);
            VELO_CUDA_TRY(norm(h, ly.ffn_norm));
            st = gemm_on(c, s, ly.w13, m->xn + o * H, rows(h), 2 * F, H, m->hbuf + o * F, F, kEpiSwiGLU);
            if (!st && fused) {
                pending[h] = true;
                st = gemm_fused_sum(c, m, s, ly.w2, m->hbuf + o * F, rows(h), F, o, h);
            } else if (!st) {
                st = gemm_on(c, s, ly.w2, m->hbuf + o * F, rows(h), H, F, m->ybf + o * H, H, kEpiStoreBF16);
                if (!st) st = reduce(h);
            }
        }
        if (st) return st;
    }
    for (int h = 0; h < 2; ++h) {
        if (bh[h]) VELO_CUDA_TRY(norm(h, m->out_norm));
        VELO_CUDA_TRY(cudaEventRecord(m->half_join[h], m->half_stream[h]));
        VELO_CUDA_TRY(cudaStreamWaitEvent(c->stream, m->half_join[h], 0));
    }
    return VELO_OK;
}

// Step profile: an event marks the start of a phase on the context stream.
cudaError_t prof_mark(velo_cuda_ctx* c, Model* m, int cls) {
    if (!m->profile) return cudaSuccess;
    if (m->prof_n == m->prof_ev.size()) {
        cudaEvent_t e;
        cudaError_t err = cudaEventCreate(&e);
        if (err != cudaSuccess) return err;
        m->prof_ev.push_back(e);
        m->prof_cls.push_back(0);
    }
    m->prof_cls[m->prof_n] = cls;
    return cudaEventRecord(m->prof_ev[m->prof_n++], c->stream);
}

// After the step's sync: the time from each mark to the next goes to the
// phase of the earlier mark.
void prof_collect(Model* m) {
    if (!m->profile) return;
    for (size_t i = 0; i + 1 < m->prof_n; ++i) {
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, m->prof_ev[i], m->prof_ev[i + 1]) == cudaSuccess &&
            m->prof_cls[i] >= 0 && m->prof_cls[i] < VELO_PHASE_COUNT)
            m->prof_ms[m->prof_cls[i]] += ms;
    }
    if (m->prof_n) m->prof_steps++;
    m->prof_n = 0;
}

// Full target rows [M][V] on every rank from the vocabulary shards
// [M][V_loc]: one all-gather into [tp][M][V_loc], then one strided copy per
// shard.  Buffers grow on demand (the stream is drained first).
int32_t gather_full_logits(velo_cuda_ctx* c, Model* m, int M, bool full) {
    cudaStream_t s = c->stream;
    const size_t per = (size_t)M * m->V_loc;
    const size_t all = per * m->tp;
    if (all > m->logits_all_cap || (full && all > m->logits_full_cap)) {
        VELO_CUDA_TRY(cudaStreamSynchronize(s));
        if (all > m->logits_all_cap) {
            if (m->logits_all) cudaFree(m->logits_all);
            m->logits_all = nullptr;
            m->logits_all_cap = 0;
            VELO_CUDA_TRY(cudaMalloc(&m->logits_all, all * 4));
            m->logits_all_cap = all;
        }
        if (full && all > m->logits_full_cap) {
            if (m->logits_full) cudaFree(m->logits_full);
            m->logits_full = nullptr;
            m->logits_full_cap = 0;
            VELO_CUDA_TRY(cudaMalloc(&m->logits_full, all * 4));
            m->logits_full_cap = all;
        }
    }
    const NcclApi* nc = nccl_api();
    if (!nc) return VELO_ERR_NCCL;
    int32_t st = nccl_check(nc->AllGather(m->logits, m->logits_all, per, ncclFloat32,
                                          static_cast<ncclComm_t>(c->nccl_comm), s),
                            nc, "ncclAllGather");
    if (st || !full) return st;
    const size_t row = (size_t)m->V_loc * 4;
    for (int r = 0; r < m->tp; ++r)
        VELO_CUDA_TRY(cudaMemcpy2DAsync(m->logits_full + (size_t)r * m->V_loc, row * m->tp,
                                        m->logits_all + (size_t)r * per, row, row, (size_t)M,
                                        cudaMemcpyDeviceToDevice, s));
    return VELO_OK;
}

// The fp32 path's layer loop and LM head (f32_path.cu), on rows x = the
// embedded tree nodes; logits [M][V_loc] out.
int32_t forward_f32(velo_cuda_ctx* c, Model* m, int B, int N) {
    cudaStream_t s = c->stream;
    const int M = B * N, H = m->H(), Hq = m->Hq(), Hkv = m->Hkv(), F = m->F(), L = m->L(), D = m->D;
    const int Nqkv = (Hq + 2 * Hkv) * D;
    const float eps = m->meta.norm_eps;
    auto mat = [](const uint8_t* p) { return reinterpret_cast<const float*>(p); };
    int32_t st = VELO_OK;
    for (int l = 0; l < L; ++l) {
        const Layer& ly = m->layers[l];
        float* nk = m->nk32 + (size_t)l * M * Hkv * D;
        float* nv = m->nv32 + (size_t)l * M * Hkv * D;
        VELO_CUDA_TRY(launch_rmsnorm_f32(m->x, ly.attn_norm, M, H, eps, m->xn32, s));
        VELO_CUDA_TRY(launch_gemm_f32(mat(ly.wqkv), m->xn32, M, Nqkv, H, m->qkv, Nqkv, kF32Store, s));
        VELO_CUDA_TRY(launch_rope_split_f32(m->qkv, m->anc, m->ctxlen, B, N, Hq, Hkv, D,
                                            m->meta.rope_freq_base, m->q32, nk, nv, s));
        TreeAttnF32Args a{};
        const size_t lo = (size_t)l * m->layer_pool_elems();
        a.q = m->q32;
        a.k_pool = static_cast<const float*>(m->k_pool) + lo;
        a.v_pool = static_cast<const float*>(m->v_pool) + lo;
        a.page_table = m->pt_batch;
        a.ctx_len = m->ctxlen;
        a.node_k = nk;
        a.node_v = nv;
        a.anc = m->anc;
        a.out = m->attn32;
        a.B = B;
        a.N = N;
        a.Hq = Hq;
        a.Hkv = Hkv;
        a.D = D;
        a.max_pages = m->max_pages;
        a.pool_pages = m->pool_pages;
        a.err = c->err_flag;
        VELO_CUDA_TRY(launch_tree_attention_f32(a, s));
        if (m->tp == 1) {
            VELO_CUDA_TRY(launch_gemm_f32(mat(ly.wo), m->attn32, M, H, Hq * D, m->x, H, kF32Add, s));
        } else {  // row-split o_proj: partial, all-reduce, residual add
            VELO_CUDA_TRY(launch_gemm_f32(mat(ly.wo), m->attn32, M, H, Hq * D, m->y, H, kF32Store, s));
            if ((st = allreduce_add(c, m, M))) return st;
        }
        VELO_CUDA_TRY(launch_rmsnorm_f32(m->x, ly.ffn_norm, M, H, eps, m->xn32, s));
        VELO_CUDA_TRY(launch_gemm_f32(mat(ly.w13), m->xn32, M, F, H, m->h32, F, kF32SwiGLU, s));
        if (m->tp == 1) {
            VELO_CUDA_TRY(launch_gemm_f32(mat(ly.w2), m->h32, M, H, F, m->x, H, kF32Add, s));
        } else {  // row-split down_proj
            VELO_CUDA_TRY(launch_gemm_f32(mat(ly.w2), m->h32, M, H, F, m->y, H, kF32Store, s));
            if ((st = allreduce_add(c, m, M))) return st;
        }
    }
    VELO_CUDA_TRY(launch_rmsnorm_f32(m->x, m->out_norm, M, H, eps, m->xn32, s));
    VELO_CUDA_TRY(launch_gemm_f32(mat(m->lm_head), m->xn32, M, m->V_loc, H, m->logits, m->V_loc,
                                  kF32Store, s));
    return VELO_OK;
}

// Write page-table row `slot`: ids pages[0..n), then `pad` (0: the rows
// velo_cuda_bind_slot leaves; an invalid id for a released slot).  Waits for
// the stream, so no step in flight still reads the old row.
int32_t write_row(velo_cuda_ctx* c, Model* m, uint32_t slot, const uint32_t* pages, size_t n, uint32_t pad) {
    uint32_t* row = m->page_table_host.data() + (size_t)slot * m->max_pages;
    for (int i = 0; i < m->max_pages; ++i) row[i] = (size_t)i < n ? pages[i] : pad;
    VELO_CUDA_TRY(cudaSetDevice(c->device));
    VELO_CUDA_TRY(cudaStreamSynchronize(c->stream));
    VELO_CUDA_TRY(cudaMemcpy(m->page_table + (size_t)slot * m->max_pages, row, (size_t)m->max_pages * 4,
                             cudaMemcpyHostToDevice));
    return VELO_OK;
}

int32_t check_model(velo_cuda_ctx* c) {
    if (!c) return fail(VELO_ERR_INVALID_ARGUMENT, "ctx is NULL");
    if (!c->model) return fail(VELO_ERR_INVALID_ARGUMENT, "no model loaded (velo_cuda_load_model)");
    return VELO_OK;
}

}  // namespace
}  // namespace velo

using velo::fail;
using velo::Model;

extern "C" {

int32_t velo_cuda_load_model(velo_cuda_ctx* c, const velo_model_desc* d, const velo_weight_desc* w,
                             int32_t n) {
    velo::Range nvtx_range("velo.load_model");
    velo::clear_last_error();
    if (!c || !d || (n > 0 && !w)) return fail(VELO_ERR_INVALID_ARGUMENT, "NULL argument");
    if (d->struct_size != 0 && d->struct_size != sizeof(velo_model_desc))
        return fail(VELO_ERR_INVALID_ARGUMENT, "velo_model_desc.struct_size %u != %zu", d->struct_size,
                    sizeof(velo_model_desc));
    // an f32 KV pool selects the fp32 path (any weight dtype, dequantised at load)
    const bool f32 = c->cfg.kv_dtype == VELO_KV_F32;
    if (d->n_head == 0 || d->n_head_kv == 0 || d->n_head % d->n_head_kv || d->n_vocab == 0 ||
        d->n_layer == 0)
        return fail(VELO_ERR_INVALID_ARGUMENT, "model shape unsupported: heads %u/%u, n_vocab %u, %u layers",
                    d->n_head, d->n_head_kv, d->n_vocab, d->n_layer);
    if (f32 && ((d->head_dim != 64 && d->head_dim != 128) || d->n_embd % 4 || d->n_ff % 4))
        return fail(VELO_ERR_INVALID_ARGUMENT,
                    "fp32 model shape unsupported: head_dim %u (64 or 128), n_embd %u and n_ff %u (by 4)",
                    d->head_dim, d->n_embd, d->n_ff);
    if (!f32 && (d->head_dim != 128 || d->n_embd % 128 || d->n_ff % 32))
        return fail(VELO_ERR_INVALID_ARGUMENT,
                    "q4_0 model shape unsupported: head_dim %u (128), n_embd %u (by 128), n_ff %u (by 32)",
                    d->head_dim, d->n_embd, d->n_ff);
    if (c->cfg.page_size != 16)
        return fail(VELO_ERR_INVALID_BLOCK_SIZE, "page_size %u: the kernels use 16-token pages",
                    c->cfg.page_size);
    const int tp = c->tp_size, rank = c->tp_rank;
    const uint32_t ff_align = f32 ? 4 : 32;
    if (tp > 1 && (d->n_head % tp || d->n_head_kv % tp || d->n_ff % tp || d->n_vocab % tp ||
                   (d->n_ff / tp) % ff_align))
        return fail(VELO_ERR_INVALID_ARGUMENT,
                    "heads %u/%u, n_ff %u and n_vocab %u must divide by tp %d (n_ff/tp by %u)",
                    d->n_head, d->n_head_kv, d->n_ff, d->n_vocab, tp, ff_align);
    VELO_CUDA_TRY(cudaSetDevice(c->device));
    velo::destroy_model(c->model);
    c->model = nullptr;
    Model* m = new Model();
    m->meta = *d;
    m->meta.struct_size = sizeof(velo_model_desc);
    m->tp = tp;
    m->rank = rank;
    m->f32 = f32;
    m->D = (int)d->head_dim;
    m->meta.n_head = d->n_head / tp;
    m->meta.n_head_kv = d->n_head_kv / tp;
    m->meta.n_ff = d->n_ff / tp;
    m->V_loc = (int)(d->n_vocab / tp);
    m->v_ofs = rank * m->V_loc;
    velo::Index ix;
    for (int i = 0; i < n; ++i)
        if (w[i].name) ix[w[i].name] = &w[i];
    // this rank's shard of a tensor (sharding.rs), kept alive until uploaded
    std::deque<std::vector<uint8_t>> bufs;
    std::deque<velo_weight_desc> descs;
    int32_t st = VELO_OK;
    auto shard = [&](const velo_weight_desc* wd, int32_t strategy) -> const velo_weight_desc* {
        if (!wd || st || tp == 1 || strategy == VELO_SHARD_REPLICATED) return wd;
        if (wd->flags & VELO_WEIGHT_SHARD) return wd;  // the caller's shard
        if (velo::on_device(wd)) {
            st = fail(VELO_ERR_INVALID_ARGUMENT, "device tensor %s must be passed as this rank's shard",
                      wd->name);
            return nullptr;
        }
        if (!wd->data || wd->dtype < VELO_DT_F32 || wd->dtype > VELO_DT_Q4_0) return wd;
        bufs.emplace_back();
        velo_weight_desc out = *wd;
        st = velo::shard_weight(*wd, strategy, tp, rank, bufs.back(), out.rows, out.cols);
        out.data = bufs.back().data();
        descs.push_back(out);
        return st ? nullptr : &descs.back();
    };
    // this rank's matrix `name`, which must have `rows` rows (after sharding)
    auto get_rows = [&](const std::string& name, uint64_t rows) -> const velo_weight_desc* {
        const velo_weight_desc* w = shard(velo::find(ix, name), velo::shard_strategy(name.c_str()));
        if (w && !st && w->rows != rows) {
            st = fail(VELO_ERR_INVALID_ARGUMENT, "matrix %s has %llu rows, this rank expects %llu",
                      name.c_str(), (unsigned long long)w->rows, (unsigned long long)rows);
            return nullptr;
        }
        return w;
    };
    const size_t H = d->n_embd, V = d->n_vocab, F = m->meta.n_ff;
    const size_t Dq = (size_t)m->meta.n_head * d->head_dim;
    cudaStream_t s = c->stream;
    const velo_weight_desc* emb = velo::find(ix, "token_embd.weight");
    if (!emb) st = fail(VELO_ERR_INVALID_ARGUMENT, "missing token_embd.weight");
    if (!st) st = velo::upload_f32(m, emb, V, H, &m->emb, s);
    if (!st) st = velo::upload_f32(m, velo::find(ix, "output_norm.weight"), 1, H, &m->out_norm, s);
    if (!st) {
        const velo_weight_desc* out = velo::find(ix, "output.weight");
        const velo_weight_desc* lm = shard(out ? out : emb, VELO_SHARD_COLUMN);  // tied fallback
        if (!st && lm && lm->rows != (uint64_t)m->V_loc)
            st = fail(VELO_ERR_INVALID_ARGUMENT, "LM head has %llu rows, this rank expects %d",
                      (unsigned long long)lm->rows, m->V_loc);
        if (!st) st = f32 ? velo::upload_f32_rows(m, {lm}, H, &m->lm_head, s)
                          : velo::upload_q4(m, {lm}, H, false, &m->lm_head, s);
    }
    auto upload = [&](const std::vector<const velo_weight_desc*>& parts, size_t cols, bool pair,
                      uint8_t** dst) {
        return f32 ? velo::upload_f32_rows(m, parts, cols, dst, s)
                   : velo::upload_q4(m, parts, cols, pair, dst, s);
    };
    for (uint32_t l = 0; !st && l < d->n_layer; ++l) {
        const std::string p = "layers." + std::to_string(l) + ".";
        velo::Layer ly;
        st = velo::upload_f32(m, velo::find(ix, p + "attention_norm.weight"), 1, H, &ly.attn_norm, s);
        if (!st) st = velo::upload_f32(m, velo::find(ix, p + "ffn_norm.weight"), 1, H, &ly.ffn_norm, s);
        if (!st) {
            const uint64_t Dk = (uint64_t)m->meta.n_head_kv * d->head_dim;
            auto* wq = get_rows(p + "attention.wq.weight", Dq);
            auto* wk = get_rows(p + "attention.wk.weight", Dk);
            auto* wv = get_rows(p + "attention.wv.weight", Dk);
            if (!st) st = upload({wq, wk, wv}, H, false, &ly.wqkv);
        }
        if (!st) {
            auto* wo = get_rows(p + "attention.wo.weight", H);
            if (!st) st = upload({wo}, Dq, false, &ly.wo);
        }
        if (!st) {
            auto* w1 = get_rows(p + "feed_forward.w1.weight", F);
            auto* w3 = get_rows(p + "feed_forward.w3.weight", F);
            if (!st) st = upload({w1, w3}, H, true, &ly.w13);
        }
        if (!st) {
            auto* w2 = get_rows(p + "feed_forward.w2.weight", H);
            if (!st) st = upload({w2}, F, false, &ly.w2);
        }
        m->layers.push_back(ly);
        bufs.clear();
        descs.clear();
    }
    // paged KV pool of the context config
    if (!st) {
        m->pool_pages = (int)(c->cfg.total_pages ? c->cfg.total_pages : 1);
        m->kv_int8 = c->cfg.kv_dtype == VELO_KV_INT8;
        m->max_slots = (int)c->cfg.max_slots;
        m->max_pages = (int)(c->cfg.max_pages_per_slot ? c->cfg.max_pages_per_slot : m->pool_pages);
        m->allocator = new velo::PageAllocator(16, (size_t)m->pool_pages);
        const size_t pe = (size_t)d->n_layer * m->layer_pool_elems();
        st = velo::dev_alloc(m, reinterpret_cast<uint8_t**>(&m->k_pool), pe * m->kv_elt());
        if (!st) st = velo::dev_alloc(m, reinterpret_cast<uint8_t**>(&m->v_pool), pe * m->kv_elt());
        if (!st && m->kv_int8) {
            const size_t se = (size_t)d->n_layer * m->layer_scale_elems();
            st = velo::dev_alloc(m, &m->k_scale, se * 2);
            if (!st) st = velo::dev_alloc(m, &m->v_scale, se * 2);
            if (!st) {
                cudaMemsetAsync(m->k_scale, 0, se * 2, s);
                cudaMemsetAsync(m->v_scale, 0, se * 2, s);
            }
        }
        if (!st) {
            cudaMemsetAsync(m->k_pool, 0, pe * m->kv_elt(), s);
            cudaMemsetAsync(m->v_pool, 0, pe * m->kv_elt(), s);
            m->page_table_host.assign((size_t)m->max_slots * m->max_pages, 0u);
            st = velo::dev_alloc(m, &m->page_table, m->page_table_host.size() * 4);
            if (!st) cudaMemsetAsync(m->page_table, 0, m->page_table_host.size() * 4, s);
        }
        if (!st) {
            cudaError_t e = cudaStreamSynchronize(s);
            if (e != cudaSuccess) st = fail(VELO_ERR_CUDA, "pool init failed: %s", cudaGetErrorString(e));
        }
    }
    if (st) {
        velo::destroy_model(m);
        return st;
    }
    c->model = m;
    return VELO_OK;
}

int32_t velo_cuda_bind_slot(velo_cuda_ctx* c, uint32_t slot, const uint32_t* pages, size_t n) {
    velo::clear_last_error();
    int32_t st = velo::check_model(c);
    if (st) return st;
    Model* m = c->model;
    if (slot >= (uint32_t)m->max_slots)
        return fail(VELO_ERR_INVALID_ARGUMENT, "slot %u >= max_slots %d", slot, m->max_slots);
    if (n > (size_t)m->max_pages)
        return fail(VELO_ERR_OUT_OF_PAGES, "OutOfPages { requested: %zu, available: %d }", n, m->max_pages);
    if (n && !pages) return fail(VELO_ERR_INVALID_ARGUMENT, "pages is NULL");
    for (size_t i = 0; i < n; ++i)
        if (pages[i] >= (uint32_t)m->pool_pages)
            return fail(VELO_ERR_OUT_OF_PAGES, "page id %u >= pool of %d pages", pages[i], m->pool_pages);
    return velo::write_row(c, m, slot, pages, n, 0u);
}

int32_t velo_cuda_slot_allocate(velo_cuda_ctx* c, uint32_t slot, size_t token_len, uint32_t* pages_out,
                                size_t pages_cap, size_t* n_pages) {
    velo::clear_last_error();
    int32_t st = velo::check_model(c);
    if (st) return st;
    Model* m = c->model;
    if (slot >= (uint32_t)m->max_slots)
        return fail(VELO_ERR_INVALID_ARGUMENT, "slot %u >= max_slots %d", slot, m->max_slots);
    const size_t req = m->allocator->pages_for_tokens(token_len);
    if (req > (size_t)m->max_pages)
        return fail(VELO_ERR_OUT_OF_PAGES, "OutOfPages { requested: %zu, available: %d } (page-table row)",
                    req, m->max_pages);
    if (pages_out && pages_cap < req)
        return fail(VELO_ERR_INVALID_ARGUMENT, "pages_out holds %zu ids, %zu needed", pages_cap, req);
    std::vector<uint32_t> got;
    size_t rq = 0, av = 0;
    st = m->allocator->allocate(slot, token_len, &got, &rq, &av);
    if (st) return fail(st, "OutOfPages { requested: %zu, available: %zu }", rq, av);
    st = velo::write_row(c, m, slot, got.data(), got.size(), 0u);
    if (st) return st;
    if (n_pages) *n_pages = got.size();
    if (pages_out)
        for (size_t i = 0; i < got.size(); ++i) pages_out[i] = got[i];
    return VELO_OK;
}

int32_t velo_cuda_slot_release(velo_cuda_ctx* c, uint32_t slot) {
    velo::clear_last_error();
    int32_t st = velo::check_model(c);
    if (st) return st;
    Model* m = c->model;
    if (slot >= (uint32_t)m->max_slots)
        return fail(VELO_ERR_INVALID_ARGUMENT, "slot %u >= max_slots %d", slot, m->max_slots);
    if (!m->allocator->mapped(slot)) return fail(VELO_ERR_UNKNOWN_HANDLE, "UnknownHandle(%u)", slot);
    // unbind first: the pages go back only once no row names them
    st = velo::write_row(c, m, slot, nullptr, 0, 0xffffffffu);
    if (st) return st;
    return m->allocator->release(slot);
}

int32_t velo_cuda_free_pages(velo_cuda_ctx* c, size_t* out) {
    velo::clear_last_error();
    const int32_t st = velo::check_model(c);
    if (st) return st;
    if (!out) return fail(VELO_ERR_INVALID_ARGUMENT, "out is NULL");
    *out = c->model->allocator->free_pages();
    return VELO_OK;
}

int32_t velo_cuda_write_kv(velo_cuda_ctx* c, uint32_t slot, int32_t layer, int32_t pos0, int32_t n,
                           const void* k, const void* v) {
    velo::Range nvtx_range("velo.write_kv");
    velo::clear_last_error();
    int32_t st = velo::check_model(c);
    if (st) return st;
    Model* m = c->model;
    if (slot >= (uint32_t)m->max_slots || layer < 0 || layer >= m->L() || pos0 < 0 || n < 0 ||
        n > velo::kAttnMaxNodes || (n && (!k || !v)))
        return fail(VELO_ERR_INVALID_ARGUMENT, "write_kv: slot %u layer %d pos0 %d n %d (n <= 64)", slot,
                    layer, pos0, n);
    if (n == 0) return VELO_OK;
    if ((pos0 + n - 1) / 16 >= m->max_pages)
        return fail(VELO_ERR_OUT_OF_PAGES, "write_kv: position %d beyond the page-table row", pos0 + n - 1);
    VELO_CUDA_TRY(cudaSetDevice(c->device));
    const size_t rows = (size_t)n * m->Hkv() * m->D;
    const size_t in_elt = m->f32 ? 4 : 2;  // host rows: f32 for f32 pools, else f16
    uint8_t* dk = nullptr;
    VELO_CUDA_TRY(cudaMalloc(&dk, rows * in_elt * 2 + 64 * 4 * 4));
    uint8_t* dv = dk + rows * in_elt;
    int32_t* meta = reinterpret_cast<int32_t*>(dv + rows * in_elt);  // path[64], len, ctx, slot
    std::vector<int32_t> hm(64 + 3);
    for (int i = 0; i < 64; ++i) hm[i] = i < n ? i : -1;
    hm[64] = n;
    hm[65] = pos0;
    hm[66] = (int32_t)slot;
    cudaError_t e = cudaMemcpy(dk, k, rows * in_elt, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(dv, v, rows * in_elt, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(meta, hm.data(), hm.size() * 4, cudaMemcpyHostToDevice);
    const size_t lo = (size_t)layer * m->layer_pool_elems() * m->kv_elt();
    if (e == cudaSuccess && m->f32) {
        velo::KvCommitF32Args a{};
        a.node_k = reinterpret_cast<const float*>(dk);
        a.node_v = reinterpret_cast<const float*>(dv);
        a.path = meta;
        a.path_len = meta + 64;
        a.ctx_len = meta + 65;
        a.slots = reinterpret_cast<const uint32_t*>(meta + 66);
        a.page_table = m->page_table;
        a.k_pool = reinterpret_cast<float*>(static_cast<uint8_t*>(m->k_pool) + lo);
        a.v_pool = reinterpret_cast<float*>(static_cast<uint8_t*>(m->v_pool) + lo);
        a.B = 1;
        a.N = n;
        a.L = 1;
        a.Hkv = m->Hkv();
        a.D = m->D;
        a.max_pages = m->max_pages;
        a.pool_pages = m->pool_pages;
        a.err = c->err_flag;
        e = velo::launch_kv_commit_f32(a, c->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    } else if (e == cudaSuccess) {
        velo::KvCommitArgs a{};
        a.node_k = reinterpret_cast<const __half*>(dk);
        a.node_v = reinterpret_cast<const __half*>(dv);
        a.path = meta;
        a.path_len = meta + 64;
        a.ctx_len = meta + 65;
        a.slots = reinterpret_cast<const uint32_t*>(meta + 66);
        a.page_table = m->page_table;
        a.k_pool = static_cast<uint8_t*>(m->k_pool) + lo;
        a.v_pool = static_cast<uint8_t*>(m->v_pool) + lo;
        a.k_scale = m->kv_int8 ? m->k_scale + (size_t)layer * m->layer_scale_elems() : nullptr;
        a.v_scale = m->kv_int8 ? m->v_scale + (size_t)layer * m->layer_scale_elems() : nullptr;
        a.B = 1;
        a.N = n;
        a.L = 1;
        a.Hkv = m->Hkv();
        a.max_pages = m->max_pages;
        a.pool_pages = m->pool_pages;
        a.kv_int8 = m->kv_int8;
        a.err = c->err_flag;
        e = velo::launch_kv_commit(a, c->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    }
    cudaFree(dk);
    if (e != cudaSuccess) return fail(VELO_ERR_CUDA, "write_kv failed: %s", cudaGetErrorString(e));
    return velo_cuda_sync(c, -1);
}

int32_t velo_cuda_read_kv(velo_cuda_ctx* c, uint32_t slot, int32_t layer, int32_t pos0, int32_t n,
                          void* k_out, void* v_out, void* ks_out, void* vs_out) {
    velo::clear_last_error();
    int32_t st = velo::check_model(c);
    if (st) return st;
    Model* m = c->model;
    if (slot >= (uint32_t)m->max_slots || layer < 0 || layer >= m->L() || pos0 < 0 || n < 0 ||
        (n && (!k_out || !v_out)))
        return fail(VELO_ERR_INVALID_ARGUMENT, "read_kv: bad arguments");
    if (n && (pos0 + n - 1) / 16 >= m->max_pages)
        return fail(VELO_ERR_OUT_OF_PAGES, "read_kv: position beyond the page-table row");
    VELO_CUDA_TRY(cudaSetDevice(c->device));
    VELO_CUDA_TRY(cudaStreamSynchronize(c->stream));
    const uint32_t* row = m->page_table_host.data() + (size_t)slot * m->max_pages;
    const size_t hd = m->D, tokb = hd * m->kv_elt();
    for (int i = 0; i < n; ++i) {
        const int pos = pos0 + i;
        const uint32_t pg = row[pos / 16];
        for (int h = 0; h < m->Hkv(); ++h) {
            const size_t tok = (((size_t)layer * m->pool_pages + pg) * m->Hkv() + h) * 16 + pos % 16;
            const size_t o = ((size_t)i * m->Hkv() + h);
            VELO_CUDA_TRY(cudaMemcpy(static_cast<uint8_t*>(k_out) + o * tokb,
                                     static_cast<uint8_t*>(m->k_pool) + tok * tokb, tokb, cudaMemcpyDeviceToHost));
            VELO_CUDA_TRY(cudaMemcpy(static_cast<uint8_t*>(v_out) + o * tokb,
                                     static_cast<uint8_t*>(m->v_pool) + tok * tokb, tokb, cudaMemcpyDeviceToHost));
            if (m->kv_int8 && ks_out)
                VELO_CUDA_TRY(cudaMemcpy(static_cast<uint16_t*>(ks_out) + o, m->k_scale + tok, 2, cudaMemcpyDeviceToHost));
            if (m->kv_int8 && vs_out)
                VELO_CUDA_TRY(cudaMemcpy(static_cast<uint16_t*>(vs_out) + o, m->v_scale + tok, 2, cudaMemcpyDeviceToHost));
        }
    }
    return VELO_OK;
}

int32_t velo_cuda_verify_step(velo_cuda_ctx* c, const velo_verify_batch* in, velo_verify_result* out) {
    velo::Range nvtx_range("velo.verify_step");
    velo::clear_last_error();
    int32_t st = velo::check_model(c);
    if (st) return st;
    if (!in || !out) return fail(VELO_ERR_INVALID_ARGUMENT, "NULL batch / result");
    if (in->struct_size != 0 && in->struct_size != sizeof(velo_verify_batch))
        return fail(VELO_ERR_INVALID_ARGUMENT, "velo_verify_batch.struct_size %u != %zu", in->struct_size,
                    sizeof(velo_verify_batch));
    Model* m = c->model;
    const int B = in->B, N = in->n_nodes;
    if (B < 0) return fail(VELO_ERR_INVALID_ARGUMENT, "B = %d", B);
    if (N < 1) return fail(VELO_ERR_EMPTY_DRAFT_WINDOW, "n_nodes = %d: a verify step needs the root node", N);
    if (N > velo::kAttnMaxNodes)
        return fail(VELO_ERR_DRAFT_TOO_MANY, "n_nodes = %d > %d", N, velo::kAttnMaxNodes);
    if (B == 0) return VELO_OK;
    if (!in->slots || !in->ctx_len || !in->tokens || !in->parents || !out->accepted_len || !out->bonus_token)
        return fail(VELO_ERR_INVALID_ARGUMENT, "NULL batch array");
    const bool sampling = in->temperature > 0.0f;
    if (!(in->temperature >= 0.0f) || std::isinf(in->temperature))
        return fail(VELO_ERR_INVALID_ARGUMENT, "temperature must be finite and >= 0");
    if (in->commit < 0 || in->commit > 2 || (in->commit == 2 && sampling))
        return fail(VELO_ERR_INVALID_ARGUMENT, "commit mode %d (0, 1 or 2; 2 is greedy only)", in->commit);
    const int V = m->V();
    bool chains = true;  // every sequence a chain: sampling takes the chain kernels
    for (int b = 0; b < B; ++b) {
        if (in->slots[b] >= (uint32_t)m->max_slots)
            return fail(VELO_ERR_INVALID_ARGUMENT, "slot %u >= max_slots", in->slots[b]);
        if (in->ctx_len[b] < 0) return fail(VELO_ERR_INVALID_ARGUMENT, "ctx_len[%d] < 0", b);
        const int last = in->ctx_len[b] + N - 1;  // deepest possible position
        if (in->ctx_len[b] > m->max_pages * 16 || (in->commit && last / 16 >= m->max_pages))
            return fail(VELO_ERR_OUT_OF_PAGES, "OutOfPages: sequence %d needs position %d, row holds %d", b,
                        last, m->max_pages * 16);
        if (in->parents[(size_t)b * N] != -1)
            return fail(VELO_ERR_INVALID_ARGUMENT, "node 0 of sequence %d must be the root (parent -1)", b);
        for (int i = 1; i < N; ++i) {
            const int p = in->parents[(size_t)b * N + i];
            if (p < 0 || p >= i) return fail(VELO_ERR_INVALID_ARGUMENT, "parents[%d][%d] = %d", b, i, p);
            if (in->commit == 2 && p != i - 1)
                return fail(VELO_ERR_INVALID_ARGUMENT, "commit of every node takes chains only (parents[n] = n-1)");
            if (p != i - 1) chains = false;
        }
        for (int i = 0; i < N; ++i)
            if (in->tokens[(size_t)b * N + i] >= (uint32_t)V)
                return fail(VELO_ERR_INVALID_ARGUMENT, "token %u >= n_vocab", in->tokens[(size_t)b * N + i]);
    }
    if (sampling && N > 1 && (!in->draft_logits || !in->uniforms))
        return fail(VELO_ERR_INVALID_ARGUMENT, "sampling needs draft_logits and uniforms");
    VELO_CUDA_TRY(cudaSetDevice(c->device));
    st = velo::ensure_work(c, m, B, N);
    if (st) return st;
    cudaStream_t s = c->stream;
    const int M = B * N, H = m->H(), Hq = m->Hq(), Hkv = m->Hkv(), F = m->F(), L = m->L();
    const int Nqkv = (Hq + 2 * Hkv) * 128;
    // inputs and the batch's page-table rows: packed into pinned memory, one copy
    const size_t mp = (size_t)m->max_pages;
    m->tokens = reinterpret_cast<uint32_t*>(m->din);
    m->parents = reinterpret_cast<int32_t*>(m->tokens + M);
    m->ctxlen = m->parents + M;
    m->slots = reinterpret_cast<uint32_t*>(m->ctxlen + B);
    m->pt_batch = m->slots + B;
    m->path_len = reinterpret_cast<int32_t*>(m->dout);
    m->bonus = reinterpret_cast<uint32_t*>(m->path_len + B);
    m->path = reinterpret_cast<int32_t*>(m->bonus + B);
    m->expected = reinterpret_cast<uint32_t*>(m->path + M);
    if (m->staging_busy) VELO_CUDA_TRY(cudaStreamSynchronize(s));  // an earlier step ended early
    m->staging_busy = true;
    {
        uint32_t* h = reinterpret_cast<uint32_t*>(m->hin);
        std::memcpy(h, in->tokens, (size_t)M * 4);
        std::memcpy(h + M, in->parents, (size_t)M * 4);
        std::memcpy(h + 2 * M, in->ctx_len, (size_t)B * 4);
        std::memcpy(h + 2 * M + B, in->slots, (size_t)B * 4);
        for (int b = 0; b < B; ++b)
            std::memcpy(h + 2 * M + 2 * B + (size_t)b * mp,
                        m->page_table_host.data() + (size_t)in->slots[b] * mp, mp * 4);
        VELO_CUDA_TRY(cudaMemcpyAsync(m->din, m->hin, ((size_t)2 * M + 2 * B + B * mp) * 4,
                                      cudaMemcpyHostToDevice, s));
    }
    const int Vl = m->V_loc;
    // the launch sequence of the step, from the ancestor masks to the KV commit
    auto body = [&]() -> int32_t {
    int32_t st = VELO_OK;
    VELO_CUDA_TRY(velo::prof_mark(c, m, VELO_PHASE_OTHER));
    VELO_CUDA_TRY(velo::launch_tree_ancestors(m->parents, B, N, m->anc, c->err_flag, s));
    VELO_CUDA_TRY(velo::launch_embed(m->emb, m->tokens, M, H, m->V(), m->x, c->err_flag, s));
    const float eps = m->meta.norm_eps;
    if (m->f32) {
        st = velo::forward_f32(c, m, B, N);
        if (st) return st;
    }
    // With tp > 1 a row-split GEMM (o_proj, down_proj) leaves its bf16 partial
    // in ybf, the group sums it in place, and the RMSNorm that follows adds it
    // to the residual stream (`pending`).
    bool pending = false;
    auto norm = [&](const float* w) -> cudaError_t {
        cudaError_t e = velo::prof_mark(c, m, VELO_PHASE_OTHER);
        if (e != cudaSuccess) return e;
        if (!pending) return velo::launch_rmsnorm_f16(m->x, w, M, H, eps, m->xn, s);
        pending = false;
        if (velo::use_ce_sum(m))
            return velo::launch_add_rmsnorm_blocked_f16(m->x, m->ybf, H / m->tp, (size_t)m->cap_M * (H / m->tp), w, M,
                                                        H, eps, m->xn, s);
        return velo::launch_add_rmsnorm_f16(m->x, m->ybf, w, M, H, eps, m->xn, s);
    };
    auto row_split = [&](const uint8_t* w, const __half* in, int K, int phase) -> int32_t {
        VELO_CUDA_TRY(velo::prof_mark(c, m, phase));
        if (m->tp == 1) return velo::gemm(c, w, in, M, H, K, m->x, H, velo::kEpiAddF32);
        if (velo::use_ce_sum(m)) {
            int32_t r = velo::ce_gemm(c, m, s, w, in, M, K, 0);
            if (r) return r;
            VELO_CUDA_TRY(velo::prof_mark(c, m, VELO_PHASE_ALLREDUCE));
            pending = true;
            return velo::ce_sum(c, m, s, M, 0, 0);
        }
        if (velo::use_fused_sum(m)) {
            // the GEMM pushes the partial to the column blocks' owners; the phase
            // after it is the gather kernel
            int32_t r = velo::gemm_push(c, m, s, w, in, M, K, 0);
            if (r) return r;
            VELO_CUDA_TRY(velo::prof_mark(c, m, VELO_PHASE_ALLREDUCE));
            pending = true;
            return velo::gather_sum(c, m, s, M, 0, 0);
        }
        int32_t r = velo::gemm(c, w, in, M, H, K, m->ybf, H, velo::kEpiStoreBF16);
        if (r) return r;
        VELO_CUDA_TRY(velo::prof_mark(c, m, VELO_PHASE_ALLREDUCE));
        pending = true;
        return velo::allreduce_bf16(c, m, M);
    };
    // tensor parallel with a second communicator: the two-stream loop (which
    // also leaves the final RMSNorm in xn); profiled steps keep one stream so
    // each phase can be timed
    const char* ov = std::getenv("VELO_TP_OVERLAP");
    const bool halves = m->tp > 1 && !m->f32 && c->nccl_comm2 && B >= 2 && !m->profile &&
                        !(ov && std::strcmp(ov, "0") == 0);
    if (halves) {
        st = velo::forward_tp_halves(c, m, B, N);
        if (st) return st;
    }
    for (int l = 0; !m->f32 && !halves && l < L; ++l) {
        const velo::Layer& ly = m->layers[l];
        __half* nk = m->nk + (size_t)l * M * Hkv * 128;
        __half* nv = m->nv + (size_t)l * M * Hkv * 128;
        VELO_CUDA_TRY(norm(ly.attn_norm));
        VELO_CUDA_TRY(velo::prof_mark(c, m, VELO_PHASE_GEMM_QKV));
        st = velo::gemm(c, ly.wqkv, m->xn, M, Nqkv, H, m->qkv, Nqkv, velo::kEpiStoreF32);
        if (st) return st;
        VELO_CUDA_TRY(velo::prof_mark(c, m, VELO_PHASE_OTHER));
        VELO_CUDA_TRY(velo::launch_rope_split(m->qkv, m->anc, m->ctxlen, B, N, Hq, Hkv, m->meta.rope_freq_base,
                                              m->q, nk, nv, s));
        velo::TreeAttnArgs a{};
        const size_t lo = (size_t)l * m->layer_pool_elems() * m->kv_elt();
        a.q = m->q;
        a.k_pool = static_cast<uint8_t*>(m->k_pool) + lo;
        a.v_pool = static_cast<uint8_t*>(m->v_pool) + lo;
        a.k_scale = m->kv_int8 ? m->k_scale + (size_t)l * m->layer_scale_elems() : nullptr;
        a.v_scale = m->kv_int8 ? m->v_scale + (size_t)l * m->layer_scale_elems() : nullptr;
        a.page_table = m->pt_batch;
        a.ctx_len = m->ctxlen;
        a.node_k = nk;
        a.node_v = nv;
        a.anc = m->anc;
        a.out = m->attn;
        a.out_f16 = 1;
        a.B = B;
        a.N = N;
        a.Hq = Hq;
        a.Hkv = Hkv;
        a.max_pages = m->max_pages;
        a.pool_pages = m->pool_pages;
        a.scale_log2 = (float)(1.4426950408889634 / std::sqrt(128.0));
        a.err = c->err_flag;
        VELO_CUDA_TRY(velo::prof_mark(c, m, VELO_PHASE_ATTENTION));
        VELO_CUDA_TRY(velo::launch_tree_attention(a, m->kv_int8 != 0, s));
        st = row_split(ly.wo, m->attn, Hq * 128, VELO_PHASE_GEMM_O);
        if (st) return st;
        VELO_CUDA_TRY(norm(ly.ffn_norm));
        VELO_CUDA_TRY(velo::prof_mark(c, m, VELO_PHASE_GEMM_FFN_UP));
        st = velo::gemm(c, ly.w13, m->xn, M, 2 * F, H, m->hbuf, F, velo::kEpiSwiGLU);
        if (!st) st = row_split(ly.w2, m->hbuf, F, VELO_PHASE_GEMM_FFN_DOWN);
        if (st) return st;
    }
    if (!m->f32) {
        if (!halves) VELO_CUDA_TRY(norm(m->out_norm));
        VELO_CUDA_TRY(velo::prof_mark(c, m, VELO_PHASE_LM_HEAD));
        st = velo::gemm(c, m->lm_head, m->xn, M, Vl, H, m->logits, Vl, velo::kEpiStoreF32);
        if (st) return st;
    }
    VELO_CUDA_TRY(velo::prof_mark(c, m, VELO_PHASE_ACCEPT_COMMIT));
    // acceptance
    velo::Range accept_range("velo.verify_step.accept_commit");
    if (m->tp > 1 && (!sampling || N == 1)) {
        // vocabulary-sharded greedy: per-shard maxima, gathered, combined
        const velo::NcclApi* nc = velo::nccl_api();
        if (!nc) return VELO_ERR_NCCL;
        VELO_CUDA_TRY(velo::launch_row_argmax_pairs(m->logits, M, Vl, m->v_ofs, m->pairs, s));
        st = velo::nccl_check(nc->AllGather(m->pairs, m->pairs_all, (size_t)M * 2, ncclInt32,
                                            static_cast<ncclComm_t>(c->nccl_comm), s),
                              nc, "ncclAllGather");
        if (st) return st;
        VELO_CUDA_TRY(velo::launch_argmax_combine(m->pairs_all, m->tp, M, m->expected, s));
        VELO_CUDA_TRY(velo::launch_tree_walk(m->tokens, m->parents, m->expected, B, N, m->path,
                                             m->path_len, m->bonus, s));
    } else if (!sampling || N == 1) {
        VELO_CUDA_TRY(velo::launch_tree_greedy(m->logits, m->tokens, m->parents, B, N, V, m->expected,
                                               m->path, m->path_len, m->bonus, s));
    } else {
        // Sampling.  With tp > 1 every rank reassembles the full target rows
        // and runs the same acceptance on the replicated draft logits and
        // uniforms, so all ranks reach the same decisions as one GPU would
        // on those rows (the rows are M x V f32, a few MB per step).
        const float* tgt = m->logits;
        if (m->tp > 1) {
            st = velo::gather_full_logits(c, m, M, true);
            if (st) return st;
            tgt = m->logits_full;
        }
        const int k = N - 1;
        const size_t need = (size_t)B * k * V;
        if (need > m->drf_cap) {
            VELO_CUDA_TRY(cudaStreamSynchronize(s));
            if (m->drf) cudaFree(m->drf);
            m->drf = nullptr;
            m->drf_cap = 0;
            VELO_CUDA_TRY(cudaMalloc(&m->drf, need * 4));
            m->drf_cap = need;
        }
        if (!chains) {
            // trees: the walk, residuals and draw on the device, no host round trip
            VELO_CUDA_TRY(cudaMemcpyAsync(m->drf, in->draft_logits, need * 4, cudaMemcpyHostToDevice, s));
            VELO_CUDA_TRY(cudaMemcpyAsync(m->uni, in->uniforms, (size_t)B * N * 4, cudaMemcpyHostToDevice, s));
            velo::AcceptTreeParams tp{};
            tp.tgt = tgt;
            tp.drf = m->drf;
            tp.tok = m->tokens;
            tp.par = m->parents;
            tp.u = m->uni;
            tp.path = m->path;
            tp.path_len = m->path_len;
            tp.bonus = m->bonus;
            tp.err_flag = c->err_flag;
            tp.B = B;
            tp.N = N;
            tp.V = V;
            tp.inv_t = 1.0f / in->temperature;
            tp.vec4 = (V % 4) == 0;
            VELO_CUDA_TRY(velo::launch_accept_tree(tp, s));
            goto sampled;
        }
        {
        std::vector<uint32_t> dt((size_t)B * k);
        for (int b = 0; b < B; ++b)
            for (int i = 0; i < k; ++i) dt[(size_t)b * k + i] = in->tokens[(size_t)b * N + i + 1];
        VELO_CUDA_TRY(cudaMemcpyAsync(m->drf, in->draft_logits, need * 4, cudaMemcpyHostToDevice, s));
        VELO_CUDA_TRY(cudaMemcpyAsync(m->uni, in->uniforms, (size_t)B * N * 4, cudaMemcpyHostToDevice, s));
        VELO_CUDA_TRY(cudaMemcpyAsync(m->dtok, dt.data(), dt.size() * 4, cudaMemcpyHostToDevice, s));
        VELO_CUDA_TRY(cudaStreamSynchronize(s));  // dt is host-stack memory
        st = velo::run_accept(c, tgt, m->drf, m->dtok, m->uni, B, k, V, in->temperature, m->acc, m->bonus);
        if (st) return st;
        // chain path: nodes 0..acc
        std::vector<int32_t> acc(B);
        VELO_CUDA_TRY(cudaMemcpyAsync(acc.data(), m->acc, (size_t)B * 4, cudaMemcpyDeviceToHost, s));
        VELO_CUDA_TRY(cudaStreamSynchronize(s));
        std::vector<int32_t> path((size_t)M, -1), plen(B);
        for (int b = 0; b < B; ++b) {
            plen[b] = acc[b] + 1;
            for (int i = 0; i < plen[b]; ++i) path[(size_t)b * N + i] = i;
        }
        VELO_CUDA_TRY(cudaMemcpyAsync(m->path, path.data(), path.size() * 4, cudaMemcpyHostToDevice, s));
        VELO_CUDA_TRY(cudaMemcpyAsync(m->path_len, plen.data(), plen.size() * 4, cudaMemcpyHostToDevice, s));
        VELO_CUDA_TRY(cudaStreamSynchronize(s));
        }
    sampled:;
    }
    if (in->commit == 2) {
        // prefill / draft decode: the whole chain is committed and reported as
        // accepted; the bonus is the argmax after the last node
        VELO_CUDA_TRY(velo::launch_chain_commit(m->expected, B, N, m->path, m->path_len, m->bonus, s));
    }
    if (in->commit && m->f32) {
        velo::KvCommitF32Args a{};
        a.node_k = m->nk32;
        a.node_v = m->nv32;
        a.path = m->path;
        a.path_len = m->path_len;
        a.ctx_len = m->ctxlen;
        a.slots = m->slots;
        a.page_table = m->page_table;
        a.k_pool = static_cast<float*>(m->k_pool);
        a.v_pool = static_cast<float*>(m->v_pool);
        a.B = B;
        a.N = N;
        a.L = L;
        a.Hkv = Hkv;
        a.D = m->D;
        a.max_pages = m->max_pages;
        a.pool_pages = m->pool_pages;
        a.err = c->err_flag;
        VELO_CUDA_TRY(velo::launch_kv_commit_f32(a, s));
    } else if (in->commit) {
        velo::KvCommitArgs a{};
        a.node_k = m->nk;
        a.node_v = m->nv;
        a.path = m->path;
        a.path_len = m->path_len;
        a.ctx_len = m->ctxlen;
        a.slots = m->slots;
        a.page_table = m->page_table;
        a.k_pool = m->k_pool;
        a.v_pool = m->v_pool;
        a.k_scale = m->k_scale;
        a.v_scale = m->v_scale;
        a.B = B;
        a.N = N;
        a.L = L;
        a.Hkv = Hkv;
        a.max_pages = m->max_pages;
        a.pool_pages = m->pool_pages;
        a.kv_int8 = m->kv_int8;
        a.err = c->err_flag;
        VELO_CUDA_TRY(velo::launch_kv_commit(a, s));
    }
    VELO_CUDA_TRY(velo::prof_mark(c, m, -1));  // end of the step
    return st;
    };  // body

    // Greedy single-GPU steps replay a captured graph of the body (one
    // launch instead of ~25); sampling (host round trip) and tensor-parallel
    // steps run it directly.
    const bool graphable = m->tp == 1 && !(sampling && N > 1) && !m->graphs_off && !m->profile;
    if (graphable) {
        const uint64_t key = ((uint64_t)B << 32) | ((uint64_t)N << 8) | (uint64_t)in->commit;
        auto it = m->graphs.find(key);
        if (it == m->graphs.end()) {
            if (cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
                cudaGetLastError();
                m->graphs_off = true;  // e.g. the legacy default stream: launch directly
                st = body();
                if (st) return st;
            } else {
                const int32_t bst = body();
                cudaGraph_t g = nullptr;
                const cudaError_t e = cudaStreamEndCapture(s, &g);
                if (bst) {
                    if (g) cudaGraphDestroy(g);
                    return bst;
                }
                if (e != cudaSuccess) return fail(VELO_ERR_CUDA, "graph capture: %s", cudaGetErrorString(e));
                cudaGraphExec_t exec = nullptr;
                const cudaError_t ei = cudaGraphInstantiate(&exec, g, 0);
                cudaGraphDestroy(g);
                if (ei != cudaSuccess) return fail(VELO_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(ei));
                it = m->graphs.emplace(key, exec).first;
            }
        }
        if (it != m->graphs.end()) VELO_CUDA_TRY(cudaGraphLaunch(it->second, s));
    } else {
        st = body();
        if (st) return st;
    }
    // path_len | bonus | path | expected: one copy into pinned memory
    const bool want_expected = out->expected && (!sampling || N == 1);
    VELO_CUDA_TRY(cudaMemcpyAsync(m->hout, m->dout, ((size_t)2 * B + (want_expected ? 2 : 1) * M) * 4,
                                  cudaMemcpyDeviceToHost, s));
    std::vector<float> gathered;
    if (out->logits && m->tp == 1)
        VELO_CUDA_TRY(cudaMemcpyAsync(out->logits, m->logits, (size_t)M * V * 4, cudaMemcpyDeviceToHost, s));
    const bool have_full = m->tp > 1 && sampling && N > 1;  // reassembled by the body
    if (out->logits && have_full)
        VELO_CUDA_TRY(cudaMemcpyAsync(out->logits, m->logits_full, (size_t)M * V * 4, cudaMemcpyDeviceToHost, s));
    if (out->logits && m->tp > 1 && !have_full) {
        const size_t per = (size_t)M * Vl;
        st = velo::gather_full_logits(c, m, M, false);
        if (st) return st;
        gathered.resize(per * m->tp);
        VELO_CUDA_TRY(cudaMemcpyAsync(gathered.data(), m->logits_all, per * m->tp * 4, cudaMemcpyDeviceToHost, s));
    }
    st = velo_cuda_sync(c, -1);
    if (st) return st;
    m->staging_busy = false;
    velo::prof_collect(m);
    if (!gathered.empty())  // [tp][M][Vl] -> [M][V]
        for (int r = 0; r < m->tp; ++r)
            for (int i = 0; i < M; ++i)
                std::memcpy(out->logits + (size_t)i * V + (size_t)r * Vl,
                            gathered.data() + ((size_t)r * M + i) * Vl, (size_t)Vl * 4);
    const int32_t* hp = reinterpret_cast<const int32_t*>(m->hout);
    for (int b = 0; b < B; ++b) out->accepted_len[b] = hp[b] - 1;
    std::memcpy(out->bonus_token, hp + B, (size_t)B * 4);
    if (out->accepted_nodes) std::memcpy(out->accepted_nodes, hp + 2 * B, (size_t)M * 4);
    if (want_expected) std::memcpy(out->expected, hp + 2 * B + M, (size_t)M * 4);
    return VELO_OK;
}

int32_t velo_cuda_profile(velo_cuda_ctx* c, int32_t enable) {
    velo::clear_last_error();
    int32_t st = velo::check_model(c);
    if (st) return st;
    Model* m = c->model;
    m->profile = enable != 0;
    m->prof_n = 0;
    m->prof_steps = 0;
    for (double& v : m->prof_ms) v = 0.0;
    return VELO_OK;
}

int32_t velo_cuda_profile_read(velo_cuda_ctx* c, double* ms, int32_t n, int32_t* steps) {
    velo::clear_last_error();
    int32_t st = velo::check_model(c);
    if (st) return st;
    if (!ms || n < VELO_PHASE_COUNT)
        return fail(VELO_ERR_INVALID_ARGUMENT, "profile_read needs %d slots", (int)VELO_PHASE_COUNT);
    for (int i = 0; i < VELO_PHASE_COUNT; ++i) ms[i] = c->model->prof_ms[i];
    if (steps) *steps = c->model->prof_steps;
    return VELO_OK;
}

int32_t velo_cuda_tp_sum_path(velo_cuda_ctx* c, int32_t* path) {
    velo::clear_last_error();
    int32_t st = velo::check_model(c);
    if (st) return st;
    if (!path) return fail(VELO_ERR_INVALID_ARGUMENT, "tp_sum_path: null output");
    const Model* m = c->model;
    *path = m->tp < 2 || m->f32         ? VELO_TP_SUM_NONE
            : velo::use_ce_sum(m)    ? VELO_TP_SUM_CE
            : velo::use_fused_sum(m) ? VELO_TP_SUM_FUSED
            : velo::use_peer_sum(m)  ? VELO_TP_SUM_PEER
                                     : VELO_TP_SUM_NCCL;
    return VELO_OK;
}

// The peer-sum barriers' time limit, exercised on one GPU: a gather call of rank 0
// in a group of 2 whose rank 1 never arrives (its flag block is memory nothing
// writes).  The entry wait and the exit wait each give up after 2 s; *code gets the
// first error the kernel recorded (0x7101: entry).
int32_t velo_cuda_tp_wait_selftest(int32_t device, int32_t* code) {
    velo::clear_last_error();
    if (!code) return fail(VELO_ERR_INVALID_ARGUMENT, "tp_wait_selftest: null output");
    VELO_CUDA_TRY(cudaSetDevice(device));
    unsigned long long* flags = nullptr;
    int* err = nullptr;
    __nv_bfloat16* buf = nullptr;
    cudaStream_t s = nullptr;
    int32_t st = VELO_OK;
    auto check = [&](cudaError_t e) {
        if (e != cudaSuccess && !st) st = fail(VELO_ERR_CUDA, "tp_wait_selftest: %s", cudaGetErrorString(e));
    };
    check(cudaMalloc(&flags, 2 * velo::kPeerFlagBytes));
    if (!st) check(cudaMalloc(&err, sizeof(int)));
    if (!st) check(cudaMalloc(&buf, 64 * sizeof(__nv_bfloat16)));
    if (!st) check(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    if (!st) check(cudaMemset(flags, 0, 2 * velo::kPeerFlagBytes));
    if (!st) check(cudaMemset(err, 0, sizeof(int)));
    if (!st) check(cudaMemset(buf, 0, 64 * sizeof(__nv_bfloat16)));
    if (!st) {
        velo::PeerGatherArgs g{};
        g.sync.flags[0] = flags;
        g.sync.flags[1] = flags + velo::kPeerFlagBytes / 8;
        g.sync.rank = 0;
        g.sync.tp = 2;
        g.sync.slot = 0;
        g.sync.err = err;
        g.stage = buf;           // slabs 0 and 1: 8 elements each
        g.slab = 8;
        g.out[0] = buf + 16;     // both "ranks'" sums land in this process
        g.out[1] = buf + 32;
        g.rows = 1;
        g.cols = 8;
        g.ld = 8;
        check(velo::launch_peer_gather(g, s));
    }
    if (!st) check(cudaStreamSynchronize(s));
    int h = 0;
    if (!st) check(cudaMemcpy(&h, err, sizeof(int), cudaMemcpyDeviceToHost));
    if (s) cudaStreamDestroy(s);
    cudaFree(buf);
    cudaFree(err);
    cudaFree(flags);
    if (!st) *code = h;
    return st;
}

}  // extern "C"
