// tp_allreduce.cu -- sum of the row-split GEMMs' bf16 partials over the
// tensor-parallel group through NVLink peer memory.
//
// Replaces, for o_proj and down_proj, the reference's CPU all-reduce
// (LlamaTensorParallelModel::all_reduce_sum_and_add, src/metal/tp_model.rs:199-277)
// and NCCL's ring in this build.  Every rank's buffers are mapped into every other
// rank's address space (CUDA IPC).  Three forms:
//   fused (peer_gather_kernel): the row-split GEMM's epilogue already stored column
//     block r of its partial into rank r's receive area, overlapping the transfer
//     with the GEMM's tiles; rank r adds its block's tp slabs (local HBM) in rank
//     order in f32 and stores the bf16 sum into every rank's sum buffer.
//   unfused (peer_allreduce_kernel): rank r owns chunk r of the rows, loads that
//     chunk from all tp buffers (its own from HBM, the others over NVLink), adds
//     them in rank order in f32 and stores the bf16 sum into all tp buffers.
//   copy engines (ce_sum_kernel with ce_signal_kernel / ce_wait_kernel): the data
//     crosses NVLink as cudaMemcpyAsync copies issued by the host; one-warp
//     kernels publish and await each phase's completion and rank r adds its tp
//     slabs locally.
// All add the same bf16 partials in the same order: identical results.
//
// Ordering: a cross-rank entry barrier (each rank publishes an epoch into every
// rank's flag block with a system-scope release, after its partial is complete,
// and waits until all tp epochs have arrived) guarantees every partial is written
// before anyone reads it and that no rank still reads the previous sum; an exit
// barrier (a system-scope counter in every rank's block, bumped by every CTA of
// every rank after its stores) guarantees every sum has landed before the kernel
// returns and the next kernel on the stream reads the buffer.  Every wait is
// bounded by the global timer (2 s): a rank that never arrives makes the others
// record an error and return instead of spinning forever.  The grid of the first
// two forms is fixed (kPeerGrid CTAs of 128 threads, at most 72 registers each and
// no dynamic shared memory, so that a CTA fits on an SM beside a GEMM or attention
// CTA of the other stream);
// each CTA counts its own calls in its rank's flag block, so the epochs need no
// host state and every rank's CTAs agree on them.
#include "kernels/tp_allreduce.h"

#include <cuda_bf16.h>

namespace velo {
namespace {

constexpr int kThreads = 128;
constexpr unsigned long long kWaitNs = 2000000000ull;
constexpr int kErrPeerEntry = 0x7101, kErrPeerExit = 0x7102, kErrCeWait = 0x7103;

__device__ __forceinline__ unsigned long long now_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void red_release_sys_add(unsigned long long* p, unsigned long long v) {
    asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint4 ld_volatile16(const void* p) {
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p)
                 : "memory");
    return v;
}

// Waits until *p >= target (bounded); false when the limit ran out.
__device__ __forceinline__ bool wait_at_least(const unsigned long long* p, unsigned long long target) {
    if (ld_acquire_sys(p) >= target) return true;
    const unsigned long long t0 = now_ns();
    for (;;) {
        __nanosleep(64);
        if (ld_acquire_sys(p) >= target) return true;
        if (now_ns() - t0 > kWaitNs) return false;
    }
}

__device__ __forceinline__ void add8(float (&acc)[8], uint4 v) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
        acc[2 * i] = __fadd_rn(acc[2 * i], f.x);
        acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], f.y);
    }
}

// Entry barrier: this rank's partial is complete (stream order); publish the
// call's epoch to every rank and wait until every rank's has arrived here.
// Returns the epoch (0 after a wait ran out; the error word is set then).
__device__ __forceinline__ unsigned long long peer_entry(const PeerSync& y) {
    __shared__ int ok_sh;
    __shared__ unsigned long long epoch_sh;
    const int tid = threadIdx.x;
    unsigned long long* my = y.flags[y.rank] + y.slot * kPeerSlotWords;
    // this CTA's call number on this slot (only this CTA of this rank touches the word)
    if (tid == 0) {
        epoch_sh = my[16 + blockIdx.x] + 1;
        ok_sh = 1;
    }
    __syncthreads();
    const unsigned long long epoch = epoch_sh;
    if (blockIdx.x == 0 && tid < y.tp) {
        __threadfence_system();
        st_release_sys(y.flags[tid] + y.slot * kPeerSlotWords + y.rank, epoch);
    }
    if (tid < y.tp && !wait_at_least(my + tid, epoch)) {
        atomicCAS(y.err, 0, kErrPeerEntry);
        ok_sh = 0;
    }
    __syncthreads();
    return ok_sh ? epoch : 0;
}

// Exit barrier: every CTA of every rank counts itself in every rank's block
// after its stores (also after a failed entry, so that the counts stay in step)
// and waits until all tp x kPeerGrid CTAs of this call have counted in its own.
__device__ __forceinline__ void peer_exit(const PeerSync& y) {
    const int tid = threadIdx.x;
    unsigned long long* my = y.flags[y.rank] + y.slot * kPeerSlotWords;
    __syncthreads();
    const unsigned long long epoch = my[16 + blockIdx.x] + 1;
    if (tid < y.tp) {
        __threadfence_system();
        red_release_sys_add(y.flags[tid] + y.slot * kPeerSlotWords + 8, 1ull);
    }
    if (tid == 0) {
        if (!wait_at_least(my + 8, epoch * (unsigned long long)y.tp * kPeerGrid)) atomicCAS(y.err, 0, kErrPeerExit);
        my[16 + blockIdx.x] = epoch;
    }
    __syncthreads();
}

__device__ __forceinline__ uint4 round_bf16x8(const float (&acc)[8]) {
    uint4 out;
    uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
        o[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    return out;
}

// vectors (8 bf16) per thread per pass: two while the loads of all ranks fit the
// register budget
template <int TP>
constexpr int kUnroll = TP <= 4 ? 2 : 1;

template <int TP>
__global__ void __launch_bounds__(kThreads) peer_allreduce_kernel(const __grid_constant__ PeerAllReduceArgs a) {
    constexpr int U = kUnroll<TP>;
    if (peer_entry(a.sync)) {
        // chunk `rank` of the vectors (8 bf16 each)
        const size_t nvec = a.n / 8;
        const size_t v0 = nvec * a.sync.rank / TP, v1 = nvec * (a.sync.rank + 1) / TP;
        const size_t stride = (size_t)gridDim.x * kThreads;
        for (size_t v = v0 + (size_t)blockIdx.x * kThreads + threadIdx.x; v < v1; v += U * stride) {
            uint4 in[U][TP];
#pragma unroll
            for (int j = 0; j < U; ++j)
                if (v + j * stride < v1)
#pragma unroll
                    for (int p = 0; p < TP; ++p) in[j][p] = ld_volatile16(a.buf[p] + a.offset + (v + j * stride) * 8);
#pragma unroll
            for (int j = 0; j < U; ++j) {
                if (v + j * stride >= v1) break;
                float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int p = 0; p < TP; ++p) add8(acc, in[j][p]);
                const uint4 out = round_bf16x8(acc);
#pragma unroll
                for (int p = 0; p < TP; ++p)
                    *reinterpret_cast<uint4*>(a.buf[p] + a.offset + (v + j * stride) * 8) = out;
            }
        }
    }
    peer_exit(a.sync);
}

// rank r's column block: tp slabs read from its own HBM, the sum pushed to all ranks
template <int TP>
__global__ void __launch_bounds__(kThreads) peer_gather_kernel(const __grid_constant__ PeerGatherArgs a) {
    constexpr int U = kUnroll<TP>;
    if (peer_entry(a.sync)) {
        const int vpr = a.cols / 8;  // vectors per row
        const size_t nvec = (size_t)a.rows * vpr;
        const size_t stride = (size_t)gridDim.x * kThreads;
        for (size_t v = (size_t)blockIdx.x * kThreads + threadIdx.x; v < nvec; v += U * stride) {
            size_t src[U], dst[U];
#pragma unroll
            for (int j = 0; j < U; ++j) {
                const size_t w = v + j * stride;
                const size_t m = w / vpr, c = (w - m * vpr) * 8;
                src[j] = m * a.cols + c;
                dst[j] = m * a.ld + c;
            }
            uint4 in[U][TP];
#pragma unroll
            for (int j = 0; j < U; ++j)
                if (v + j * stride < nvec)
#pragma unroll
                    for (int p = 0; p < TP; ++p) in[j][p] = ld_volatile16(a.stage + p * a.slab + src[j]);
#pragma unroll
            for (int j = 0; j < U; ++j) {
                if (v + j * stride >= nvec) break;
                float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int p = 0; p < TP; ++p) add8(acc, in[j][p]);
                const uint4 out = round_bf16x8(acc);
#pragma unroll
                for (int p = 0; p < TP; ++p) *reinterpret_cast<uint4*>(a.out[p] + dst[j]) = out;
            }
        }
    }
    peer_exit(a.sync);
}

// ---- copy-engine form
__device__ __forceinline__ unsigned long long* ce_block(const PeerSync& y, int p) {
    return y.flags[p] + (kCeSlot0 + y.slot) * kPeerSlotWords;
}

__global__ void ce_signal_kernel(const __grid_constant__ PeerSync y, int phase) {
    __shared__ unsigned long long epoch_sh;
    unsigned long long* ctr = ce_block(y, y.rank) + 16 + phase;
    if (threadIdx.x == 0) {
        epoch_sh = *ctr + 1;
        *ctr = epoch_sh;
    }
    __syncthreads();
    const int p = threadIdx.x;
    if (p < y.tp) {
        __threadfence_system();
        st_release_sys(ce_block(y, p) + 8 * phase + y.rank, epoch_sh);
    }
}

__global__ void ce_wait_kernel(const __grid_constant__ PeerSync y, int phase) {
    const unsigned long long* my = ce_block(y, y.rank);
    const unsigned long long epoch = my[16 + phase];  // set by this call's signal on this stream
    const int p = threadIdx.x;
    if (p < y.tp && !wait_at_least(my + 8 * phase + p, epoch)) atomicCAS(y.err, 0, kErrCeWait);
}

template <int TP>
__global__ void __launch_bounds__(256) ce_sum_kernel(const __grid_constant__ CeSumArgs a) {
    const size_t nvec = a.n / 8;
    for (size_t v = (size_t)blockIdx.x * 256 + threadIdx.x; v < nvec; v += (size_t)gridDim.x * 256) {
        uint4 in[TP];
#pragma unroll
        for (int p = 0; p < TP; ++p)
            in[p] = ld_volatile16((p == a.rank ? a.own : a.stage + p * a.slab) + v * 8);
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int p = 0; p < TP; ++p) add8(acc, in[p]);
        *reinterpret_cast<uint4*>(a.out + v * 8) = round_bf16x8(acc);
    }
}

bool sync_ok(const PeerSync& y) {
    return y.tp >= 2 && y.tp <= kPeerMaxRanks && y.rank >= 0 && y.rank < y.tp && y.slot >= 0 && y.slot <= 3 &&
           y.err != nullptr;
}

}  // namespace

cudaError_t launch_peer_allreduce(const PeerAllReduceArgs& a, cudaStream_t stream) {
    if (!sync_ok(a.sync) || a.n % 8 || a.offset % 8) return cudaErrorInvalidValue;
    switch (a.sync.tp) {
        case 2: peer_allreduce_kernel<2><<<kPeerGrid, kThreads, 0, stream>>>(a); break;
        case 4: peer_allreduce_kernel<4><<<kPeerGrid, kThreads, 0, stream>>>(a); break;
        case 8: peer_allreduce_kernel<8><<<kPeerGrid, kThreads, 0, stream>>>(a); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_peer_gather(const PeerGatherArgs& a, cudaStream_t stream) {
    if (!sync_ok(a.sync) || a.cols <= 0 || a.cols % 8 || a.ld % 8 || a.rows < 0 || a.slab % 8)
        return cudaErrorInvalidValue;
    switch (a.sync.tp) {
        case 2: peer_gather_kernel<2><<<kPeerGrid, kThreads, 0, stream>>>(a); break;
        case 4: peer_gather_kernel<4><<<kPeerGrid, kThreads, 0, stream>>>(a); break;
        case 8: peer_gather_kernel<8><<<kPeerGrid, kThreads, 0, stream>>>(a); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

bool peer_tp_supported(int tp) { return tp == 2 || tp == 4 || tp == 8; }

cudaError_t launch_ce_signal(const PeerSync& y, int phase, cudaStream_t stream) {
    if (!sync_ok(y) || y.slot > 1 || (phase != kCePhaseSlabs && phase != kCePhaseSums)) return cudaErrorInvalidValue;
    ce_signal_kernel<<<1, 32, 0, stream>>>(y, phase);
    return cudaGetLastError();
}

cudaError_t launch_ce_wait(const PeerSync& y, int phase, cudaStream_t stream) {
    if (!sync_ok(y) || y.slot > 1 || (phase != kCePhaseSlabs && phase != kCePhaseSums)) return cudaErrorInvalidValue;
    ce_wait_kernel<<<1, 32, 0, stream>>>(y, phase);
    return cudaGetLastError();
}

cudaError_t launch_ce_sum(const CeSumArgs& a, int sm_count, cudaStream_t stream) {
    if (a.n % 8 || a.slab % 8 || a.rank < 0 || a.rank >= a.tp) return cudaErrorInvalidValue;
    if (a.n == 0) return cudaSuccess;
    const size_t nvec = a.n / 8;
    size_t grid = (nvec + 255) / 256;
    const size_t cap = (size_t)(sm_count > 0 ? sm_count : 148) * 4;
    if (grid > cap) grid = cap;
    switch (a.tp) {
        case 2: ce_sum_kernel<2><<<(unsigned)grid, 256, 0, stream>>>(a); break;
        case 4: ce_sum_kernel<4><<<(unsigned)grid, 256, 0, stream>>>(a); break;
        case 8: ce_sum_kernel<8><<<(unsigned)grid, 256, 0, stream>>>(a); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace velo
