// tp_allreduce.cu -- sum of the row-split GEMMs' bf16 partials over the
// tensor-parallel group through NVLink peer memory.
//
// Replaces, for o_proj and down_proj, the reference's CPU all-reduce
// (LlamaTensorParallelModel::all_reduce_sum_and_add, src/metal/tp_model.rs:199-277)
// and NCCL's ring in this build.  Every rank's partial buffer is mapped into every
// other rank's address space (CUDA IPC), so one kernel does the whole sum: rank r
// owns chunk r of the rows, loads that chunk from all tp buffers (its own from
// HBM, the others over NVLink), adds them in rank order in f32, and stores the
// bf16 sum into all tp buffers.  Each byte of partial crosses NVLink once in each
// direction, in one pass; all ranks end with identical values.
//
// Ordering: a cross-rank entry barrier (each rank publishes an epoch into every
// rank's flag block with a system-scope release, after its partial is complete,
// and waits until all tp epochs have arrived) guarantees every partial is written
// before anyone reads it and that no rank still reads the previous sum; an exit
// barrier (a system-scope counter in every rank's block, bumped by every CTA of
// every rank after its stores) guarantees every sum has landed before the kernel
// returns and the next kernel on the stream reads the buffer.  Every wait is
// bounded by the global timer (2 s): a rank that never arrives makes the others
// record an error and return instead of spinning forever.  The grid is small
// (kPeerGrid CTAs of 256 threads, no dynamic shared memory) and fixed; each CTA
// counts its own calls in its rank's flag block, so the epochs need no host state
// and every rank's CTAs agree on them.
#include "kernels/tp_allreduce.h"

#include <cuda_bf16.h>

namespace velo {
namespace {

constexpr int kThreads = 256;
constexpr unsigned long long kWaitNs = 2000000000ull;
constexpr int kErrPeerEntry = 0x7101, kErrPeerExit = 0x7102;

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

// 8 bf16 of every rank's buffer at element e, summed in rank order (f32), stored
// as bf16 into every rank's buffer
__device__ __forceinline__ void sum_vectors(const PeerAllReduceArgs& a, size_t e0, size_t e1, bool two) {
    uint4 in[2][kPeerMaxRanks];
#pragma unroll
    for (int p = 0; p < kPeerMaxRanks; ++p)
        if (p < a.tp) {
            in[0][p] = ld_volatile16(a.buf[p] + e0);
            if (two) in[1][p] = ld_volatile16(a.buf[p] + e1);
        }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        if (j == 1 && !two) break;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int p = 0; p < kPeerMaxRanks; ++p)
            if (p < a.tp) add8(acc, in[j][p]);
        uint4 out;
        uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
            o[i] = *reinterpret_cast<const uint32_t*>(&h);
        }
        const size_t e = j ? e1 : e0;
#pragma unroll
        for (int p = 0; p < kPeerMaxRanks; ++p)
            if (p < a.tp) *reinterpret_cast<uint4*>(a.buf[p] + e) = out;
    }
}

__global__ void __launch_bounds__(kThreads) peer_allreduce_kernel(PeerAllReduceArgs a) {
    __shared__ int ok_sh;
    __shared__ unsigned long long epoch_sh;
    const int tid = threadIdx.x;
    unsigned long long* my = a.flags[a.rank] + a.slot * kPeerSlotWords;
    // this CTA's call number on this slot (only this CTA of this rank touches the word)
    if (tid == 0) {
        epoch_sh = my[16 + blockIdx.x] + 1;
        ok_sh = 1;
    }
    __syncthreads();
    const unsigned long long epoch = epoch_sh;
    // ---- entry: this rank's partial is complete (stream order); tell everyone
    if (blockIdx.x == 0 && tid < a.tp) {
        __threadfence_system();
        st_release_sys(a.flags[tid] + a.slot * kPeerSlotWords + a.rank, epoch);
    }
    if (tid < a.tp && !wait_at_least(my + tid, epoch)) {
        atomicCAS(a.err, 0, kErrPeerEntry);
        ok_sh = 0;
    }
    __syncthreads();
    if (ok_sh) {
        // ---- chunk `rank` of the vectors (8 bf16 each), two vectors per thread per pass
        const size_t nvec = a.n / 8;
        const size_t v0 = nvec * a.rank / a.tp, v1 = nvec * (a.rank + 1) / a.tp;
        const size_t stride = (size_t)gridDim.x * kThreads;
        for (size_t v = v0 + (size_t)blockIdx.x * kThreads + tid; v < v1; v += 2 * stride)
            sum_vectors(a, a.offset + v * 8, a.offset + (v + stride) * 8, v + stride < v1);
    }
    // ---- exit: every CTA of every rank counts itself in every rank's block (also
    // after a failed entry, so that the counts stay in step)
    __syncthreads();
    if (tid < a.tp) {
        __threadfence_system();
        red_release_sys_add(a.flags[tid] + a.slot * kPeerSlotWords + 8, 1ull);
    }
    if (tid == 0) {
        if (!wait_at_least(my + 8, epoch * (unsigned long long)a.tp * kPeerGrid)) atomicCAS(a.err, 0, kErrPeerExit);
        my[16 + blockIdx.x] = epoch;
    }
    __syncthreads();
}

}  // namespace

cudaError_t launch_peer_allreduce(const PeerAllReduceArgs& a, cudaStream_t stream) {
    if (a.tp < 2 || a.tp > kPeerMaxRanks || a.rank < 0 || a.rank >= a.tp || a.n % 8 || a.offset % 8 ||
        a.slot < 0 || a.slot > 3)
        return cudaErrorInvalidValue;
    peer_allreduce_kernel<<<kPeerGrid, kThreads, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace velo
