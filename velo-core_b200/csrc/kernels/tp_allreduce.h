// tp_allreduce.h -- the tensor-parallel sum of a row-split GEMM's bf16 partials
// over NVLink peer memory (tp_allreduce.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

namespace velo {

constexpr int kPeerMaxRanks = 8;
// CTAs per launch: fixed, so that the exit count a call waits for (calls x ranks x
// CTAs) does not depend on the call's size
constexpr int kPeerGrid = 128;
// flag block of one rank, per slot (u64 words): [0, 8) the ranks' entry epochs,
// 8 the exit count, [16, 16 + kPeerGrid) this rank's CTAs' call counters
constexpr int kPeerSlotWords = 16 + kPeerGrid;
constexpr size_t kPeerFlagBytes = 4 * kPeerSlotWords * 8;  // 4 slots

struct PeerAllReduceArgs {
    __nv_bfloat16* buf[kPeerMaxRanks];  // every rank's partial buffer (own one included)
    unsigned long long* flags[kPeerMaxRanks];  // every rank's flag block
    size_t offset;       // elements: where this call's rows start in every buffer
    size_t n;            // elements to sum (a multiple of 8)
    int rank, tp, slot;  // slot: one of 4 independent call sequences (one per stream)
    int* err;            // device error word (a wait ran out)
};

// Sum n bf16 elements at `offset` over the tp ranks' buffers, in place on every
// rank: rank r adds chunk r of all buffers in rank order (f32) and writes the
// bf16 sum back into all of them, between a cross-rank entry barrier (every
// partial written) and an exit barrier (every sum written).  Every rank makes the
// same sequence of calls on each slot; the calls are counted on the device, so a
// captured graph of them stays in step.  All waits are bounded (2 s), after which
// the kernel records an error and returns.
cudaError_t launch_peer_allreduce(const PeerAllReduceArgs& a, cudaStream_t stream);

}  // namespace velo
