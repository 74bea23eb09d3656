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
// CTAs) does not depend on the call's size.  128 CTAs of 128 threads moved a
// config-5 gather faster than 256 or 512 (tp4: 57.3 us against 65.6 and 65.9;
// tp2: 44.9 against 51.1 and 49.8), and the unfused sum at tp4 (93.6 against 101.5).
constexpr int kPeerGrid = 128;
// flag block of one rank, per slot (u64 words): [0, 8) the ranks' entry epochs,
// 8 the exit count, [16, 16 + kPeerGrid) this rank's CTAs' call counters
constexpr int kPeerSlotWords = 16 + kPeerGrid;
constexpr size_t kPeerFlagBytes = 4 * kPeerSlotWords * 8;  // 4 slots

// The cross-rank barriers of one call.  Every rank makes the same sequence of
// calls on each slot; the calls are counted on the device, so a captured graph of
// them stays in step.  All waits are bounded (2 s), after which the kernel
// records an error in *err and returns.
struct PeerSync {
    unsigned long long* flags[kPeerMaxRanks];  // every rank's flag block
    int rank, tp, slot;  // slot: one of 4 independent call sequences (one per stream)
    int* err;            // device error word (a wait ran out)
};

struct PeerAllReduceArgs {
    PeerSync sync;
    __nv_bfloat16* buf[kPeerMaxRanks];  // every rank's partial buffer (own one included)
    size_t offset;       // elements: where this call's rows start in every buffer
    size_t n;            // elements to sum (a multiple of 8)
};

// Sum n bf16 elements at `offset` over the tp ranks' buffers, in place on every
// rank: rank r adds chunk r of all buffers in rank order (f32) and writes the
// bf16 sum back into all of them, between a cross-rank entry barrier (every
// partial written) and an exit barrier (every sum written).
cudaError_t launch_peer_allreduce(const PeerAllReduceArgs& a, cudaStream_t stream);

struct PeerGatherArgs {
    PeerSync sync;
    // this rank's receive area at the call's first row: slab s (at s * slab
    // elements) holds rank s's partial of this rank's `cols` columns, row stride cols
    const __nv_bfloat16* stage;
    size_t slab;
    // every rank's sum buffer at (the call's first row, this rank's first column),
    // row stride ld
    __nv_bfloat16* out[kPeerMaxRanks];
    int rows, cols, ld;  // cols % 8 == 0
};

// Second half of the fused sum: the row-split GEMMs pushed their partials of
// column block r to rank r (kEpiPeerBF16); after the entry barrier rank r adds
// its tp slabs in rank order (f32), rounds to bf16 and stores the sum into
// every rank's sum buffer, then waits at the exit barrier.  The values equal
// launch_peer_allreduce's.
cudaError_t launch_peer_gather(const PeerGatherArgs& a, cudaStream_t stream);

// Group sizes the kernels are built for (2, 4, 8); others keep NCCL.
bool peer_tp_supported(int tp);

// ---- copy-engine form: the data crosses NVLink as cudaMemcpyAsync copies
// (copy engines, no SMs); these kernels only order them and add.
// Per slot of the flag block (slots 2 and 3; u64 words): [0, 8) the ranks'
// "slab sent" epochs, [8, 16) the ranks' "sum sent" epochs, 16 / 17 this rank's
// call counters of the two phases.
constexpr int kCeSlot0 = 2;
constexpr int kCePhaseSlabs = 0, kCePhaseSums = 1;
static_assert(kCeSlot0 + 2 <= 4, "the copy-engine slots lie in the 4-slot flag block");
static_assert(16 + 2 <= kPeerSlotWords, "a slot holds the copy-engine entries and counters");

// One warp: count this call on `phase` (a device counter, so graphs stay in
// step) and publish the count to every rank's entry `rank` of the phase, with a
// system-scope release.  Issued on the stream after the copies it announces.
cudaError_t launch_ce_signal(const PeerSync& y, int phase, cudaStream_t stream);
// One warp: wait (bounded, 2 s; 0x7103 in the error word when it runs out)
// until every rank has published this call's count of `phase`.
cudaError_t launch_ce_wait(const PeerSync& y, int phase, cudaStream_t stream);

struct CeSumArgs {
    const __nv_bfloat16* own;   // this rank's partial of its own column block
    const __nv_bfloat16* stage; // receive area: slab s at s * slab (s != rank)
    size_t slab;
    __nv_bfloat16* out;         // this rank's column block of the sum
    size_t n;                   // elements per block (rows x cols, a multiple of 8)
    int rank, tp;
};
// out = bf16(sum over s in rank order of the tp partials, in f32): the values of
// launch_peer_gather / launch_peer_allreduce.
cudaError_t launch_ce_sum(const CeSumArgs& a, int sm_count, cudaStream_t stream);

}  // namespace velo
