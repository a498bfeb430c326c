// ep.cuh - expert-parallel slot exchange over peer memory (NVLink P2P).
//
// Each rank computes the routed slots (token, k) of its own experts; every
// rank needs all slots for the ordered combine (attention is replicated).
// Instead of a collective on zero-padded slots, each rank writes its slots
// straight into every rank's exchange buffer (CUDA IPC mappings of peer
// device memory, plain stores), then publishes a step epoch into each
// peer's flag array; the combine waits (bounded) for every peer's epoch and
// sums the slots in the reference's order. Every slot has one writer, so the
// result is bit-identical to one GPU holding all experts.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace dsv4 {

constexpr int kEpMaxRanks = 8;
constexpr unsigned kErrEpWait = 8u;  // device error word: a peer's epoch never arrived

// One rank's exchange buffer (one per MoE layer):
//   [0, 256)    flags[r]: last step epoch rank r finished writing here
//   [256, 512)  counters of this rank: [0] epoch, [1] push CTAs done
//   [512, ...)  slots: 2 halves x [slot_cap][H] fp32, step epoch e uses half e & 1
struct EpExchange {
  float* slots[kEpMaxRanks];     // every rank's slots, as mapped in this process
  unsigned* flags[kEpMaxRanks];  // every rank's flag array
  unsigned* ctr = nullptr;       // this rank's counters
  int rank = 0, world = 0;
  size_t half_floats = 0;        // slot_cap * H
};

size_t ep_exchange_bytes(int slot_cap, int H);
EpExchange ep_exchange_make(void* const* bufs, int rank, int world, int slot_cap, int H);

// Slots of experts [lo, hi) from this rank's routed buffer into the current
// half of every rank's buffer, then this step's epoch into every peer's flags.
cudaError_t ep_push(const EpExchange& x, const float* routed, const int* idx, int n_slots, int H,
                    int lo, int hi, cudaStream_t st);

// Waits for every peer's epoch, then out = bf16(sum_k slot + shared) from the
// current half, in the reference's order.
cudaError_t ep_combine(const EpExchange& x, const float* shared, const int* idx, int n_tokens,
                       int topk, int H, float* out, unsigned* err, cudaStream_t st);

}  // namespace dsv4
