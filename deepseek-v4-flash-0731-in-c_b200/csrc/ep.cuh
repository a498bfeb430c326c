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
//   [0, 64)      flags[r]: last step epoch rank r finished writing slots here
//   [64, 128)    gflags[r]: last step epoch rank r finished writing tokens here
//   [256, 512)   counters of this rank: [0] epoch, [1] CTAs done
//   [512, ...)   slots: 2 halves x [slot_cap][H] fp32, step epoch e uses half e & 1
//   then         tokens: [tok_cap][H] fp32 (the gathered inputs of every rank)
struct EpExchange {
  float* slots[kEpMaxRanks];     // every rank's slots, as mapped in this process
  float* tokens[kEpMaxRanks];    // every rank's gathered-token rows
  unsigned* flags[kEpMaxRanks];  // every rank's slot flag array
  unsigned* gflags[kEpMaxRanks]; // every rank's token flag array
  unsigned* ctr = nullptr;       // this rank's counters
  int rank = 0, world = 0;
  size_t half_floats = 0;        // slot_cap * H
};

size_t ep_exchange_bytes(int slot_cap, int tok_cap, int H);
EpExchange ep_exchange_make(void* const* bufs, int rank, int world, int slot_cap, int tok_cap,
                            int H);

// Token-parallel step (each rank brings its own n_local tokens): this rank's
// rows go to rows [rank * n_local, +n_local) of every rank's token buffer,
// then this step's epoch (new: counter + 1) into each peer's token flags.
cudaError_t ep_gather(const EpExchange& x, const float* x_local, int n_local, int H,
                      cudaStream_t st);
// Waits (bounded) for every peer's token epoch of this step.
cudaError_t ep_gather_wait(const EpExchange& x, unsigned* err, cudaStream_t st);
// Slots of experts [lo, hi) for all world * n_local tokens go only to the
// token's owner (rank t / n_local, its slot (t % n_local) * topk + k), then
// this step's epoch into each peer's slot flags.
cudaError_t ep_push_owner(const EpExchange& x, const float* routed, const int* idx, int n_local,
                          int topk, int H, int lo, int hi, cudaStream_t st);
// Waits for every peer's slot epoch, then the ordered combine of this rank's
// n_local tokens: slots from its own buffer, router ids and shared-expert
// rows at token offset rank * n_local.
cudaError_t ep_combine_owner(const EpExchange& x, const float* shared, const int* idx,
                             int n_local, int topk, int H, float* out, unsigned* err,
                             cudaStream_t st);

// Slots of experts [lo, hi) from this rank's routed buffer into the current
// half of every rank's buffer, then this step's epoch into every peer's flags.
cudaError_t ep_push(const EpExchange& x, const float* routed, const int* idx, int n_slots, int H,
                    int lo, int hi, cudaStream_t st);

// Waits for every peer's epoch, then out = bf16(sum_k slot + shared) from the
// current half, in the reference's order.
cudaError_t ep_combine(const EpExchange& x, const float* shared, const int* idx, int n_tokens,
                       int topk, int H, float* out, unsigned* err, cudaStream_t st);

}  // namespace dsv4
