// sample.cuh - speculative-decoding acceptance (device and host forms).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace dsv4 {

// Device: one target token per logits row [rows][vocab].
cudaError_t argmax_rows(const float* logits, int rows, int vocab, int* out, cudaStream_t st);
// top_p = 1 sampling with uniforms[rows] (53-bit, in the reference's draw order).
cudaError_t sample_rows(const float* logits, int rows, int vocab, double temperature,
                        const double* uniforms, int* out, cudaStream_t st);
// Row targets of the proposed + 1 verify rows, then the acceptance chain.
// result holds 2 * proposed + 6 ints: [0] emitted, [1] commit length,
// [2] accepted drafts, [3] uniforms consumed, [4 ..] emitted tokens, then
// the row targets.
cudaError_t accept_device(const int* proposal, int proposed, const float* logits, int vocab,
                          double temperature, const double* uniforms, int eos_id, int* result,
                          cudaStream_t st);

// Host restatements of src/cli/dsv4_run.c:248-355 and :951-1043.
uint64_t rng_next_host(uint64_t* state);
int argmax_host(const float* logits, int vocab);
int sample_top_p_host(const float* logits, int vocab, double temperature, double top_p,
                      uint64_t* state);
int accept_chain_host(const int* proposal, int proposed, const float* logits, int vocab,
                      double temperature, double top_p, uint64_t* state, int eos_id, int* tokens,
                      int* n_commit, int* n_accepted, int* n_samples);

}  // namespace dsv4
