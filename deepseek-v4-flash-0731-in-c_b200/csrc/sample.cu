// sample.cu - speculative-decoding acceptance: greedy argmax and temperature
// sampling over the verify rows' logits, and the accept/correct/bonus chain.
//
// Reference: src/cli/dsv4_run.c - rng_next :248-254, sample_top_p :308-353
// (comparator :80-87), argmax_logits :355, the verify-step acceptance loop
// :951-1043. The reference runs all of it on the host over logits it holds
// in host memory; here the verify rows' logits stay in HBM and the device
// reduces each [vocab] row to one target token, then one thread walks the
// chain, so only a handful of ints cross PCIe per verify step.
//
// Host restatements (exact, same order of operations) are exported too: the
// drop-in sampler for hosts that keep logits in host memory, and the top-p
// < 1 path, which needs a full sort of the row.
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <vector>
#include <algorithm>

#include "sample.cuh"

namespace dsv4 {
namespace {

constexpr int kRowThreads = 1024;

// First index of the maximum under strict ">" scanning ascending indices:
// larger value wins, the lower index on equal values; NaN never wins, except
// that a NaN at index 0 is never displaced (every comparison with it is
// false), which the reference's loop also does.
__device__ __forceinline__ bool argmax_better(float ov, int oi, float bv, int bi) {
  constexpr int kNone = 0x7FFFFFFF;
  if (oi == kNone) return false;
  if (bi == kNone) return true;
  return ov > bv || (ov == bv && oi < bi);
}

__global__ void __launch_bounds__(kRowThreads) row_argmax_kernel(const float* __restrict__ logits,
                                                                 int vocab, int* __restrict__ out) {
  constexpr int kNone = 0x7FFFFFFF;
  const float* row = logits + static_cast<size_t>(blockIdx.x) * vocab;
  __shared__ float sv[32];
  __shared__ int si[32];
  float bv = -INFINITY;
  int bi = kNone;
  for (int v = threadIdx.x; v < vocab; v += blockDim.x) {
    const float x = row[v];
    if (x == x && argmax_better(x, v, bv, bi)) { bv = x; bi = v; }  // NaN never competes
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (argmax_better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
  }
  if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = sv[0];
    int i = si[0];
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
      if (argmax_better(sv[w], si[w], v, i)) { v = sv[w]; i = si[w]; }
    const float x0 = row[0];
    out[blockIdx.x] = (x0 != x0 || i == kNone) ? 0 : i;
  }
}

// Temperature sampling with top_p = 1 (src/cli/dsv4_run.c:311-331): the
// weights exp((l - max) / T) in double, target = u * total, the first index
// whose running sum exceeds the target. Thread t owns a contiguous chunk; the
// chunk sums are scanned across the block and the owning thread rescans its
// chunk. The sums are formed in a different order than the reference's
// single loop, so a target within a few ulps of a running sum can pick the
// neighbouring token; the host sampler is exact.
__global__ void __launch_bounds__(kRowThreads) row_sample_kernel(const float* __restrict__ logits,
                                                                 int vocab, double inv_t,
                                                                 const double* __restrict__ uni,
                                                                 int* __restrict__ out) {
  const float* row = logits + static_cast<size_t>(blockIdx.x) * vocab;
  __shared__ float smax[32];
  __shared__ double wsum[33];  // [32] = block total
  __shared__ int found;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  float mx = -INFINITY;
  for (int v = threadIdx.x; v < vocab; v += blockDim.x) mx = fmaxf(mx, row[v]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) smax[warp] = mx;
  if (threadIdx.x == 0) found = 0x7FFFFFFF;
  __syncthreads();
  mx = smax[0];
  for (int w = 1; w < nw; ++w) mx = fmaxf(mx, smax[w]);
  const double dmx = mx;
  const int chunk = (vocab + blockDim.x - 1) / blockDim.x;
  const int b0 = min(vocab, static_cast<int>(threadIdx.x) * chunk), b1 = min(vocab, b0 + chunk);
  double s = 0.0;
  for (int v = b0; v < b1; ++v) s += exp((static_cast<double>(row[v]) - dmx) * inv_t);
  // exclusive scan of the chunk sums
  double incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const double w = lane < nw ? wsum[lane] : 0.0;
    double wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double t = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += t;
    }
    if (lane < nw) wsum[lane] = wi - w;
    if (lane == 31) wsum[32] = wi;
  }
  __syncthreads();
  const double off = wsum[warp] + (incl - s);
  const double total = wsum[32];
  const double target = uni[blockIdx.x] * total;
  if (b0 < b1 && target < off + s) {
    double cum = off;
    for (int v = b0; v < b1; ++v) {
      cum += exp((static_cast<double>(row[v]) - dmx) * inv_t);
      if (target < cum) {
        atomicMin(&found, v);
        break;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) out[blockIdx.x] = found == 0x7FFFFFFF ? vocab - 1 : found;
}

// The acceptance loop of src/cli/dsv4_run.c:951-1043 over precomputed row
// targets (targets[r] = the argmax or sample of row r). result: [0] emitted
// tokens, [1] positions to commit, [2] accepted drafts, [3] uniforms the
// reference would have consumed, [4 ..] the emitted tokens.
__global__ void accept_chain_kernel(const int* __restrict__ proposal, int P,
                                    const int* __restrict__ targets, int eos, int sampled,
                                    int* __restrict__ result) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  int accepted = 0, correction = -1, samples = 0;
  while (accepted < P) {
    const int t = targets[accepted];
    samples += sampled;
    if (proposal[accepted] != t) { correction = t; break; }
    ++accepted;
    if (t == eos) break;
  }
  int eos_at = -1;
  for (int i = 0; i < accepted; ++i)
    if (proposal[i] == eos) { eos_at = i; break; }
  int* tok = result + 4;
  int n = 0, commit;
  if (eos_at >= 0) {
    for (int i = 0; i <= eos_at; ++i) tok[n++] = proposal[i];
    commit = eos_at + 1;
  } else if (accepted < P) {
    for (int i = 0; i < accepted; ++i) tok[n++] = proposal[i];
    tok[n++] = correction;
    commit = accepted + 1;
  } else {
    for (int i = 0; i < P; ++i) tok[n++] = proposal[i];
    tok[n++] = targets[P];
    samples += sampled;
    commit = P + 1;
  }
  result[0] = n;
  result[1] = commit;
  result[2] = accepted;
  result[3] = samples;
}

}  // namespace

cudaError_t argmax_rows(const float* logits, int rows, int vocab, int* out, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  if (vocab <= 0) return cudaErrorInvalidValue;
  row_argmax_kernel<<<rows, kRowThreads, 0, st>>>(logits, vocab, out);
  return cudaGetLastError();
}

cudaError_t sample_rows(const float* logits, int rows, int vocab, double temperature,
                        const double* uniforms, int* out, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  if (vocab <= 0) return cudaErrorInvalidValue;
  const double inv_t = temperature > 1e-5 ? 1.0 / temperature : 1e5;
  row_sample_kernel<<<rows, kRowThreads, 0, st>>>(logits, vocab, inv_t, uniforms, out);
  return cudaGetLastError();
}

cudaError_t accept_device(const int* proposal, int proposed, const float* logits, int vocab,
                          double temperature, const double* uniforms, int eos_id, int* result,
                          cudaStream_t st) {
  if (proposed < 0 || vocab <= 0) return cudaErrorInvalidValue;
  int* targets = result + 5 + proposed;
  cudaError_t e = temperature == 0.0
                      ? argmax_rows(logits, proposed + 1, vocab, targets, st)
                      : sample_rows(logits, proposed + 1, vocab, temperature, uniforms, targets, st);
  if (e != cudaSuccess) return e;
  accept_chain_kernel<<<1, 32, 0, st>>>(proposal, proposed, targets, eos_id,
                                        temperature == 0.0 ? 0 : 1, result);
  return cudaGetLastError();
}

// ------------------------------------------------------------ host side --

uint64_t rng_next_host(uint64_t* state) {
  uint64_t x = *state;
  x ^= x << 13;
  x ^= x >> 7;
  x ^= x << 17;
  *state = x;
  return x;
}

int argmax_host(const float* logits, int vocab) {
  int best = 0;
  for (int v = 1; v < vocab; ++v)
    if (logits[v] > logits[best]) best = v;
  return best;
}

int sample_top_p_host(const float* logits, int vocab, double temperature, double top_p,
                      uint64_t* state) {
  struct Item {
    double w;
    int id;
  };
  std::vector<Item> it(static_cast<size_t>(vocab));
  double mx = logits[0];
  for (int v = 1; v < vocab; ++v)
    if (logits[v] > mx) mx = logits[v];
  double total = 0.0;
  const double inv_t = temperature > 1e-5 ? 1.0 / temperature : 1e5;
  for (int v = 0; v < vocab; ++v) {
    it[v].w = std::exp((static_cast<double>(logits[v]) - mx) * inv_t);
    it[v].id = v;
    total += it[v].w;
  }
  const double u = static_cast<double>(rng_next_host(state) >> 11) * (1.0 / 9007199254740992.0);
  if (top_p == 1.0) {
    const double target = u * total;
    double cum = 0.0;
    for (int i = 0; i < vocab; ++i) {
      cum += it[i].w;
      if (target < cum) return it[i].id;
    }
    return it[vocab - 1].id;
  }
  // the reference's comparator is a total order (weight desc, id asc), so
  // any correct sort gives its permutation
  std::sort(it.begin(), it.end(), [](const Item& a, const Item& b) {
    return a.w > b.w || (a.w == b.w && a.id < b.id);
  });
  double kept = 0.0;
  int keep = vocab;
  const double thr = total * top_p;
  for (int i = 0; i < vocab; ++i) {
    kept += it[i].w;
    if (kept >= thr) { keep = i + 1; break; }
  }
  const double target = u * kept;
  double cum = 0.0;
  for (int i = 0; i < keep; ++i) {
    cum += it[i].w;
    if (target < cum) return it[i].id;
  }
  return it[keep - 1].id;
}

int accept_chain_host(const int* proposal, int P, const float* logits, int vocab,
                      double temperature, double top_p, uint64_t* state, int eos_id, int* tokens,
                      int* n_commit, int* n_accepted, int* n_samples) {
  int accepted = 0, correction = -1, samples = 0;
  auto target_of = [&](int r) {
    const float* row = logits + static_cast<size_t>(r) * vocab;
    if (temperature == 0.0) return argmax_host(row, vocab);
    ++samples;
    return sample_top_p_host(row, vocab, temperature, top_p, state);
  };
  while (accepted < P) {
    const int t = target_of(accepted);
    if (proposal[accepted] != t) { correction = t; break; }
    ++accepted;
    if (t == eos_id) break;
  }
  int eos_at = -1;
  for (int i = 0; i < accepted; ++i)
    if (proposal[i] == eos_id) { eos_at = i; break; }
  int n = 0;
  if (eos_at >= 0) {
    for (int i = 0; i <= eos_at; ++i) tokens[n++] = proposal[i];
    *n_commit = eos_at + 1;
  } else if (accepted < P) {
    for (int i = 0; i < accepted; ++i) tokens[n++] = proposal[i];
    tokens[n++] = correction;
    *n_commit = accepted + 1;
  } else {
    const int bonus = target_of(P);
    for (int i = 0; i < P; ++i) tokens[n++] = proposal[i];
    tokens[n++] = bonus;
    *n_commit = P + 1;
  }
  *n_accepted = accepted;
  *n_samples = samples;
  return n;
}

}  // namespace dsv4
