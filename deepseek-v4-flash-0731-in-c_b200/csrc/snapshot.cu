// snapshot.cu - the speculative transaction on the latent KV ring and on
// per-position state buffers, in HBM.
//
// Reference: dsv4_context_snapshot_take / _restore / _commit_prefix
// (src/dsv4/dsv4_model.c:2842-2890, :2892-2933, :2993-3056) and the
// per-position captures (:2935-2991). Before a verify step writes positions
// [start, start + n) into the window ring (slot = position % window), take
// saves the rows those slots hold and the state buffers; after acceptance,
// commit_prefix(k) keeps the first k verified positions and puts the saved
// rows back for the rest, and restore undoes the whole step. The reference
// commits by restoring every saved row and re-applying the first k
// positions' post-verify rows; when n <= window the slots are distinct and
// that equals restoring only the slots of positions >= k, which is what is
// done here (no post-verify row copies are kept).
#include <cstring>
#include <vector>

#include "attn.cuh"
#include "snapshot.cuh"

namespace dsv4 {
namespace {

// One block per listed row: copy the row's codes, scale codes and RoPE
// values between the cache and a packed [n][kKvRowBytes] buffer.
__global__ void kv_rows_copy_kernel(Fp8KvCache c, SnapRows rows, uint8_t* __restrict__ buf,
                                    int to_cache) {
  const int i = blockIdx.x;
  if (i >= rows.n) return;
  const long long r = rows.row[i];
  if (r < 0 || r >= c.rows) return;
  uint8_t* b = buf + static_cast<size_t>(i) * kv_row_bytes(c);
  uint8_t* codes = c.codes + r * c.nope;
  uint8_t* scales = c.scales + r * kKvScaleSlots;
  uint8_t* rope = reinterpret_cast<uint8_t*>(c.rope + r * c.rope_dim);
  const int nc = c.nope, nr = c.rope_dim * 2;
  for (int j = threadIdx.x; j < nc + kKvScaleSlots + nr; j += blockDim.x) {
    uint8_t* cell = j < nc ? codes + j : (j < nc + kKvScaleSlots ? scales + (j - nc)
                                                                  : rope + (j - nc - kKvScaleSlots));
    if (to_cache) *cell = b[j];
    else b[j] = *cell;
  }
}

// Row-to-row copies inside one cache (tree verify: the accepted path's
// scratch rows into their ring slots). Distinct destinations; a source row
// is never also a destination.
__global__ void kv_rows_move_kernel(Fp8KvCache c, SnapRows src, SnapRows dst) {
  const int i = blockIdx.x;
  if (i >= src.n) return;
  const long long rs = src.row[i], rd = dst.row[i];
  if (rs < 0 || rs >= c.rows || rd < 0 || rd >= c.rows) return;
  for (int j = threadIdx.x; j < c.nope; j += blockDim.x) c.codes[rd * c.nope + j] = c.codes[rs * c.nope + j];
  for (int j = threadIdx.x; j < kKvScaleSlots; j += blockDim.x)
    c.scales[rd * kKvScaleSlots + j] = c.scales[rs * kKvScaleSlots + j];
  for (int j = threadIdx.x; j < c.rope_dim; j += blockDim.x)
    c.rope[rd * c.rope_dim + j] = c.rope[rs * c.rope_dim + j];
}

}  // namespace

cudaError_t kv_rows_move(const Fp8KvCache& c, const SnapRows& src, const SnapRows& dst,
                         cudaStream_t st) {
  if (src.n <= 0) return cudaSuccess;
  if (dst.n != src.n) return cudaErrorInvalidValue;
  kv_rows_move_kernel<<<src.n, 128, 0, st>>>(c, src, dst);
  return cudaGetLastError();
}

cudaError_t kv_rows_save(const Fp8KvCache& c, const SnapRows& rows, uint8_t* buf,
                         cudaStream_t st) {
  if (rows.n <= 0) return cudaSuccess;
  kv_rows_copy_kernel<<<rows.n, 256, 0, st>>>(c, rows, buf, 0);
  return cudaGetLastError();
}

cudaError_t kv_rows_load(const Fp8KvCache& c, const SnapRows& rows, const uint8_t* buf,
                         cudaStream_t st) {
  if (rows.n <= 0) return cudaSuccess;
  kv_rows_copy_kernel<<<rows.n, 256, 0, st>>>(c, rows, const_cast<uint8_t*>(buf), 1);
  return cudaGetLastError();
}

}  // namespace dsv4
