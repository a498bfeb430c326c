// snapshot.cuh - device row save/load for the KV-ring transaction.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "attn.cuh"

namespace dsv4 {

constexpr int kMaxSnapPositions = 64;  // verify rows per step (<= 64, src/cli/dsv4_run.c:256)

// Cache rows to save or load, passed by value to the kernel.
struct SnapRows {
  int n;
  long long row[kMaxSnapPositions];
};

// Bytes of one cached position in the packed snapshot buffer.
__host__ __device__ inline int kv_row_bytes(const Fp8KvCache& c) {
  return c.nope + kKvScaleSlots + 2 * c.rope_dim;
}

// buf[i] <- cache row rows.row[i]
cudaError_t kv_rows_save(const Fp8KvCache& c, const SnapRows& rows, uint8_t* buf, cudaStream_t st);
// cache row rows.row[i] <- buf[i]
cudaError_t kv_rows_load(const Fp8KvCache& c, const SnapRows& rows, const uint8_t* buf,
                         cudaStream_t st);

// cache row dst.row[i] <- cache row src.row[i]
cudaError_t kv_rows_move(const Fp8KvCache& c, const SnapRows& src, const SnapRows& dst,
                         cudaStream_t st);

}  // namespace dsv4
