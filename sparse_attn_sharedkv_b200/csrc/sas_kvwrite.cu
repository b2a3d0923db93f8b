// Paged-cache writer: appends new key rows of each batch into a paged KV
// pool [blocks, block_size, 1, D] through its block table, the step that
// precedes the attention path.  Layout (golden.py:315-360): logical position
// p of batch b lives at pool[block_table[b, p / bs], p % bs].
//
// One warp per new row: the row's batch is found by a binary search over
// cu_new, then the row (D * 2 bytes) moves as 16-byte vectors, coalesced on
// both sides.  A position past the table, an unmapped page (-1) or a page
// outside the pool is not written; it is recorded in the optional error word
// (code SAS_ERR_DEVICE, site 50, detail = the row index).  HBM-bound copy:
// 2 x row bytes per row.

#include <cuda_runtime.h>
#include <stdint.h>

#include "sas.h"

namespace {

constexpr int kWarpsPerBlock = 8;

__global__ void __launch_bounds__(32 * kWarpsPerBlock)
    kv_append_kernel(uint8_t* __restrict__ pool, int32_t num_blocks, int32_t block_size,
                     int32_t row_bytes, const int32_t* __restrict__ block_table,
                     int32_t table_len, const uint8_t* __restrict__ rows,
                     const int32_t* __restrict__ cu_new, const int32_t* __restrict__ start_pos,
                     int32_t batch, int32_t total_new, int32_t* err) {
  const int warp = (int)(blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5));
  const int lane = threadIdx.x & 31;
  if (warp >= total_new) return;
  // Batch of this row: the last b with cu_new[b] <= warp.
  int lo = 0, hi = batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(cu_new + mid) <= warp) lo = mid;
    else hi = mid - 1;
  }
  const int b = lo;
  const int pos = __ldg(start_pos + b) + (warp - __ldg(cu_new + b));
  const int lb = pos >= 0 ? pos / block_size : -1;
  const int blk = (lb >= 0 && lb < table_len) ? __ldg(block_table + (size_t)b * table_len + lb) : -1;
  if (blk < 0 || blk >= num_blocks) {
    if (lane == 0 && err != nullptr && atomicCAS(err, 0, SAS_ERR_DEVICE) == 0) {
      err[1] = 50;
      err[2] = warp;
      err[3] = b;
    }
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(rows + (size_t)warp * row_bytes);
  uint4* dst = reinterpret_cast<uint4*>(
      pool + ((size_t)blk * block_size + (size_t)(pos - lb * block_size)) * row_bytes);
  for (int i = lane; i < (row_bytes >> 4); i += 32) dst[i] = __ldg(src + i);
}

}  // namespace

extern "C" int sas_kv_append(void* pool, int32_t num_blocks, int32_t block_size,
                             int32_t row_bytes, const int32_t* block_table, int32_t table_len,
                             const void* rows, const int32_t* cu_new, const int32_t* start_pos,
                             int32_t batch, int32_t total_new, int32_t* err, void* stream) {
  if (total_new < 0 || batch <= 0 || block_size <= 0 || num_blocks < 0 || table_len < 0)
    return SAS_ERR_INVALID;
  if (row_bytes <= 0 || (row_bytes & 15) != 0) return SAS_ERR_INVALID;
  if (total_new == 0) return SAS_OK;
  if (!pool || !block_table || !rows || !cu_new || !start_pos) return SAS_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(pool) & 15) || (reinterpret_cast<uintptr_t>(rows) & 15))
    return SAS_ERR_INVALID;
  const int blocks = (total_new + kWarpsPerBlock - 1) / kWarpsPerBlock;
  kv_append_kernel<<<blocks, 32 * kWarpsPerBlock, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<uint8_t*>(pool), num_blocks, block_size, row_bytes, block_table,
      table_len, reinterpret_cast<const uint8_t*>(rows), cu_new, start_pos, batch, total_new, err);
  return cudaGetLastError() == cudaSuccess ? SAS_OK : SAS_ERR_CUDA;
}
