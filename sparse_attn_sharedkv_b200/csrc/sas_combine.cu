// Split-KV log-sum-exp combine (the flash-decode reduction the reference
// schedules in metadata.py:795-827 / 925-954 but never runs).
//
// A query row whose 64-key tiles were split over several workers has one
// fp32 partial per piece: O_i (already divided by its own row sum) and
// LSE_i = ln(sum_i).  The exact result is
//     LSE = log(sum_i exp(LSE_i)),   O = sum_i exp(LSE_i - LSE) * O_i,
// the sink having been counted once, in piece 0.  Pieces with no attended
// key carry LSE_i = -inf and contribute nothing.
//
// Grid: (split rows, head blocks of 4).  Each warp owns one head: lanes read
// the piece LSEs, reduce max / sum with shuffles, then stream the 512-wide
// rows with 16-byte loads.  HBM-bound: bytes = pieces * (H * d_v * 4) read +
// H * d_v * 2 written per split row.

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "sas.h"
#include "sas_kernels.h"

namespace sas {
namespace {

constexpr int kHeadsPerBlock = 4;

template <bool kBf16>
__global__ void __launch_bounds__(32 * kHeadsPerBlock)
    sas_combine_kernel(const int32_t* __restrict__ row_token, const int32_t* __restrict__ row_pieces,
                       const int32_t* __restrict__ row_base, int stride,
                       const float* __restrict__ o_part,
                       const float* __restrict__ lse_part, int num_heads, int dv,
                       void* __restrict__ out, float* __restrict__ lse_out) {
  const int row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.y * kHeadsPerBlock + warp;
  if (head >= num_heads) return;
  const int token = __ldg(row_token + (size_t)row * stride);
  const int pieces = __ldg(row_pieces + (size_t)row * stride);
  const int base = __ldg(row_base + (size_t)row * stride);
  // Unused entries of a device-built plan's split section (sized for the
  // worst case) carry no pieces.
  if (pieces <= 0) return;

  // Max of the piece LSEs.
  float mx = -INFINITY;
  for (int i = lane; i < pieces; i += 32)
    mx = fmaxf(mx, __ldg(lse_part + (size_t)(base + i) * num_heads + head));
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
  const float ref = (mx == -INFINITY) ? 0.f : mx;
  for (int i = lane; i < pieces; i += 32)
    sum += expf(__ldg(lse_part + (size_t)(base + i) * num_heads + head) - ref);
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float total_lse = (mx == -INFINITY) ? -INFINITY : ref + logf(sum);
  const float inv = (sum > 0.f) ? 1.f / sum : 0.f;

  // Each lane owns dims [8*lane + 256*k, +8) for k = 0, 1 (d_v = 512).
  float acc[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i] = 0.f;
  for (int p = 0; p < pieces; ++p) {
    const float l = __ldg(lse_part + (size_t)(base + p) * num_heads + head);
    const float w = (l == -INFINITY) ? 0.f : expf(l - ref) * inv;
    if (w == 0.f) continue;
    const float* src = o_part + ((size_t)(base + p) * num_heads + head) * dv;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(src + 256 * k + 8 * lane));
      const float4 b = __ldg(reinterpret_cast<const float4*>(src + 256 * k + 8 * lane + 4));
      acc[8 * k + 0] += w * a.x; acc[8 * k + 1] += w * a.y;
      acc[8 * k + 2] += w * a.z; acc[8 * k + 3] += w * a.w;
      acc[8 * k + 4] += w * b.x; acc[8 * k + 5] += w * b.y;
      acc[8 * k + 6] += w * b.z; acc[8 * k + 7] += w * b.w;
    }
  }
  char* dst = reinterpret_cast<char*>(out) + ((size_t)token * num_heads + head) * dv * 2;
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    uint32_t w4[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (kBf16) {
        __nv_bfloat162 h = __floats2bfloat162_rn(acc[8 * k + 2 * i], acc[8 * k + 2 * i + 1]);
        w4[i] = *reinterpret_cast<uint32_t*>(&h);
      } else {
        __half2 h = __floats2half2_rn(acc[8 * k + 2 * i], acc[8 * k + 2 * i + 1]);
        w4[i] = *reinterpret_cast<uint32_t*>(&h);
      }
    }
    *reinterpret_cast<uint4*>(dst + (256 * k + 8 * lane) * 2) =
        make_uint4(w4[0], w4[1], w4[2], w4[3]);
  }
  if (lane == 0) lse_out[(size_t)token * num_heads + head] = total_lse;
}

}  // namespace

int launch_combine(const int32_t* row_token, const int32_t* row_pieces, const int32_t* row_base,
                   int stride, int n, const float* o_partial,
                   const float* lse_partial, int num_heads, int head_dim_v, int dtype, void* out,
                   float* lse, cudaStream_t stream) {
  if (n <= 0) return SAS_OK;
  if (head_dim_v != 512) return SAS_ERR_UNSUPPORTED;
  dim3 grid(n, (num_heads + kHeadsPerBlock - 1) / kHeadsPerBlock);
  if (dtype == SAS_DTYPE_BF16)
    sas_combine_kernel<true><<<grid, 32 * kHeadsPerBlock, 0, stream>>>(
        row_token, row_pieces, row_base, stride, o_partial, lse_partial, num_heads, head_dim_v,
        out, lse);
  else
    sas_combine_kernel<false><<<grid, 32 * kHeadsPerBlock, 0, stream>>>(
        row_token, row_pieces, row_base, stride, o_partial, lse_partial, num_heads, head_dim_v,
        out, lse);
  return cudaGetLastError() == cudaSuccess ? SAS_OK : SAS_ERR_CUDA;
}

}  // namespace sas
