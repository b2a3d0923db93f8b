// Sparse shared-KV attention forward for B200 (sm_100a): tcgen05 + TMEM.
//
// One persistent CTA per SM owns 64 query heads of a "worker" span of the
// plan (sas_plan.cpp): a contiguous run of (query token, 64-key tile) units.
// Calls with more than 64 heads use two CTAs per worker, one per head group;
// the pair walks the same tiles at the same time, so the second read of
// every key row is an L2 hit.
//
// Per tile of 64 key slots (window keys then compressed keys, golden.py
// tile order), 16 warps in five roles:
//
//   producer warps 4-7  slot -> (cache, logical pos) -> block table -> row
//                       for 16 keys each (paged window load, kernel.py:
//                       3580-3600, top-k gather, kernel.py:2606-2751, -1 stop
//                       and threshold masks, golden.py:28-66) into a per-tile
//                       valid mask; 16 consecutive rows of one cache move as
//                       one 16-row TMA box per 64-column chunk, other rows by
//                       TMA tile::gather4 (4 rows x 128 B per op) into the
//                       128B-swizzled K tile
//   Q warp 9            Q tile (64 heads) by 64 x 64 TMA boxes, next row's Q
//                       prefetched into L2
//   MMA warp 8 (1 lane) S = Q K^T  : 36 x tcgen05.mma.ws M64 N64 K16 (d_qk 576)
//                       O += P V   : 8 x tcgen05.mma.ws M64 N256 K16, where V is
//                                    the same smem K tile read MN-major (d_v 512)
//   softmax warps 0-3   tcgen05.ld of S, mask, scale, online softmax seeded
//                       by the sink (golden.py:156-196) in the exp2 domain,
//                       P rounded to the input dtype into smem, lazy O
//                       rescale in TMEM; hands m and l of each (row, piece) on
//   epilogue warps 12-15 O / l -> out (or fp32 split partials) and the LSE
//                       (kernel.py:3110-3245) through coalescing staging, then
//                       release O to the next row, overlapping its QK/softmax
//
// TMEM (512 columns): O[64 x 512] fp32 as two .ws M64 N256 accumulators
// (cols 0-255, all 128 lanes); S[64 x 64] fp32 double-buffered, each buffer
// as kQkPartials (2) partial sums over interleaved 64-dim chunks (cols
// 256-511), so the 36 small QK MMAs form independent accumulation chains.
// Shared memory: Q 72 KB and two K stages of 72 KB; P of a tile is written
// into its stage's rope chunk (dims 512..575), which PV does not read.
// 512 threads at 128 registers: every role fits without spills.
//
// Every wait on an mbarrier is bounded: on timeout the thread records an
// error in the caller's error word, raises the CTA abort flag and leaves its
// loop; no trap, no unbounded spin.

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "sas.h"
#include "sas_dev.cuh"
#include "sas_internal.h"
#include "sas_kernels.h"

namespace sas {
namespace {

constexpr int kNumSoftmaxWarps = 4;
constexpr int kProducerWarp0 = 4;  // producer warps 4..7 gather key rows
constexpr int kNumProducerWarps = 4;
constexpr int kMmaWarp = 8;
constexpr int kQWarp = 9;          // loads Q tiles by TMA, prefetches the next row's Q into L2
// Warps 10 and 11 issue the TMA loads of chunks kHelperChunk0.. (chunk group
// 2) of the rows that producer warps 2h, 2h + 1 resolved, so that a gathered
// tile's ~144 TMA ops spread over six issuing warps instead of four.
constexpr int kHelperWarp0 = 10;
constexpr int kNumHelperWarps = 2;
constexpr int kHelperChunk0 = 6;
constexpr int kEpiWarp0 = 12;      // epilogue warps 12..15 (TMEM lane quarters 0..3)
constexpr int kNumEpiWarps = 4;
constexpr int kThreads = 32 * 16;
constexpr int kEpiThreads = 32 * kNumEpiWarps;
constexpr int kSoftmaxThreads = 32 * kNumSoftmaxWarps;
constexpr int kProducerThreads = 32 * kNumProducerWarps;

// A K stage completes in three chunk groups (chunks 3g .. 3g + 2), each with
// its own barrier, so QK starts on the first chunks while the rest land.
constexpr int kChunkGroups = 3;
__host__ __device__ constexpr int chunk_group(int c) { return c / 3; }

constexpr int kMaxChunks = 9;                   // d_qk / 64
constexpr int kChunkBytes = kHeadsPerCta * 128;  // 64 rows x 64 bf16 = 8 KB
constexpr int kQBytes = kMaxChunks * kChunkBytes;
constexpr int kStageBytes = kMaxChunks * kChunkBytes;
constexpr int kSmemQ = 0;
constexpr int kSmemK0 = kSmemQ + kQBytes;
constexpr int kSmemTiles = kSmemK0 + 2 * kStageBytes;  // 221184
constexpr int kSmemDynamic = kSmemTiles + 1024;        // + runtime 1 KB alignment slack
// P (64 x 64 bf16, 8 KB) of tile j lives in chunk 8 of tile j's own K stage:
// that chunk holds dims 512..575, which only QK reads (V is dims 0..511), so
// it is free once S(j) is complete and is double-buffered with the stages.
constexpr int kPChunk = 8;
// FwdArgs::gather: key rows by cp.async 16 B from the four producer warps
// (kGatherLsu), or (any other value) by TMA boxes and tile::gather4 from the
// producers and the gather helpers.
constexpr int kGatherLsu = 0;

// TMEM columns.
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemO = 0;     // O[:, 0:256) at +0, O[:, 256:512) at +128
constexpr uint32_t kTmemS = 256;   // S buffer b, partial p at +256 + 128 b + 32 p

struct Ctl {
  uint64_t kv_full[2][kChunkGroups];  // [stage][chunk group]
  uint64_t kv_empty[2];  // PV number k (stage k % 2) completes phase k / 2 of kv_empty[k % 2]
  uint64_t q_full, q_empty;
  uint64_t s_full[2];
  uint64_t s_empty[2];
  // P(t) written: phase t / 2 of p_full[t % 2].  Two barriers, so that the
  // softmax can never complete two phases of one before its consumer tested
  // the first (P(t + 2) needs S(t + 2), which needs PV(t) issued).
  uint64_t p_full[2];
  uint64_t o_free, drain;
  uint64_t xbar[2];               // softmax partner exchange (bounded, no bar.sync)
  uint64_t gready[kNumHelperWarps][2];  // [helper][stage]: the tile's sources are in gsrc
  int32_t gsrc_row[2][kTileKeys];       // [stage][slot]: source row of each key slot
  int8_t gsrc_pool[2][kTileKeys];       // [stage][slot]: source cache (-1: none)
  uint32_t tmem_base;
  volatile int abort;
  uint16_t valid[2][4];          // per stage: slot bits of keys 16w..16w+15
  float red[2][2][kHeadsPerCta];  // [parity][half][row]: partner exchange
  // Final statistics of a (row, piece), softmax -> epilogue warps, double-
  // buffered by the parity of the piece's ordinal k: the softmax writes
  // buffer k % 2 once the epilogue has read piece k - 2 from it (fin_free).
  uint64_t fin_full[2];
  uint64_t fin_free[2];
  uint64_t o_full;                  // O of a (row, piece) complete (last PV committed)
  float fin_m[2][kHeadsPerCta];     // running max (log2 domain)
  float fin_l[2][2][kHeadsPerCta];  // [parity][half][head] partial row sums
  // Epilogue staging: per epilogue warp, 32 head rows x 32 bytes, so each
  // global store instruction writes whole 32-byte sectors of 16 rows.
  alignas(128) uint8_t epi[kNumEpiWarps][32 * 32];
};

// Ring slot (half, row) of a ring row (kRowRing): ring index i = 64 half +
// row holds the cache position p = i (mod 128) of [hi - 127, hi], hi being
// the query's own position (the window's last key); it is attended when
// p >= win_lo.  Positions below 0 have no key (zero row).
__device__ __forceinline__ SlotSrc resolve_ring(const FwdArgs& a, const Row& rv, int half,
                                                int row, int* err) {
  const int hi = rv.win_lo + rv.window - 1;
  const int i = half * 64 + row;
  const int pos = hi - ((hi - i) & (kRingKeys - 1));
  SlotSrc r{-1, 0, pos >= rv.win_lo};
  if (pos >= 0) {
    const int lb = pos / a.ori_block_size;
    if (lb < a.ori_table_len) {
      const int blk = __ldg(a.ori_block_table + (size_t)rv.b * a.ori_table_len + lb);
      if (blk >= 0 && blk < a.ori_num_blocks)
        r.row = blk * a.ori_block_size + (pos - lb * a.ori_block_size);
      else if (blk >= a.ori_num_blocks)
        record_error(err, SAS_ERR_DEVICE, 10, blk);
    } else {
      record_error(err, SAS_ERR_DEVICE, 11, pos);
    }
  }
  return r;
}

// cp.async of `count` key rows of this warp's 16-key block: local key
// lbase + k (k < count) sits at smem row key0 + lbase + k and its source is
// (r, p) of lane lbase + k.  Rows without a source are zero-filled (src-size 0).
__device__ __forceinline__ void lsu_rows(const FwdArgs& a, uint32_t sK, int key0, int lbase,
                                         int count, int r, int p, int lane, uint32_t row_bytes,
                                         int gran) {
  for (int k = 0; k < count; ++k) {
    const int row = __shfl_sync(0xffffffffu, r, lbase + k);
    const int pool = __shfl_sync(0xffffffffu, p, lbase + k);
    const bool has = (pool >= 0 && row >= 0);
    const char* src = reinterpret_cast<const char*>(pool == 1 ? a.cmp_kv : a.ori_kv);
    if (has) src += (size_t)row * row_bytes;
    else src = reinterpret_cast<const char*>(a.ori_kv);
    const int key = key0 + lbase + k;
    for (int gi = lane; gi < gran; gi += 32)
      cp_async_16(sK + (gi >> 3) * kChunkBytes + swz(key, gi & 7), src + gi * 16,
                  has ? 16u : 0u);
  }
}

// Chunks of [c0, c1) that fall in chunk group cg (chunks 3 cg .. 3 cg + 2).
__device__ __forceinline__ uint32_t group_chunks(int cg, int c0, int c1) {
  return (uint32_t)max(0, min(3 * cg + 3, c1) - max(3 * cg, c0));
}

// TMA gather of chunks c0 .. nchunks - 1 of this warp's 16 key rows (smem
// rows key0 .. key0 + 15): lanes 0..3 each move a group of 4 consecutive
// keys with one tile::gather4 per 64-column chunk (4 rows x 128 B into 512 B
// of the swizzled chunk).  Slots without a source read an out-of-range row,
// which TMA fills with zeros.  A group whose rows come from both caches
// (window / compressed boundary) is moved by cp.async instead (whole rows).
// Lane 0 arms the chunk-group barriers with the TMA bytes each receives.
__device__ __forceinline__ void tma_rows(const FwdArgs& a, const CUtensorMap* tm_ori,
                                         const CUtensorMap* tm_cmp, int c0, int nchunks,
                                         uint32_t sK,
                                         const uint32_t (&bar)[kChunkGroups], int key0, int r,
                                         int p, int lane, uint32_t row_bytes, int gran) {
  const int g = lane & 3;
  int row[4], pool[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    row[i] = __shfl_sync(0xffffffffu, r, 4 * g + i);
    pool[i] = __shfl_sync(0xffffffffu, p, 4 * g + i);
  }
  int P = -1;
  bool mixed = false;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (pool[i] >= 0) {
      if (P < 0) P = pool[i];
      else if (pool[i] != P) mixed = true;
    }
  }
  const uint32_t mixed_mask = __ballot_sync(0xffffffffu, mixed) & 0xFu;
  if (lane == 0) {
    const uint32_t groups = (uint32_t)(4 - __popc(mixed_mask));
#pragma unroll
    for (int cg = 0; cg < kChunkGroups; ++cg)
      mbar_expect_tx(bar[cg], groups * 4u * 128u * group_chunks(cg, c0, nchunks));
  }
  __syncwarp();
  if (lane < 4 && !mixed) {
    const CUtensorMap* m = (P == 1) ? tm_cmp : tm_ori;
    const int sentinel = (P == 1) ? a.cmp_rows : a.ori_rows;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (pool[i] < 0 || row[i] < 0) row[i] = sentinel;
    const uint32_t dst = sK + (uint32_t)(key0 + 4 * lane) * 128u;
    for (int c = c0; c < nchunks; ++c)
      tma_gather4(dst + c * kChunkBytes, m, c * 64, row[0], row[1], row[2], row[3],
                  bar[chunk_group(c)]);
  }
  for (uint32_t mm = mixed_mask; mm != 0u; mm &= mm - 1u)
    lsu_rows(a, sK, key0, 4 * (__ffs(mm) - 1), 4, r, p, lane, row_bytes, gran);
}

// This warp's 16 key rows of a tile (smem rows 16 pw .. 16 pw + 15) into the
// stage at sK, chunks c0 .. nchunks - 1: one 16-row TMA box per chunk when
// the rows are 16 consecutive rows of one cache (window keys inside one
// page, contiguous compressed positions), else tile::gather4 groups
// (tma_rows); cp.async of whole rows in LSU mode (c0 = 0).  Lane 0 arrives
// once on each chunk-group barrier, arming the TMA bytes.
__device__ __forceinline__ void load_tile_rows(const FwdArgs& a, const SlotSrc& sa, int c0,
                                               int nchunks, uint32_t sK,
                                               const uint32_t (&bar)[kChunkGroups], int pw,
                                               int lane, bool lsu, uint32_t row_bytes, int gran,
                                               const CUtensorMap* tm_ori,
                                               const CUtensorMap* tm_cmp,
                                               const CUtensorMap* tm_ori16,
                                               const CUtensorMap* tm_cmp16) {
  if (lsu) {
    __syncwarp();
    if (lane == 0) {
#pragma unroll
      for (int cg = 0; cg < kChunkGroups; ++cg) mbar_arrive(bar[cg]);
    }
    lsu_rows(a, sK, pw * 16, 0, 16, sa.row, sa.pool, lane, row_bytes, gran);
    return;
  }
  const int row0 = __shfl_sync(0xffffffffu, sa.row, 0);
  const int pool0 = __shfl_sync(0xffffffffu, sa.pool, 0);
  const bool run16 = __all_sync(0xffffffffu, pool0 >= 0 && sa.pool == pool0 && sa.row >= 0 &&
                                                 sa.row == row0 + (lane & 15));
  if (run16) {
    if (lane == 0) {
#pragma unroll
      for (int cg = 0; cg < kChunkGroups; ++cg)
        mbar_expect_tx(bar[cg], 16u * 128u * group_chunks(cg, c0, nchunks));
      const CUtensorMap* m = (pool0 == 1) ? tm_cmp16 : tm_ori16;
      const uint32_t dst = sK + (uint32_t)(pw * 16) * 128u;
      for (int c = c0; c < nchunks; ++c)
        tma_load_2d(dst + c * kChunkBytes, m, c * 64, row0, bar[chunk_group(c)]);
    }
  } else {
    tma_rows(a, tm_ori, tm_cmp, c0, nchunks, sK, bar, pw * 16, sa.row, sa.pool, lane, row_bytes,
             gran);
  }
}

// Gather helper h: chunks kHelperChunk0 .. nchunks - 1 of tile rows 32 h ..
// 32 h + 31 (lane l: row 32 h + l), whose sources producer warps 2h and
// 2h + 1 left in gsrc.  Per 16-row block the same split as the producer's:
// a 16-row box per chunk when the block is 16 consecutive rows of one cache,
// else tile::gather4 per 4-row group; a group that mixes the two caches was
// moved whole by the producer's cp.async.  Lane 0 arrives once on the chunk
// group 2 barrier, arming the bytes of all ops.
__device__ __forceinline__ void helper_rows(const FwdArgs& a, const CUtensorMap* tm_ori,
                                            const CUtensorMap* tm_cmp,
                                            const CUtensorMap* tm_ori16,
                                            const CUtensorMap* tm_cmp16, const int32_t* gr,
                                            const int8_t* gp, int h, int lane, uint32_t sK,
                                            uint32_t bar, int nchunks) {
  const int row = gr[32 * h + lane];
  const int pool = gp[32 * h + lane];
  const uint32_t nch = (uint32_t)(nchunks - kHelperChunk0);
  const int row0 = __shfl_sync(0xffffffffu, row, lane & 16);
  const int pool0 = __shfl_sync(0xffffffffu, pool, lane & 16);
  const uint32_t run = __ballot_sync(0xffffffffu, pool0 >= 0 && pool == pool0 && row >= 0 &&
                                                      row == row0 + (lane & 15));
  const bool run_blk = ((run >> (lane & 16)) & 0xffffu) == 0xffffu;
  const int gl = lane & ~3;
  int prow[4], ppool[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    prow[i] = __shfl_sync(0xffffffffu, row, gl + i);
    ppool[i] = __shfl_sync(0xffffffffu, pool, gl + i);
  }
  int P = -1;
  bool mixed = false;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (ppool[i] >= 0) {
      if (P < 0) P = ppool[i];
      else if (ppool[i] != P) mixed = true;
    }
  }
  const bool box_leader = run_blk && (lane & 15) == 0;
  const bool grp_leader = !run_blk && (lane & 3) == 0 && !mixed;
  const uint32_t nbox = (uint32_t)__popc(__ballot_sync(0xffffffffu, box_leader));
  const uint32_t ngrp = (uint32_t)__popc(__ballot_sync(0xffffffffu, grp_leader));
  if (lane == 0) mbar_expect_tx(bar, (nbox * 16u + ngrp * 4u) * 128u * nch);
  __syncwarp();
  if (box_leader) {
    const CUtensorMap* m = (pool0 == 1) ? tm_cmp16 : tm_ori16;
    const uint32_t dst = sK + (uint32_t)(32 * h + (lane & 16)) * 128u;
    for (int c = kHelperChunk0; c < nchunks; ++c)
      tma_load_2d(dst + c * kChunkBytes, m, c * 64, row0, bar);
  }
  if (grp_leader) {
    const CUtensorMap* m = (P == 1) ? tm_cmp : tm_ori;
    const int sentinel = (P == 1) ? a.cmp_rows : a.ori_rows;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (ppool[i] < 0 || prow[i] < 0) prow[i] = sentinel;
    const uint32_t dst = sK + (uint32_t)(32 * h + lane) * 128u;
    for (int c = kHelperChunk0; c < nchunks; ++c)
      tma_gather4(dst + c * kChunkBytes, m, c * 64, prow[0], prow[1], prow[2], prow[3], bar);
  }
}

// Chunk group cg of S[sb] = Q K^T for the K tile at kb (chunks 3 cg ..
// 3 cg + 2): chunk c accumulates into partial c % kQkPartials, so
// consecutive MMAs rotate over the partials and their dependent chains
// overlap in the pipe; a partial's first chunk starts it at ks = 0.  Descriptors are
// built once and advanced by constant offsets (all shared addresses are
// below 256 KB, so the 14-bit address field never carries).
template <int kChunks>
__device__ __forceinline__ void issue_qk_group(uint32_t d, uint32_t sQ, uint32_t kb,
                                               uint32_t idesc, int cg) {
  const uint64_t dq = smem_desc(sQ, 16, 1024);
  const uint64_t dk = smem_desc(kb, 16, 1024);
  const int c0 = 3 * cg;
  const int nc = min(3, kChunks - c0);
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      if (i < nc) {
        const int c = c0 + i;
        const uint64_t off = (uint64_t)((c * kChunkBytes + ks * 32) >> 4);
        mma_ws(d + 32u * (c % kQkPartials), dq + off, dk + off, idesc,
               (c < kQkPartials && ks == 0) ? 0u : 1u);
      }
    }
  }
}

// O (+)= P V for the K tile at kb: P (64 x 64) from the rope chunk, V = dims
// 0..511 of the same tile read MN-major, two N = 256 halves.
__device__ __forceinline__ void issue_pv(uint32_t o, uint32_t kb, uint32_t idesc, bool first) {
  const uint64_t dp = smem_desc(kb + kPChunk * kChunkBytes, 16, 1024);
  const uint64_t dv = smem_desc(kb, kChunkBytes, 1024);
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
    for (int hv = 0; hv < 2; ++hv) {
      const uint64_t boff = (uint64_t)((4 * hv * kChunkBytes + ks * 2048) >> 4);
      mma_ws(o + 128u * hv, dp + (uint64_t)((ks * 32) >> 4), dv + boff, idesc,
             (first && ks == 0) ? 0u : 1u);
    }
  }
}

// Slots of tile j resolved by producer warp pw: keys 16 pw .. 16 pw + 15
// (lanes 16..31 mirror lanes 0..15).  `stopped`: a -1 occurred in an
// earlier tile of the row (the compressed scan stops there); each warp
// scans the whole tile for -1, so the stop prefix needs no cross-warp
// exchange.  Returns the slot source, its valid ballot in *valid.
__device__ __forceinline__ SlotSrc resolve_tile(const FwdArgs& a, const Row& rv,
                                                const QueryKeys& qk, const int* idx_row, int j,
                                                int pw, int lane, bool* stopped,
                                                uint32_t* valid, int* err) {
  uint64_t m1mask = 0;
  if (idx_row != nullptr) {
    const int ca = j * kTileKeys + lane - rv.window;
    const int cb = ca + 32;
    const bool ma = (ca >= 0 && ca < qk.cmp) && (__ldg(idx_row + ca) == -1);
    const bool mb = (cb >= 0 && cb < qk.cmp) && (__ldg(idx_row + cb) == -1);
    m1mask = (uint64_t)__ballot_sync(0xffffffffu, ma) |
             ((uint64_t)__ballot_sync(0xffffffffu, mb) << 32);
  }
  const int ka = pw * 16 + (lane & 15);
  const bool blk = *stopped || ((m1mask & ((1ull << ka) - 1ull)) != 0);
  const SlotSrc src = resolve_slot(a, rv, qk, j * kTileKeys + ka, idx_row, blk, err);
  if (m1mask != 0) *stopped = true;
  *valid = __ballot_sync(0xffffffffu, src.valid);
  return src;
}

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------

template <bool kBf16, int kChunks, bool kTrace>
__global__ void __launch_bounds__(kThreads, 1)
    sas_fwd_kernel(const FwdArgs args, const __grid_constant__ CUtensorMap tm_q,
                   const __grid_constant__ CUtensorMap tm_ori,
                   const __grid_constant__ CUtensorMap tm_cmp,
                   const __grid_constant__ CUtensorMap tm_ori16,
                   const __grid_constant__ CUtensorMap tm_cmp16) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ Ctl ctl;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int hg = args.head_groups;
  const int worker = blockIdx.x / hg;
  const int group = blockIdx.x % hg;
  const int* plan = args.plan;
  const int* rows = plan + plan[H_ROWS_OFF];
  constexpr int nchunks = kChunks;  // d_qk / 64
  int* err = args.err;
  long long* tr = (kTrace && (int)blockIdx.x == args.trace_cta) ? args.trace : nullptr;
  // Trace instances also record every CTA's start and end on the global
  // timer (ns), region 2 from 6144: [2 CTA] start, [2 CTA + 1] end.
  if (kTrace && threadIdx.x == 0 && args.trace != nullptr && blockIdx.x < 1024u)
    args.trace[2 * kTraceRegion + 6144 + 2 * blockIdx.x] = (long long)global_ns();

  // 1024-byte aligned tile area.
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t sQ = base + kSmemQ;
  const uint32_t sK0 = base + kSmemK0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      // Per producer warp: one arrival from lane 0 after the valid bits are
      // written (arming the TMA bytes in TMA mode) and one cp.async
      // completion arrival per lane.
      for (int g = 0; g < kChunkGroups; ++g)
        mbar_init(smem_addr(&ctl.kv_full[i][g]),
                  kNumProducerWarps + kProducerThreads + (g == 2 ? kNumHelperWarps : 0));
      mbar_init(smem_addr(&ctl.kv_empty[i]), 1);
      mbar_init(smem_addr(&ctl.s_full[i]), 1);
      mbar_init(smem_addr(&ctl.s_empty[i]), kSoftmaxThreads);
    }
    for (int h = 0; h < kNumHelperWarps; ++h)
      for (int i = 0; i < 2; ++i) mbar_init(smem_addr(&ctl.gready[h][i]), 2);
    mbar_init(smem_addr(&ctl.q_full), 1);
    mbar_init(smem_addr(&ctl.q_empty), 1);
    mbar_init(smem_addr(&ctl.p_full[0]), kSoftmaxThreads);
    mbar_init(smem_addr(&ctl.p_full[1]), kSoftmaxThreads);
    mbar_init(smem_addr(&ctl.o_free), kEpiThreads);
    mbar_init(smem_addr(&ctl.o_full), 1);
    mbar_init(smem_addr(&ctl.drain), 1);
    mbar_init(smem_addr(&ctl.xbar[0]), kSoftmaxThreads);
    mbar_init(smem_addr(&ctl.xbar[1]), kSoftmaxThreads);
    mbar_init(smem_addr(&ctl.fin_full[0]), kSoftmaxThreads);
    mbar_init(smem_addr(&ctl.fin_full[1]), kSoftmaxThreads);
    mbar_init(smem_addr(&ctl.fin_free[0]), kEpiThreads);
    mbar_init(smem_addr(&ctl.fin_free[1]), kEpiThreads);
    ctl.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    asm volatile(
        "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
            smem_addr(&ctl.tmem_base)),
        "r"(kTmemCols)
        : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl.tmem_base;

  const Span span = (worker < plan[H_NUM_WORKERS]) ? load_span(plan, worker) : Span{-1, 0, -1, 0, 0};

  if (warp >= kProducerWarp0 && warp < kProducerWarp0 + kNumProducerWarps) {
    // ======================= producers =======================
    const int pw = warp - kProducerWarp0;
    const bool leader = (pw == 0);
    const bool lsu = (args.gather == kGatherLsu);
    const int D = args.head_dim;
    const uint32_t row_bytes = (uint32_t)D * 2u;
    const int gran = D >> 3;  // 16-byte granules per row
    uint32_t kv_empty_par = 3u;  // bit = stage
    int stage = 0, produced = 0;
    bool ok = true;
    // Ring state: the stages hold the ring of sequence ring_b around
    // position ring_hi, ring half h in stage h ^ ring_sigma.
    bool ring_live = false;
    int ring_b = -1, ring_hi = 0, ring_sigma = 0;
    RowStream rs(rows, span.r0, span.r1);
    for (int r = span.r0; ok && span.r0 >= 0 && r <= span.r1; ++r) {
      const Row rv = rs.take(r);
      const int tiles = row_tiles(rv);
      const int ja = (r == span.r0) ? span.t0 : 0;
      const int jb = (r == span.r1) ? span.t1 : (tiles > 0 ? tiles : 1);
      if (tiles == 0 || ja >= jb) continue;

      // ---- ring rows: the window stays in the stages from query to query ----
      // The next query of the sequence (position hi + 1) keeps every key but
      // the one at hi - 127, whose slot receives the new key: per stage, the
      // rope chunk (overwritten by P) is loaded again for all 64 rows and,
      // in the stage holding the new key, chunks 0..7 of its 4-row group.
      // Any other row (a piece of a split row, another sequence, a gap)
      // loads both stages whole.
      if ((rv.flags & kRowRing) && !lsu && ja == 0 && jb == 2) {
        const int hi = rv.win_lo + rv.window - 1;
        const bool warm = ring_live && rv.b == ring_b && hi == ring_hi + 1;
        if (!warm) ring_sigma = stage;
        const int new_half = (hi >> 6) & 1, new_row = hi & 63;
        const int c_new = min(nchunks, kPChunk);  // chunks of the new row not in the rope load
        for (int k = 0; k < 2; ++k) {
          const int half = stage ^ ring_sigma;
          const SlotSrc sa = resolve_ring(args, rv, half, pw * 16 + (lane & 15), err);
          const uint32_t va_cur = __ballot_sync(0xffffffffu, sa.valid);
          if (args.slot_dump != nullptr && lane < 16)
            dump_slot(args, rv.token, half * kTileKeys + pw * 16 + lane, sa);
          if (leader && lane == 0) trace_in(tr, 0, 0, 3 * produced, 4096);
          if (!__all_sync(0xffffffffu, wait_bar(&ctl, &ctl.kv_empty[stage],
                                                (kv_empty_par >> stage) & 1u, err, 2))) {
            ok = false;
            break;
          }
          if (leader && lane == 0) trace_in(tr, 0, 0, 3 * produced + 1, 4096);
          kv_empty_par ^= 1u << stage;
          uint32_t bar[kChunkGroups];
#pragma unroll
          for (int cg = 0; cg < kChunkGroups; ++cg) bar[cg] = smem_addr(&ctl.kv_full[stage][cg]);
          const uint32_t sK = sK0 + stage * kStageBytes;
          if (lane == 0) ctl.valid[stage][pw] = (uint16_t)(va_cur & 0xffffu);
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_addr(&ctl.gready[pw >> 1][stage]));
          const bool owner = warm && half == new_half && (new_row >> 4) == pw;
          if (owner && lane == 0) {
#pragma unroll
            for (int cg = 0; cg < kChunkGroups; ++cg)
              mbar_add_tx(bar[cg], 4u * 128u * group_chunks(cg, 0, c_new));
          }
          __syncwarp();
          load_tile_rows(args, sa, warm ? kPChunk : 0, nchunks, sK, bar, pw, lane, false,
                         row_bytes, gran, &tm_ori, &tm_cmp, &tm_ori16, &tm_cmp16);
          if (owner) {
            // chunks 0 .. c_new - 1 of the 4-row group holding the new key
            // (its three neighbours are rewritten with the same rows)
            const int g = (new_row & 15) >> 2;
            int rr[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              rr[q] = __shfl_sync(0xffffffffu, sa.row, 4 * g + q);
              if (rr[q] < 0) rr[q] = args.ori_rows;  // out of range: zero-filled
            }
            if (lane == 0) {
              const uint32_t dst = sK + (uint32_t)(pw * 16 + 4 * g) * 128u;
              for (int c = 0; c < c_new; ++c)
                tma_gather4(dst + c * kChunkBytes, &tm_ori, c * 64, rr[0], rr[1], rr[2], rr[3],
                            bar[chunk_group(c)]);
            }
          }
#pragma unroll
          for (int cg = 0; cg < kChunkGroups; ++cg) cp_async_arrive_noinc(bar[cg]);
          if (leader && lane == 0) trace_in(tr, 0, 0, 3 * produced + 2, 4096);
          ++produced;
          stage ^= 1;
        }
        ring_live = ok;
        ring_b = rv.b;
        ring_hi = hi;
        continue;
      }
      ring_live = false;

      // ---- key tiles (key bounds precomputed by the planner) ----
      QueryKeys qk;
      qk.window = rv.window;
      qk.win_lo = rv.win_lo;
      qk.cmp = rv.cmp;
      qk.thr = rv.thr;
      qk.cmp_len = 0;
      const int* idx_row = (args.scenario == SAS_SCENARIO_SCFA)
                               ? args.cmp_indices + (size_t)rv.token * args.topk
                               : nullptr;
      // Slots before this piece may hold a -1 that stops the scan: 512
      // indices per step, 16 independent loads per lane in flight.
      bool stopped = false;
      if (idx_row != nullptr && ja > 0) {
        const int lim = min(ja * kTileKeys - rv.window, qk.cmp);
        for (int c0 = 0; c0 < lim && !stopped; c0 += 512) {
          bool m1 = false;
#pragma unroll
          for (int u = 0; u < 16; ++u) {
            const int c = c0 + 32 * u + lane;
            m1 |= (c < lim) && (__ldg(idx_row + c) == -1);
          }
          stopped = __any_sync(0xffffffffu, m1);
        }
      }
      // Tiles are resolved one ahead, so the index and block-table loads of
      // the next tile overlap this tile's wait for its stage.
      uint32_t va = 0;
      SlotSrc nxt = resolve_tile(args, rv, qk, idx_row, ja, pw, lane, &stopped, &va, err);
      for (int j = ja; j < jb; ++j) {
        const SlotSrc sa = nxt;
        const uint32_t va_cur = va;
        if (args.slot_dump != nullptr && lane < 16)
          dump_slot(args, rv.token, j * kTileKeys + pw * 16 + lane, sa);
        if (j + 1 < jb) {
          nxt = resolve_tile(args, rv, qk, idx_row, j + 1, pw, lane, &stopped, &va, err);
        }
        if (leader && lane == 0) trace_in(tr, 0, 0, 3 * produced, 4096);
        if (!__all_sync(0xffffffffu,
                        wait_bar(&ctl, &ctl.kv_empty[stage], (kv_empty_par >> stage) & 1u, err, 2))) {
          ok = false;
          break;
        }
        if (leader && lane == 0) trace_in(tr, 0, 0, 3 * produced + 1, 4096);
        kv_empty_par ^= 1u << stage;
        uint32_t bar[kChunkGroups];
#pragma unroll
        for (int cg = 0; cg < kChunkGroups; ++cg) bar[cg] = smem_addr(&ctl.kv_full[stage][cg]);
        const uint32_t sK = sK0 + stage * kStageBytes;
        if (lane == 0) ctl.valid[stage][pw] = (uint16_t)(va_cur & 0xffffu);
        // The gather helper of this warp pair loads chunks kHelperChunk0.. in
        // TMA mode; it reads the sources from gsrc once both warps arrived.
        if (lane < 16) {
          ctl.gsrc_row[stage][pw * 16 + lane] = sa.row;
          ctl.gsrc_pool[stage][pw * 16 + lane] = (int8_t)sa.pool;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(&ctl.gready[pw >> 1][stage]));
        load_tile_rows(args, sa, 0, lsu ? nchunks : min(nchunks, kHelperChunk0), sK, bar, pw,
                       lane, lsu, row_bytes, gran, &tm_ori, &tm_cmp, &tm_ori16, &tm_cmp16);
#pragma unroll
        for (int cg = 0; cg < kChunkGroups; ++cg) cp_async_arrive_noinc(bar[cg]);
        if (leader && lane == 0) trace_in(tr, 0, 0, 3 * produced + 2, 4096);
        ++produced;
        stage ^= 1;
      }
    }
    cp_async_wait_all();
  } else if (warp >= kHelperWarp0 && warp < kHelperWarp0 + kNumHelperWarps) {
    // ======================= gather helpers =======================
    // Same tile sequence as the producers: per tile, wait until producer
    // warps 2h, 2h + 1 have the stage free and its sources in gsrc, then
    // load chunk group 2 of their rows (plain TMA tiles) or just arrive
    // (ring rows, cp.async mode: the producers load every chunk).
    const int h = warp - kHelperWarp0;
    const bool lsu = (args.gather == kGatherLsu);
    uint32_t gready_par = 0u;  // bit = stage
    int stage = 0;
    bool ok = true;
    RowStream rs(rows, span.r0, span.r1);
    for (int r = span.r0; ok && span.r0 >= 0 && r <= span.r1; ++r) {
      const Row rv = rs.take(r);
      const int tiles = row_tiles(rv);
      const int ja = (r == span.r0) ? span.t0 : 0;
      const int jb = (r == span.r1) ? span.t1 : (tiles > 0 ? tiles : 1);
      if (tiles == 0 || ja >= jb) continue;
      const bool ring = (rv.flags & kRowRing) && !lsu && ja == 0 && jb == 2;
      for (int j = ja; j < jb; ++j) {
        if (!__all_sync(0xffffffffu, wait_bar(&ctl, &ctl.gready[h][stage],
                                              (gready_par >> stage) & 1u, err, 3))) {
          ok = false;
          break;
        }
        gready_par ^= 1u << stage;
        const uint32_t bar = smem_addr(&ctl.kv_full[stage][2]);
        if (ring || lsu || nchunks <= kHelperChunk0) {
          if (lane == 0) mbar_arrive(bar);
        } else {
          helper_rows(args, &tm_ori, &tm_cmp, &tm_ori16, &tm_cmp16, ctl.gsrc_row[stage],
                      ctl.gsrc_pool[stage], h, lane, sK0 + stage * kStageBytes, bar, nchunks);
        }
        stage ^= 1;
      }
    }
  } else if (warp == kQWarp) {
    // ======================= Q loader =======================
    // Q of a row (64 heads of this group, one 64 x 64 TMA box per chunk) is
    // loaded once the last QK of the previous row has released the Q buffer;
    // the next row's Q is prefetched into L2 meanwhile, so that wait is
    // followed by an L2 read rather than an HBM one.
    if (lane == 0) {
      const uint32_t q_bytes = (uint32_t)kHeadsPerCta * (uint32_t)args.head_dim * 2u;
      uint32_t q_empty_par = 1u;
      int q_loads = 0;
      int next = span.r0;  // first row whose Q has not been prefetched
      auto qrow_of = [&](int r, int* qrow) -> bool {
        const Row rv = load_row(rows, r);
        const int tiles = row_tiles(rv);
        const int ja = (r == span.r0) ? span.t0 : 0;
        const int jb = (r == span.r1) ? span.t1 : (tiles > 0 ? tiles : 1);
        *qrow = rv.token * args.num_heads + group * kHeadsPerCta;
        return tiles > 0 && ja < jb;
      };
      for (int r = span.r0; span.r0 >= 0 && r <= span.r1; ++r) {
        int qrow;
        if (!qrow_of(r, &qrow)) continue;
        // L2 prefetch of the next row that has key tiles.
        for (next = max(next, r + 1); next <= span.r1; ++next) {
          int nq;
          if (qrow_of(next, &nq)) {
            for (int c = 0; c < nchunks; ++c) tma_prefetch_2d(&tm_q, c * 64, nq);
            ++next;
            break;
          }
        }
        if (!wait_bar(&ctl, &ctl.q_empty, q_empty_par, err, 1)) break;
        q_empty_par ^= 1u;
        trace_in(tr, 3, 4096, q_loads++, 2048);
        mbar_expect_tx(smem_addr(&ctl.q_full), q_bytes);
        for (int c = 0; c < nchunks; ++c)
          tma_load_2d(sQ + c * kChunkBytes, &tm_q, c * 64, qrow, smem_addr(&ctl.q_full));
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ======================= MMA issuer =======================
    if (lane == 0) {
      const uint32_t idesc_qk = instr_desc(64, 64, kBf16, false, false);
      const uint32_t idesc_pv = instr_desc(64, 256, kBf16, false, true);
      // Barrier parities as bits: kv_full (bit = stage), s_empty (bit = S buffer).
      uint32_t kv_full_par = 0u, s_empty_par = 3u;
      uint32_t q_full_par = 0u, p_full_par = 0u, o_free_par = 1u;
      int pv_issued = 0, qk_issued = 0, q_seen = 0;
      bool ok = true;
      // Shared memory the MMAs read is written by TMA (async proxy) or by the
      // softmax threads, which fence it to the async proxy before arriving on
      // p_full, so this thread needs no proxy fence of its own.
      // The worker's tiles form one stream across rows; tile t uses K stage
      // t % 2 and S buffer t % 2.  QKs and PVs are issued as two independent
      // in-order streams, each step as soon as its inputs are in: PV(t)
      // after QK(t) and P(t) (and, for a row's first PV, the epilogue's
      // release of O); QK(t) one chunk group at a time after its Q, its S
      // buffer (released by softmax(t - 2)) and the group's K rows.  A PV
      // that is ready goes first: it releases the K stage that the load two
      // tiles ahead waits for.  Nothing else orders the two streams, so a row
      // boundary or a late softmax does not hold back the next QK.
      TileCursor qc(rows, span), pc(rows, span);
      int qstage = 0, pstage = 0;
      int pending = 0;            // tiles whose QK is issued and PV is not
      int qg = 0;                 // chunk groups of QK(qc) issued
      bool q_ok = false, s_ok = false, p_ok = false, o_ok = false;
      long long t_idle = clock64();
      while (ok && (qc.valid || pending > 0)) {
        bool progress = false;
        // ---- PV of the oldest tile whose QK is issued ----
        if (pending > 0) {
          if (!p_ok && mbar_test(smem_addr(&ctl.p_full[pstage]), (p_full_par >> pstage) & 1u)) {
            p_ok = true;
            p_full_par ^= 1u << pstage;
          }
          if (!o_ok) {
            if (!pc.first()) {
              o_ok = true;
            } else if (mbar_test(smem_addr(&ctl.o_free), o_free_par)) {
              o_ok = true;
              o_free_par ^= 1u;
            }
          }
          if (p_ok && o_ok) {
            trace(tr, 1, 4 * pv_issued + 2);
            tc_fence_after();
            issue_pv(tmem + kTmemO, sK0 + pstage * kStageBytes, idesc_pv, pc.first());
            trace(tr, 1, 4 * pv_issued + 3);
            tc_commit(smem_addr(&ctl.kv_empty[pstage]));
            if (pc.last()) tc_commit(smem_addr(&ctl.o_full));
            ++pv_issued;
            --pending;
            pc.advance();
            pstage ^= 1;
            p_ok = o_ok = false;
            progress = true;
          }
        }
        // ---- QK of the next tile, one chunk group at a time ----
        if (qc.valid) {
          if (!q_ok) {
            if (!qc.first()) {
              q_ok = true;
            } else if (mbar_test(smem_addr(&ctl.q_full), q_full_par)) {
              q_ok = true;
              q_full_par ^= 1u;
              trace_in(tr, 3, 6144, q_seen++, 2048);
            }
          }
          if (q_ok && !s_ok) trace_in(tr, 3, 1024, 2 * qk_issued + 1, 1024);
          if (q_ok && !s_ok &&
              mbar_test(smem_addr(&ctl.s_empty[qstage]), (s_empty_par >> qstage) & 1u)) {
            s_ok = true;
            s_empty_par ^= 1u << qstage;
            trace(tr, 1, 4 * qk_issued);
          }
          if (s_ok &&
              mbar_test(smem_addr(&ctl.kv_full[qstage][qg]), (kv_full_par >> qstage) & 1u)) {
            trace_in(tr, 3, 2048, 3 * qk_issued + qg, 2048);
            tc_fence_after();
            issue_qk_group<nchunks>(tmem + kTmemS + 128u * qstage, sQ,
                                    sK0 + qstage * kStageBytes, idesc_qk, qg);
            progress = true;
            if (++qg == kChunkGroups) {
              kv_full_par ^= 1u << qstage;
              trace(tr, 1, 4 * qk_issued + 1);
              ++qk_issued;
              tc_commit(smem_addr(&ctl.s_full[qstage]));
              if (qc.last()) tc_commit(smem_addr(&ctl.q_empty));
              trace_in(tr, 3, 1024, 2 * qk_issued, 1024);
              qc.advance();
              qstage ^= 1;
              ++pending;
              qg = 0;
              q_ok = s_ok = false;
            }
          }
        }
        if (progress) {
          t_idle = clock64();
        } else {
          if (ctl.abort) {
            ok = false;
            break;
          }
          if (clock64() - t_idle > kWaitCycles) {
            record_error(err, SAS_ERR_DEVICE, 23, pv_issued);
            ctl.abort = 1;
            ok = false;
            break;
          }
        }
      }
      // Drain: the commit arrives once every MMA issued above has finished,
      // so TMEM is never released under an in-flight MMA (also on abort).
      tc_commit(smem_addr(&ctl.drain));
      wait_bar(&ctl, &ctl.drain, 0u, err, 25);
    }
    __syncwarp();
  } else if (warp >= kEpiWarp0) {
    // ======================= epilogue =======================
    // Per (row, piece) with key tiles, in plan order: wait until its O is
    // complete (o_full, committed after its last PV) and its statistics are
    // in (fin_full), write O / l and the LSE (or the fp32 split partials),
    // then release O (o_free) for the next piece's first PV.  Warp w reads
    // TMEM lanes 32 (w % 4) .. +31: heads (w & 1) * 32 + lane, key half w / 2
    // of the .ws accumulator layout.
    const int ew = warp - kEpiWarp0;
    const int half = ew >> 1;
    const int m0 = (ew & 1) * 32;
    const int m = m0 + lane;
    const int dv = args.head_dim_v;
    const uint32_t obase = tmem + ((uint32_t)(ew * 32) << 16) + kTmemO;
    const int nlive = min(32, max(0, args.num_heads - (group * kHeadsPerCta + m0)));
    uint8_t* stg = ctl.epi[ew];
    int k = 0;  // pieces finished
    RowStream rs(rows, span.r0, span.r1);
    for (int r = span.r0; span.r0 >= 0 && r <= span.r1; ++r) {
      const Row rv = rs.take(r);
      const int tiles = row_tiles(rv);
      const int ja = (r == span.r0) ? span.t0 : 0;
      const int jb = (r == span.r1) ? span.t1 : (tiles > 0 ? tiles : 1);
      if (tiles == 0 || ja >= jb) continue;
      const int fp = k & 1;
      if (!__all_sync(0xffffffffu, wait_bar(&ctl, &ctl.o_full, (uint32_t)(k & 1), err, 40)))
        break;
      if (!__all_sync(0xffffffffu,
                      wait_bar(&ctl, &ctl.fin_full[fp], (uint32_t)((k >> 1) & 1), err, 41)))
        break;
      tc_fence_after();
      if (ew == 0 && lane == 0) trace_in(tr, 3, 0, 3 * k + 1, 1024);
      const float m_run = ctl.fin_m[fp][m];
      const float l_tot = ctl.fin_l[fp][0][m] + ctl.fin_l[fp][1][m];
      mbar_arrive(smem_addr(&ctl.fin_free[fp]));  // statistics read: the buffer is free
      const float inv = (l_tot > 0.f) ? 1.f / l_tot : 0.f;
      const float lse = (m_run + log2f(l_tot)) * kLn2;
      const bool split = rv.partial_base >= 0;
      const int piece = (r == span.r0) ? span.piece0 : 0;
      const size_t row0 = split ? (size_t)(rv.partial_base + piece) * args.num_heads +
                                      group * kHeadsPerCta + m0
                                : (size_t)rv.token * args.num_heads + group * kHeadsPerCta + m0;
      char* seg_base = split ? reinterpret_cast<char*>(args.o_partial + row0 * dv)
                             : reinterpret_cast<char*>(args.out) + row0 * dv * 2;
      for (int c = 0; c < 8; ++c) {
        uint32_t v[32];
        tmem_ld32(obase + 32u * c, v);
        tmem_wait_ld();
        epi_block<kBf16>(v, c, half, inv, split, seg_base, dv, stg, lane, nlive);
      }
      if (half == 0 && lane < nlive) {
        if (split)
          args.lse_partial[row0 + lane] = lse;
        else
          args.lse[row0 + lane] = lse;
      }
      tc_fence_before();
      mbar_arrive(smem_addr(&ctl.o_free));
      if (ew == 0 && lane == 0) trace_in(tr, 3, 0, 3 * k + 2, 1024);
      ++k;
    }
  } else if (warp < kNumSoftmaxWarps) {
    // ======================= softmax =======================
    const int L = threadIdx.x;           // TMEM lane 0..127
    const int m = L & (kHeadsPerCta - 1);  // head row inside the group
    const int half = L >> 6;             // key half / output half
    const int head = group * kHeadsPerCta + m;
    const bool live = head < args.num_heads;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const float c2 = args.softmax_scale * kLog2e;
    const float sink = live ? __ldg(args.sinks + head) : -INFINITY;
    uint32_t kv_full_par = 0u, s_full_par = 0u;  // bit = stage / S buffer
    int pv_count = 0;  // PVs released by this thread's p_full arrivals so far
    int rows_done = 0;
    // Completion of PV number k: phase k/2 of kv_empty[k % 2] (its commit
    // also releases the K stage).  When softmax waits for PV k, PV k-2 is
    // complete (the S of the current tile is only produced after the PV two
    // tiles back freed its K stage) and PV k+2 is not yet released, so
    // kv_empty[k % 2] is exactly one phase short of or at the awaited
    // completion and the parity test is exact.

    uint32_t xph = 0u;  // bit = exchange barrier
    int stage = 0, sbuf = 0, xpar = 0;
    // Partner exchange through ctl.red[xpar], ordered by the bounded
    // mbarrier ctl.xbar[xpar] (all 128 softmax threads arrive, then wait).

    bool ok = true;
    const int dv = args.head_dim_v;

    for (int r = span.r0; ok && span.r0 >= 0 && r <= span.r1; ++r) {
      // (loaded at the row start, not prefetched: the softmax's registers go
      // to the score tile)
      const Row rv = load_row(rows, r);
      const int tiles = row_tiles(rv);
      const int ja = (r == span.r0) ? span.t0 : 0;
      const int jb = (r == span.r1) ? span.t1 : (tiles > 0 ? tiles : 1);
      if (ja >= jb) continue;
      const size_t orow = (size_t)rv.token * args.num_heads + head;
      if (tiles == 0) {
        // No key slot: out = 0, lse = sink (golden.py:162-200), padded rows 0.
        if (live) {
          uint4* o = reinterpret_cast<uint4*>(reinterpret_cast<char*>(args.out) +
                                              (orow * dv + half * (dv / 2)) * 2);
          for (int i = 0; i < dv / 16; ++i) o[i] = make_uint4(0, 0, 0, 0);
          if (half == 0) args.lse[orow] = (rv.flags & kRowPadded) ? 0.f : sink;
        }
        continue;
      }
      const bool first_piece = (ja == 0);
      float m_run = first_piece ? sink * kLog2e : -INFINITY;  // log2 domain
      float l_run = (first_piece && half == 0) ? 1.f : 0.f;
      for (int j = ja; j < jb; ++j) {
        const int st = stage, sb = sbuf;
        stage ^= 1;
        sbuf ^= 1;
        if (!__all_sync(0xffffffffu, wait_bar(&ctl, &ctl.s_full[sb], (s_full_par >> sb) & 1u, err, 30))) { ok = false; break; }
        s_full_par ^= 1u << sb;
        if (threadIdx.x == 0) trace_in(tr, 2, 0, 4 * pv_count + 3, 6144);
        if (!__all_sync(0xffffffffu, wait_bar(&ctl, &ctl.kv_full[st][0], (kv_full_par >> st) & 1u, err, 31))) { ok = false; break; }
        kv_full_par ^= 1u << st;
        if (threadIdx.x == 0) trace_in(tr, 2, 0, 4 * pv_count, 6144);
        tc_fence_after();
        uint32_t sraw[32];
        {
          // S = sum of the partial accumulators (two: both loaded before one
          // wait; four: 16 columns at a time).
          const uint32_t ts = tmem + lane_off + kTmemS + 128u * sb;
          tmem_ld32(ts, sraw);
          if constexpr (kQkPartials == 2) {
            uint32_t t2[32];
            tmem_ld32(ts + 32u, t2);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i)
              sraw[i] = __float_as_uint(__uint_as_float(sraw[i]) + __uint_as_float(t2[i]));
          } else {
            tmem_wait_ld();
          }
#pragma unroll
          for (int pp = (kQkPartials == 2 ? 2 : 1); pp < kQkPartials; ++pp) {
#pragma unroll
            for (int h16 = 0; h16 < 2; ++h16) {
              uint32_t t1[16];
              tmem_ld16(ts + 32u * pp + 16u * h16, t1);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 16; ++i)
                sraw[16 * h16 + i] =
                    __float_as_uint(__uint_as_float(sraw[16 * h16 + i]) + __uint_as_float(t1[i]));
            }
          }
        }
        tc_fence_before();
        mbar_arrive(smem_addr(&ctl.s_empty[sb]));
        if (lane == 0) trace_in(tr, 0, 4096, 4 * pv_count + warp, 4096);
        const uint32_t vb = (uint32_t)ctl.valid[st][2 * half] |
                            ((uint32_t)ctl.valid[st][2 * half + 1] << 16);
        float x[32];
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float v = ((vb >> i) & 1u) ? __uint_as_float(sraw[i]) * c2 : -INFINITY;
          x[i] = v;
          mx = fmaxf(mx, v);
        }
        ctl.red[xpar][half][m] = mx;
        mbar_arrive(smem_addr(&ctl.xbar[xpar]));
        const bool xw = wait_bar(&ctl, &ctl.xbar[xpar], (xph >> xpar) & 1u, err, 34);
        xph ^= 1u << xpar;
        if (!__all_sync(0xffffffffu, xw)) { ok = false; break; }
        mx = fmaxf(mx, ctl.red[xpar][half ^ 1][m]);
        xpar ^= 1;
        if (threadIdx.x == 0) trace_in(tr, 2, 0, 4 * pv_count + 1, 6144);
        const float m_new = fmaxf(m_run, mx);
        const bool rescale = (m_new - m_run) > kRescaleThreshold;  // NaN (-inf,-inf) -> false
        float alpha = 1.f;
        if (rescale) {
          alpha = exp2f(m_run - m_new);
          m_run = m_new;
          l_run *= alpha;
        }
        const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
        float lsum = 0.f;
        // P(j) into chunk 8 of tile j's own stage (free: S(j) is complete),
        // one 16-byte granule (8 keys) at a time.
        uint8_t* prow = gbase + kSmemK0 + st * kStageBytes + kPChunk * kChunkBytes;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          uint32_t pk[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int i = 8 * g + 2 * q;
            const float p0 = ex2_approx(x[i] - m_use);
            const float p1 = ex2_approx(x[i + 1] - m_use);
            lsum += p0 + p1;
            pk[q] = pack2<kBf16>(p0, p1);
          }
          *reinterpret_cast<uint4*>(prow + swz(m, 4 * half + g)) =
              make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
        l_run += lsum;
        fence_proxy_async();
        // The running max moved by more than the lazy threshold: O must be
        // rescaled after PV(j-1) (number pv_count - 1) and before PV(j).
        if (j > ja && __any_sync(0xffffffffu, rescale)) {
          const int kp = pv_count - 1;  // PV(j-1): phase kp / 2 of kv_empty[kp % 2]
          if (!__all_sync(0xffffffffu, wait_bar(&ctl, &ctl.kv_empty[kp & 1],
                                                (uint32_t)((kp >> 1) & 1), err, 32))) {
            ok = false;
            break;
          }
          tc_fence_after();
          // 16 columns at a time (a rare path; keeps the softmax's registers low)
#pragma unroll 1
          for (int c = 0; c < 16; ++c) {
            const uint32_t ta = tmem + lane_off + kTmemO + 16u * c;
            uint32_t v[16];
            tmem_ld16(ta, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * alpha);
            tmem_st16(ta, v);
          }
          tmem_wait_st();
        }
        tc_fence_before();
        if (threadIdx.x == 0) trace_in(tr, 2, 0, 4 * pv_count + 2, 6144);
        mbar_arrive(smem_addr(&ctl.p_full[st]));
        ++pv_count;
      }
      if (!ok) break;
      // ---- hand this (row, piece)'s statistics to the epilogue (producer
      // warps); m_run is identical in both key halves ----
      const int fp = rows_done & 1;
      // The epilogue has read piece rows_done - 2 from this buffer (phase
      // rows_done / 2 - 1 of fin_free[fp]; the first use passes at once).
      if (!__all_sync(0xffffffffu, wait_bar(&ctl, &ctl.fin_free[fp],
                                            (uint32_t)(((rows_done >> 1) & 1) ^ 1), err, 35)))
        break;
      if (half == 0) ctl.fin_m[fp][m] = m_run;
      ctl.fin_l[fp][half][m] = l_run;
      mbar_arrive(smem_addr(&ctl.fin_full[fp]));
      if (threadIdx.x == 0) trace_in(tr, 3, 0, 3 * rows_done, 1024);
      ++rows_done;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (kTrace && threadIdx.x == 0 && args.trace != nullptr && blockIdx.x < 1024u)
    args.trace[2 * kTraceRegion + 6144 + 2 * blockIdx.x + 1] = (long long)global_ns();
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

}  // namespace

// cuTensorMapEncodeTiled through the runtime's driver entry point (no
// link-time dependency on libcuda).
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2D map over a row-major [rows, cols] 16-bit matrix with a (64 x box_rows)
// box, 128-byte swizzle, zero fill out of range.
static bool make_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols,
                     uint32_t box_rows) {
  auto fn = encode_fn();
  if (fn == nullptr || base == nullptr || rows == 0) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <bool kBf16, int kChunks, bool kTrace>
static int launch_one(const FwdArgs& args, int grid, cudaStream_t stream, const CUtensorMap& tm_q,
                      const CUtensorMap& tm_ori, const CUtensorMap& tm_cmp,
                      const CUtensorMap& tm_ori16, const CUtensorMap& tm_cmp16) {
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(sas_fwd_kernel<kBf16, kChunks, kTrace>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmemDynamic) != cudaSuccess)
      return SAS_ERR_CUDA;
    configured = true;
  }
  sas_fwd_kernel<kBf16, kChunks, kTrace><<<grid, kThreads, kSmemDynamic, stream>>>(
      args, tm_q, tm_ori, tm_cmp, tm_ori16, tm_cmp16);
  return cudaGetLastError() == cudaSuccess ? SAS_OK : SAS_ERR_CUDA;
}

int launch_fwd(const FwdArgs& args, int grid, cudaStream_t stream) {
  const bool bf16 = args.dtype == SAS_DTYPE_BF16;
  if (args.head_dim != 576 && args.head_dim != 512) return SAS_ERR_UNSUPPORTED;
  // Key-cache maps: one-row boxes (gather4 and single rows) and 16-row
  // boxes (runs of 16 consecutive rows).
  alignas(64) CUtensorMap tm_q, tm_ori, tm_cmp, tm_ori16, tm_cmp16;
  const uint64_t D = (uint64_t)args.head_dim;
  if (!make_map(&tm_q, args.q, (uint64_t)args.total_tokens * args.num_heads, D, kHeadsPerCta))
    return SAS_ERR_CUDA;
  if (!make_map(&tm_ori, args.ori_kv, (uint64_t)args.ori_rows, D, 1)) return SAS_ERR_CUDA;
  // A cache with fewer than 16 rows never takes the 16-row run path, so its
  // 16-row map is encoded with a box that fits the cache.
  const uint32_t ori_box = args.ori_rows < 16 ? (uint32_t)args.ori_rows : 16u;
  const uint32_t cmp_box = args.cmp_rows < 16 ? (uint32_t)args.cmp_rows : 16u;
  if (!make_map(&tm_ori16, args.ori_kv, (uint64_t)args.ori_rows, D, ori_box)) return SAS_ERR_CUDA;
  if (args.cmp_kv != nullptr && args.cmp_rows > 0) {
    if (!make_map(&tm_cmp, args.cmp_kv, (uint64_t)args.cmp_rows, D, 1)) return SAS_ERR_CUDA;
    if (!make_map(&tm_cmp16, args.cmp_kv, (uint64_t)args.cmp_rows, D, cmp_box)) return SAS_ERR_CUDA;
  } else {
    tm_cmp = tm_ori;
    tm_cmp16 = tm_ori16;
  }
  // The trace instances carry the clock-trace stores; the others have none.
#define SAS_LAUNCH(B, C, T) launch_one<B, C, T>(args, grid, stream, tm_q, tm_ori, tm_cmp, tm_ori16, tm_cmp16)
  const bool t = args.trace != nullptr;
  if (args.head_dim == 576) {
    if (bf16) return t ? SAS_LAUNCH(true, 9, true) : SAS_LAUNCH(true, 9, false);
    return t ? SAS_LAUNCH(false, 9, true) : SAS_LAUNCH(false, 9, false);
  }
  if (bf16) return t ? SAS_LAUNCH(true, 8, true) : SAS_LAUNCH(true, 8, false);
  return t ? SAS_LAUNCH(false, 8, true) : SAS_LAUNCH(false, 8, false);
#undef SAS_LAUNCH
}

}  // namespace sas
