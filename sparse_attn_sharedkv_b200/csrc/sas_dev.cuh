// Device helpers shared by the attention kernels (sas_fwd.cu: one CTA per
// 64-head group; sas_fwd_pair.cu: a cluster of two CTAs issuing
// cta_group::2 MMAs): PTX wrappers for mbarriers, TMA, tcgen05 and TMEM,
// the plan walk (rows, worker spans, tile cursor), the slot -> key-row
// resolution of golden.py:28-66 and the coalesced epilogue stores.
// Included once per translation unit; everything is internal to it.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "sas.h"
#include "sas_internal.h"
#include "sas_kernels.h"

namespace sas {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // lazy O rescale (log2 units)

constexpr long long kWaitCycles = 4000000000LL;  // ~2 s at 2 GHz

// Independent S accumulators per tile: QK chunk c accumulates into partial
// c % kQkPartials and the softmax sums the partials it reads from TMEM.  Two
// partials (two accumulation chains, both read before one TMEM wait) measured
// faster than one or four on the benchmark workloads.
#ifndef SAS_QK_PARTIALS
#define SAS_QK_PARTIALS 2
#endif
constexpr int kQkPartials = SAS_QK_PARTIALS;

// ---------------------------------------------------------------------------
// PTX helpers.
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
               "r"(bytes)
               : "memory");
}

// Raises the transaction count of the current phase without arriving.
__device__ __forceinline__ void mbar_add_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

// 2D tiled TMA load of one box at (x, y) into shared memory.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Four rows (y0..y3) of one 128-byte column block x, written to 4 consecutive
// 128-byte rows at dst (the box of the map is one row high).
__device__ __forceinline__ void tma_gather4(uint32_t dst, const CUtensorMap* map, int x, int y0,
                                            int y1, int y2, int y3, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y0), "r"(y1), "r"(y2), "r"(y3), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}

__device__ __forceinline__ void cp_async_arrive_noinc(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// D[tmem] (+)= A[smem] * B[smem], weight-stationary form (M = 64 uses all
// 128 TMEM lanes: columns [0, N/2) on lanes 0-63, [N/2, N) on lanes 64-127).
__device__ __forceinline__ void mma_ws(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.ws.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 consecutive 32-bit columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// 16 consecutive 32-bit columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (sm_100 version 1).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor of kind::f16 with fp32 accumulation.
__host__ __device__ constexpr uint32_t instr_desc(int m, int n, bool bf16, bool a_mn, bool b_mn) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

// Byte offset of (row, 16-byte granule) inside a 128B-swizzled [rows x 64]
// 16-bit chunk: rows are 128 B apart, granules XOR-permuted by row % 8.
__device__ __forceinline__ uint32_t swz(int row, int granule) {
  return (uint32_t)(row * 128 + ((granule ^ (row & 7)) << 4));
}


struct Row {
  int token, b, s, slots, flags, first_worker, partial_base, window, win_lo, cmp, thr;
};

__device__ __forceinline__ Row load_row(const int* rows, int r) {
  const int4* p = reinterpret_cast<const int4*>(rows + (size_t)r * kRowInts);
  int4 a = __ldg(p), c = __ldg(p + 1), e = __ldg(p + 2);
  return Row{a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w, e.x, e.y, e.z};
}

// Plan rows of a worker span, each fetched one row ahead of its use so the
// global-load latency overlaps the previous row's work.
struct RowStream {
  const int* rows;
  int r1;
  Row next;
  __device__ __forceinline__ RowStream(const int* rows_, int r0, int r1_) : rows(rows_), r1(r1_) {
    if (r0 >= 0 && r0 <= r1) next = load_row(rows, r0);
  }
  __device__ __forceinline__ Row take(int r) {
    const Row cur = next;
    if (r + 1 <= r1) next = load_row(rows, r + 1);
    return cur;
  }
};

// Diagnostic clock trace of one CTA (FwdArgs::trace_cta), compiled only into
// the kernel instances launched with a trace buffer: 4 regions of 8192
// entries.  Single-CTA kernel layout (each sub-range holds the events of as
// many tiles / rows as fit; later ones are dropped, never written into the
// next sub-range):
//   region 0  [0, 4096) producer per tile (3 t: before the stage wait, stage
//             free, loads issued); [4096, 8192) S released by softmax warp w
//             of tile t (4 t + w)
//   region 1  MMA per tile: 4 t QK start (S buffer free), 4 t + 1 QK issued,
//             4 t + 2 / 4 t + 3 PV issue start / end
//   region 2  [0, 6144) softmax per tile (4 t: K rows seen, + 1 max exchanged,
//             + 2 P written, + 3 S seen); [6144, 8192) every CTA's start / end
//             on the global timer (ns), 2 per CTA
//   region 3  [0, 1024) rows: 3 k statistics handed on, 3 k + 1 / 3 k + 2
//             epilogue start / end; [1024, 2048) MMA loop per tile (2 t QK
//             committed, 2 t + 1 waiting for its S buffer); [2048, 4096) chunk
//             group g of tile t seen by the MMA issuer (3 t + g); [4096, 6144)
//             Q load issues; [6144, 8192) Q arrivals
constexpr int kTraceRegion = 8192;
__device__ __forceinline__ void trace(long long* tr, int region, int idx) {
  if (tr != nullptr && idx >= 0 && idx < kTraceRegion)
    tr[region * kTraceRegion + idx] = clock64();
}
// Entry base + idx of a region, written only while idx < limit.
__device__ __forceinline__ void trace_in(long long* tr, int region, int base, int idx,
                                         int limit) {
  if (tr != nullptr && idx >= 0 && idx < limit) tr[region * kTraceRegion + base + idx] = clock64();
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ void record_error(int* err, int code, int site, int detail) {
  if (err != nullptr && atomicCAS(err, 0, code) == 0) {
    err[1] = site;
    err[2] = detail;
    err[3] = (int)blockIdx.x;
  }
}

// Bounded wait; on timeout records the error and raises the CTA abort flag.
template <class CtlT>
__device__ __forceinline__ bool wait_bar(CtlT* ctl, uint64_t* bar, uint32_t parity, int* err,
                                         int site) {
  const uint32_t a = smem_addr(bar);
  if (mbar_try_wait(a, parity)) return true;
  long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(a, parity)) return true;
    if (ctl->abort) return false;
    if (clock64() - t0 > kWaitCycles) {
      record_error(err, SAS_ERR_DEVICE, site, (int)parity);
      ctl->abort = 1;
      return false;
    }
  }
}

// 2^x by the MUFU approximation (PTX ex2.approx.ftz.f32: relative error
// about 2^-22, results below 2^-126 flushed to zero; 2^-inf = 0): the
// softmax's P, which is rounded to bf16 / fp16 right after.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <bool kBf16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (kBf16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

// Iterate over the (row, tile range) segments of this CTA's worker span.
struct Span {
  int r0, t0, r1, t1, piece0;
};

__device__ __forceinline__ Span load_span(const int* plan, int worker) {
  const int* w = plan + plan[H_WORKERS_OFF] + worker * kWorkerInts;
  return Span{__ldg(w), __ldg(w + 1), __ldg(w + 2), __ldg(w + 3), __ldg(w + 4)};
}

__device__ __forceinline__ int row_tiles(const Row& rv) {
  return (rv.slots + kTileKeys - 1) / kTileKeys;
}

// Walks the (row, tile) units of a worker span in plan order, skipping rows
// without key tiles.  first / last: the tile opens / closes its (row, piece).
struct TileCursor {
  RowStream rs;
  Span span;
  int r, j, ja, jb;
  bool valid;
  __device__ __forceinline__ TileCursor(const int* rows, const Span& sp)
      : rs(rows, sp.r0, sp.r1), span(sp), r(sp.r0 - 1), j(0), ja(0), jb(0), valid(false) {
    next_row();
  }
  __device__ __forceinline__ void next_row() {
    valid = false;
    while (span.r0 >= 0 && ++r <= span.r1) {
      const Row rv = rs.take(r);
      const int tiles = row_tiles(rv);
      ja = (r == span.r0) ? span.t0 : 0;
      jb = (r == span.r1) ? span.t1 : (tiles > 0 ? tiles : 1);
      if (tiles > 0 && ja < jb) {
        j = ja;
        valid = true;
        return;
      }
    }
  }
  __device__ __forceinline__ void advance() {
    if (++j >= jb) next_row();
  }
  __device__ __forceinline__ bool first() const { return j == ja; }
  __device__ __forceinline__ bool last() const { return j + 1 == jb; }
};

// Source of one key slot: pool 0 = window cache (ori_kv), 1 = compressed
// cache (cmp_kv), -1 = masked slot; row = block * block_size + offset in that
// pool, or -1 for an attended position whose page is unmapped (zero row).
struct SlotSrc {
  int row;
  int pool;
  bool valid;
};

// golden.py:28-66 / 125-150 for slot `slot` of query row `rv`.  `blocked`:
// a -1 precedes this slot in the compressed scan.  Page ids outside the pool
// are recorded in the error word and read as zero rows.
__device__ __forceinline__ SlotSrc resolve_slot(const FwdArgs& a, const Row& rv,
                                                const QueryKeys& qk, int slot,
                                                const int* idx_row, bool blocked, int* err) {
  SlotSrc r{-1, -1, false};
  if (slot < rv.window) {
    const int pos = qk.win_lo + slot;
    const int lb = pos / a.ori_block_size;
    r.valid = true;
    r.pool = 0;
    if (lb < a.ori_table_len) {
      const int blk = __ldg(a.ori_block_table + (size_t)rv.b * a.ori_table_len + lb);
      if (blk >= 0 && blk < a.ori_num_blocks)
        r.row = blk * a.ori_block_size + (pos - lb * a.ori_block_size);
      else if (blk >= a.ori_num_blocks)
        record_error(err, SAS_ERR_DEVICE, 10, blk);
    } else {
      record_error(err, SAS_ERR_DEVICE, 11, pos);
    }
  } else if (slot < rv.window + rv.cmp) {
    const int c = slot - rv.window;
    int pos = c;
    bool ok = true;
    if (idx_row != nullptr) {
      pos = __ldg(idx_row + c);
      ok = !blocked && pos >= 0 && pos < qk.thr;
    }
    if (ok) {
      r.valid = true;
      r.pool = 1;
      const int lb = pos / a.cmp_block_size;
      if (lb < a.cmp_table_len) {
        const int blk = __ldg(a.cmp_block_table + (size_t)rv.b * a.cmp_table_len + lb);
        if (blk >= 0 && blk < a.cmp_num_blocks)
          r.row = blk * a.cmp_block_size + (pos - lb * a.cmp_block_size);
        else if (blk >= a.cmp_num_blocks)
          record_error(err, SAS_ERR_DEVICE, 12, blk);
      } else {
        record_error(err, SAS_ERR_DEVICE, 13, pos);
      }
    }
  }
  return r;
}


// Diagnostic record of the key source of slot `slot` of token `token`
// (FwdArgs::slot_dump): 2 * row + cache, -2 - cache for an attended position
// whose page is unmapped, -1 for a masked slot.
__device__ __forceinline__ void dump_slot(const FwdArgs& a, int token, int slot,
                                          const SlotSrc& s) {
  if (slot >= a.slot_dump_cap) return;
  const int v = s.valid ? (s.row >= 0 ? s.row * 2 + s.pool : -2 - s.pool) : -1;
  a.slot_dump[(size_t)token * a.slot_dump_cap + slot] = v;
}

// Coalesced store of one warp's 32 rows x 32 bytes: lane i holds row i's
// 32 bytes in v[0..1].  The rows go through the warp's 1 KB staging buffer
// (16-byte slot q of row i at slot q ^ ((i >> 2) & 1): conflict-free both
// ways) and come back out as 16 rows per store instruction (lane j: row
// 16 s + j / 2, slot j % 2), i.e. whole 32-byte sectors.  Rows at or past
// `nlive` (heads >= H) are not written.
__device__ __forceinline__ void warp_store_rows32(uint8_t* stg, int lane, const uint4 (&v)[2],
                                                  char* seg0, size_t stride, int nlive) {
#pragma unroll
  for (int q = 0; q < 2; ++q)
    *reinterpret_cast<uint4*>(stg + lane * 32 + ((q ^ ((lane >> 2) & 1)) << 4)) = v[q];
  __syncwarp();
  const int u = lane & 1;
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const int hl = 16 * s + (lane >> 1);
    const uint4 w = *reinterpret_cast<const uint4*>(stg + hl * 32 + ((u ^ ((hl >> 2) & 1)) << 4));
    if (hl < nlive) *reinterpret_cast<uint4*>(seg0 + (size_t)hl * stride + u * 16) = w;
  }
  __syncwarp();
}

// Epilogue of one 32-column block c of O (this thread's head row): scale by
// 1 / l and store, as bf16/fp16 into out or as fp32 into the split partials.
// Column block c is accumulator c / 4, dims (c / 4) * 256 + half * 128 +
// (c % 4) * 32.  seg_base: the warp's first head row in out or in the
// partials, as bytes.
template <bool kBf16>
__device__ __forceinline__ void epi_block(const uint32_t (&v)[32], int c, int half, float inv,
                                          bool split, char* seg_base, int dv, uint8_t* stg,
                                          int lane, int nlive) {
  const int d0 = (c >> 2) * 256 + half * 128 + (c & 3) * 32;
  if (split) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 w[2];
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        const int i = 8 * q + 4 * g;
        w[g] = make_uint4(__float_as_uint(__uint_as_float(v[i]) * inv),
                          __float_as_uint(__uint_as_float(v[i + 1]) * inv),
                          __float_as_uint(__uint_as_float(v[i + 2]) * inv),
                          __float_as_uint(__uint_as_float(v[i + 3]) * inv));
      }
      warp_store_rows32(stg, lane, w, seg_base + (size_t)(d0 + 8 * q) * 4, (size_t)dv * 4, nlive);
    }
  } else {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint4 w[2];
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        const int i = 16 * h + 8 * g;
        w[g] = make_uint4(
            pack2<kBf16>(__uint_as_float(v[i]) * inv, __uint_as_float(v[i + 1]) * inv),
            pack2<kBf16>(__uint_as_float(v[i + 2]) * inv, __uint_as_float(v[i + 3]) * inv),
            pack2<kBf16>(__uint_as_float(v[i + 4]) * inv, __uint_as_float(v[i + 5]) * inv),
            pack2<kBf16>(__uint_as_float(v[i + 6]) * inv, __uint_as_float(v[i + 7]) * inv));
      }
      warp_store_rows32(stg, lane, w, seg_base + (size_t)(d0 + 16 * h) * 2, (size_t)dv * 2,
                        nlive);
    }
  }
}

}  // namespace
}  // namespace sas
