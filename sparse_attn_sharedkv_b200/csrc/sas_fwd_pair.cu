// Sparse shared-KV attention forward for calls with 65..128 query heads on
// B200 (sm_100a): a cluster of two CTAs on two SMs shares every key tile and
// issues cta_group::2 MMAs (M = 128 heads, 64 per CTA).
//
// Per pair tile of 64 key slots (window keys then compressed keys, golden.py
// tile order), CTA r gathers the rows of slots 32 r .. 32 r + 31 only:
//
//   QK   S = Q K^T, 36 x tcgen05.mma.cta_group::2 M128 N64 K16: A = the
//        CTA's 64 heads of Q, B = the CTA's 32 key rows (N split between
//        the CTAs), D = S[64 heads x 64 keys] in each CTA's TMEM
//   PV   O += P V, 8 x M128 N256 K16: A = the CTA's P[64 heads x 64 keys],
//        B = V[64 keys x 128 columns] of each CTA (N split), so each CTA
//        needs every key of the tile for its half of d_v.  A mover thread
//        copies the CTA's own rows of its d_v half into its V buffer and the
//        peer's d_v half of the same rows into the peer's V buffer with bulk
//        shared-memory copies (distributed shared memory), 16 KB each way
//        per tile, completing on the destination CTA's barrier.
//
// Because a CTA holds only 32 of the tile's key rows, the gathered rows
// (36 KB per region) and the V buffers (32 KB, double-buffered) are
// separate: a gather region is free again once QK has read it and the
// movers have copied it out, so the next gathers start while the tile's
// softmax and PV are still running, and each SM issues half the gather
// operations of a 64-head CTA walking the same tiles.
//
// Warp roles in each CTA (512 threads):
//   0-3    softmax: S from TMEM, mask, online softmax seeded by the sink
//          (golden.py:156-196) in the exp2 domain, P into shared memory,
//          lazy O rescale in TMEM, statistics of each (row, piece)
//   4-7    producers: slot -> (cache, position) -> block table -> row
//          (golden.py:28-66, kernel.py:2606-2751), validity of all 64 slots,
//          TMA tile::gather4 / 8-row boxes of the CTA's 32 rows
//   8      CTA 0: MMA issuer for the pair; CTA 1: relay that forwards its
//          readiness barriers to CTA 0 (remote mbarrier arrivals)
//   9      Q loader (TMA, next row's Q prefetched into L2)
//   10     mover: V rows into both CTAs' V buffers (bulk copies)
//   12-15  epilogue: O / l -> out (or fp32 split partials) and the LSE
//
// The leader's tcgen05.commit arrives on the barriers of both CTAs
// (.multicast::cluster).  Every wait is bounded: on timeout the thread
// records an error, raises its CTA's abort flag and leaves its loop; both
// CTAs then meet at the final cluster barrier.  No TMA load here uses
// .multicast::cluster, and no load reads another GPU's memory.

#include "sas_dev.cuh"

namespace sas {
namespace {

constexpr int kPThreads = 512;
constexpr int kPSoftmaxThreads = 128;
constexpr int kPProducerWarp0 = 4;
constexpr int kPMmaWarp = 8;
constexpr int kPQWarp = 9;
constexpr int kPMoverWarp0 = 10;
constexpr int kPPvWarp = 11;       // CTA 0: PV issuer; CTA 1: second relay thread
constexpr int kPEpiWarp0 = 12;
constexpr int kPEpiThreads = 128;
constexpr int kPProducerThreads = 128;

constexpr int kOwnKeys = 32;                      // key rows a CTA gathers per tile
constexpr int kSlotBytes = kOwnKeys * 128;        // one 64-column chunk of 32 rows
constexpr int kRegionBytes = 9 * kSlotBytes;      // 36 KB
constexpr int kNumRegions = 2;
constexpr int kQChunkBytes = kHeadsPerCta * 128;  // 64 heads x 64 columns
constexpr int kVChunkBytes = kTileKeys * 128;     // 64 keys x 64 columns
constexpr int kPSmemQ = 0;
constexpr int kPSmemR0 = kPSmemQ + 9 * kQChunkBytes;
constexpr int kPSmemV = kPSmemR0 + kNumRegions * kRegionBytes;
constexpr int kVBufBytes = 4 * kVChunkBytes;       // 32 KB
constexpr int kPSmemP = kPSmemV + 2 * kVBufBytes;
constexpr int kPSmemTiles = kPSmemP + kHeadsPerCta * 128;
constexpr int kPSmemDynamic = kPSmemTiles + 1024;  // + runtime 1 KB alignment slack
constexpr int kValidRing = 4;                      // tiles whose valid bits are in flight

constexpr uint32_t kPTmemCols = 512;
constexpr uint32_t kPTmemO = 0;
constexpr uint32_t kPTmemS = 256;

// Dims chunk (64 columns) held by chunk j of CTA r's V buffer: CTA r supplies
// d_v columns 256 hv + 128 r .. + 127 of the N = 256 PV MMA number hv.
__host__ __device__ constexpr int v_chunk_dims(int r, int j) { return 4 * (j >> 1) + 2 * r + (j & 1); }

struct PairCtl {
  uint64_t kv_full[kNumRegions][3];  // the CTA's rows of a region landed, per chunk group
  uint64_t kv_free[kNumRegions];     // QK read the region (commit) and the movers copied it
  uint64_t vfull[kValidRing];        // valid bits of tile t in valid[t % 4]
  uint64_t vfree[kValidRing];        // the softmax has read them
  // V buffer b of this CTA holds tile 2 k + b (phase k): the CTA's mover
  // arms 32 KB, its own and the peer's bulk copies complete 16 KB each.
  uint64_t vin[2];
  uint64_t pv_done[2];               // PV(2 k + b) complete (commit): V buffer b free, O updated
  uint64_t p_full;                   // P(t) written
  uint64_t q_full, q_empty;
  uint64_t s_full[2], s_empty[2];
  uint64_t o_full, o_free, drain;
  uint64_t xbar[2];
  uint64_t fin_full[2], fin_free[2];
  // Leader only: CTA 1's readiness, arrived remotely by CTA 1's roles:
  // its rows of a region (mover, once all three chunk groups are in), its V
  // buffer (mover), P and the S / O releases (one lane per softmax /
  // epilogue warp), Q (Q loader).
  uint64_t m_kv_full[kNumRegions];
  uint64_t m_vin[2], m_p_full, m_q_full, m_s_empty[2], m_o_free;
  uint32_t tmem_base;
  volatile int abort;
  uint16_t valid[kValidRing][4];
  float red[2][2][kHeadsPerCta];
  float fin_m[2][kHeadsPerCta];
  float fin_l[2][2][kHeadsPerCta];
  alignas(128) uint8_t epi[4][32 * 32];
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t peer_addr(uint32_t a, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}

// A mirror barrier of the leader (arrived by CTA 1's relay), polled relaxed:
// it only orders the leader's MMA issue after CTA 1's shared memory was
// complete (see arrive_remote).
__device__ __forceinline__ bool try_wait_mirror(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.relaxed.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on a mirror barrier; on timeout records the error and raises
// the CTA abort flag.
__device__ __forceinline__ bool wait_mirror(PairCtl* ctl, uint64_t* bar, uint32_t parity,
                                            int* err, int site) {
  const uint32_t a = smem_addr(bar);
  if (try_wait_mirror(a, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (try_wait_mirror(a, parity)) return true;
    if (ctl->abort) return false;
    if (clock64() - t0 > kWaitCycles) {
      record_error(err, SAS_ERR_DEVICE, site, (int)parity);
      ctl->abort = 1;
      return false;
    }
  }
}

// Bulk copy of `bytes` from this CTA's shared memory to shared memory of a
// CTA of the cluster (dst, bar: shared::cluster addresses in the same CTA),
// completing `bytes` on that CTA's barrier.
__device__ __forceinline__ void bulk_s2s(uint32_t dst, uint32_t src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, "
      "[%3];" ::"r"(dst),
      "r"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// Arrival on a barrier of the other CTA of the pair (shared::cluster
// address).  Relaxed: every forwarded phase guards shared memory that was
// complete before the local phase it mirrors completed (TMA and bulk-copy
// transactions, or generic stores fenced to the async proxy before their
// arrival), so the arrival only signals; a release here would wait for the
// issuing thread's outstanding memory operations on every forward.
__device__ __forceinline__ void arrive_remote(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar)
               : "memory");
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// D[tmem] (+)= A[smem] * B[smem] over the CTA pair (M = 128: 64 rows per CTA;
// B split by N between the CTAs; D in each CTA's TMEM, columns [0, N/2) on
// lanes 0-63 and [N/2, N) on lanes 64-127).  Issued by the leader CTA only.
__device__ __forceinline__ void mma2(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                     uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on the barrier at the same offset in both CTAs when every MMA
// the leader issued so far has completed.
__device__ __forceinline__ void commit_both(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], %1;" ::"r"(bar),
      "h"((uint16_t)3)
      : "memory");
}

// Validity of slot `slot` of row rv (golden.py:28-66): window slots always,
// compressed slots unless a -1 precedes them in the scan, the index is
// negative or at / past the causal threshold.
__device__ __forceinline__ bool slot_valid(const Row& rv, int thr, int slot, const int* idx_row,
                                           bool blocked) {
  if (slot < rv.window) return true;
  if (slot >= rv.window + rv.cmp) return false;
  if (idx_row == nullptr) return true;
  const int pos = __ldg(idx_row + (slot - rv.window));
  return !blocked && pos >= 0 && pos < thr;
}

// Resolution of one tile for producer warp pw of CTA rank: the -1 scan of
// the whole tile (each warp scans all 64 slots, so the stop prefix needs no
// exchange), the valid bits of slots 16 pw .. 16 pw + 15 (lanes 0-15) and
// the source of the warp's gathered slots 32 rank + 8 pw + (lane & 7).
struct TileRes {
  SlotSrc src;
  uint32_t valid16;
};

__device__ __forceinline__ TileRes resolve_pair_tile(const FwdArgs& a, const Row& rv,
                                                     const QueryKeys& qk, const int* idx_row,
                                                     int j, int pw, int rank, int lane,
                                                     bool* stopped, int* err) {
  uint64_t m1mask = 0;
  if (idx_row != nullptr) {
    const int ca = j * kTileKeys + lane - rv.window;
    const int cb = ca + 32;
    const bool ma = (ca >= 0 && ca < qk.cmp) && (__ldg(idx_row + ca) == -1);
    const bool mb = (cb >= 0 && cb < qk.cmp) && (__ldg(idx_row + cb) == -1);
    m1mask = (uint64_t)__ballot_sync(0xffffffffu, ma) |
             ((uint64_t)__ballot_sync(0xffffffffu, mb) << 32);
  }
  const int kv = pw * 16 + (lane & 15);
  const bool bv = *stopped || ((m1mask & ((1ull << kv) - 1ull)) != 0);
  const bool v = slot_valid(rv, qk.thr, j * kTileKeys + kv, idx_row, bv);
  const int ko = kOwnKeys * rank + 8 * pw + (lane & 7);
  const bool bo = *stopped || ((m1mask & ((1ull << ko) - 1ull)) != 0);
  TileRes t;
  t.src = resolve_slot(a, rv, qk, j * kTileKeys + ko, idx_row, bo, err);
  t.valid16 = __ballot_sync(0xffffffffu, v) & 0xffffu;
  if (m1mask != 0) *stopped = true;
  return t;
}

// cp.async of rows k = lbase .. lbase + count - 1 of this warp's 8 (smem row
// key0 + k of each 32-row slot, source (r, p) of lane k); rows without a
// source are zero-filled.
__device__ __forceinline__ void lsu_rows8(const FwdArgs& a, uint32_t region, int key0, int lbase,
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
      cp_async_16(region + (gi >> 3) * kSlotBytes + swz(key, gi & 7), src + gi * 16,
                  has ? 16u : 0u);
  }
}

__device__ __forceinline__ uint32_t group_chunks3(int cg, int nchunks) {
  return (uint32_t)max(0, min(3 * cg + 3, nchunks) - 3 * cg);
}

// The warp's 8 key rows of a tile into rows 8 pw .. 8 pw + 7 of every slot of
// the region: one 8-row TMA box per chunk when they are 8 consecutive rows of
// one cache, else tile::gather4 per 4-row group (cp.async for a group that
// mixes the two caches).  Rows without a source read an out-of-range row,
// which TMA fills with zeros.  Lane 0 arrives once on each chunk-group
// barrier, arming the TMA bytes.
__device__ __forceinline__ void load_own_rows(const FwdArgs& a, const SlotSrc& s, int nchunks,
                                              uint32_t region, const uint32_t (&bar)[3], int pw,
                                              int lane, uint32_t row_bytes, int gran,
                                              const CUtensorMap* tm_ori, const CUtensorMap* tm_cmp,
                                              const CUtensorMap* tm_ori8,
                                              const CUtensorMap* tm_cmp8) {
  const int row0 = __shfl_sync(0xffffffffu, s.row, 0);
  const int pool0 = __shfl_sync(0xffffffffu, s.pool, 0);
  const bool run8 = __all_sync(0xffffffffu, pool0 >= 0 && s.pool == pool0 && s.row >= 0 &&
                                                s.row == row0 + (lane & 7));
  const int key0 = 8 * pw;
  if (run8) {
    if (lane == 0) {
#pragma unroll
      for (int cg = 0; cg < 3; ++cg)
        mbar_expect_tx(bar[cg], 8u * 128u * group_chunks3(cg, nchunks));
      const CUtensorMap* m = (pool0 == 1) ? tm_cmp8 : tm_ori8;
      const uint32_t dst = region + (uint32_t)key0 * 128u;
      for (int c = 0; c < nchunks; ++c)
        tma_load_2d(dst + c * kSlotBytes, m, c * 64, row0, bar[c / 3]);
    }
    return;
  }
  const int g = lane & 1;  // lanes 0, 1: groups of rows 0-3 and 4-7
  int row[4], pool[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    row[i] = __shfl_sync(0xffffffffu, s.row, 4 * g + i);
    pool[i] = __shfl_sync(0xffffffffu, s.pool, 4 * g + i);
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
  const uint32_t mixed_mask = __ballot_sync(0xffffffffu, mixed) & 0x3u;
  if (lane == 0) {
    const uint32_t groups = (uint32_t)(2 - __popc(mixed_mask));
#pragma unroll
    for (int cg = 0; cg < 3; ++cg)
      mbar_expect_tx(bar[cg], groups * 4u * 128u * group_chunks3(cg, nchunks));
  }
  __syncwarp();
  if (lane < 2 && !mixed) {
    const CUtensorMap* m = (P == 1) ? tm_cmp : tm_ori;
    const int sentinel = (P == 1) ? a.cmp_rows : a.ori_rows;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (pool[i] < 0 || row[i] < 0) row[i] = sentinel;
    const uint32_t dst = region + (uint32_t)(key0 + 4 * lane) * 128u;
    for (int c = 0; c < nchunks; ++c)
      tma_gather4(dst + c * kSlotBytes, m, c * 64, row[0], row[1], row[2], row[3], bar[c / 3]);
  }
  for (uint32_t mm = mixed_mask; mm != 0u; mm &= mm - 1u)
    lsu_rows8(a, region, key0, 4 * (__ffs(mm) - 1), 4, s.row, s.pool, lane, row_bytes, gran);
}

// L2 prefetch of this warp's 8 gathered rows of a later tile (lane l: row
// l % 8, 128-byte lines 3 (l / 8) .. 3 (l / 8) + 2 of it), so that the tile's
// TMA loads, issued once its region is free, read L2 instead of HBM.
__device__ __forceinline__ void prefetch_own_rows(const FwdArgs& a, const SlotSrc& src, int lane,
                                                  uint32_t row_bytes) {
  if (src.pool < 0 || src.row < 0) return;
  const char* base = reinterpret_cast<const char*>(src.pool == 1 ? a.cmp_kv : a.ori_kv) +
                     (size_t)src.row * row_bytes;
  const int lines = (int)(row_bytes >> 7);
  const int l0 = 3 * (lane >> 3);
  for (int l = l0; l < l0 + 3 && l < lines; ++l)
    asm volatile("prefetch.global.L2 [%0];" ::"l"(base + l * 128) : "memory");
}

// Chunk group cg of S = Q K^T over the pair: chunk c of Q (64 heads) against
// chunk slot c of the CTA's 32 key rows, into partial c % kQkPartials.
template <int kChunks>
__device__ __forceinline__ void issue_qk_pair(uint32_t d, uint32_t sQ, uint32_t region,
                                              uint32_t idesc, int cg) {
  const uint64_t dq = smem_desc(sQ, 16, 1024);
  const uint64_t dk = smem_desc(region, 16, 1024);
  const int c0 = 3 * cg;
  const int nc = min(3, kChunks - c0);
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      if (i < nc) {
        const int c = c0 + i;
        mma2(d + 32u * (c % kQkPartials), dq + (uint64_t)((c * kQChunkBytes + ks * 32) >> 4),
             dk + (uint64_t)((c * kSlotBytes + ks * 32) >> 4), idesc,
             (c < kQkPartials && ks == 0) ? 0u : 1u);
      }
    }
  }
}

// O (+)= P V over the pair: P (64 heads x 64 keys) of each CTA, V chunks
// 2 hv, 2 hv + 1 of each CTA's V buffer (MN-major, 64 rows).
__device__ __forceinline__ void issue_pv_pair(uint32_t o, uint32_t sP, uint32_t sV,
                                              uint32_t idesc, bool first) {
  const uint64_t dp = smem_desc(sP, 16, 1024);
  const uint64_t dv = smem_desc(sV, kVChunkBytes, 1024);
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
    for (int hv = 0; hv < 2; ++hv)
      mma2(o + 128u * hv, dp + (uint64_t)((ks * 32) >> 4),
           dv + (uint64_t)((2 * hv * kVChunkBytes + ks * 2048) >> 4), idesc,
           (first && ks == 0) ? 0u : 1u);
  }
}

// Rows with key tiles and total tiles of a worker span.
__device__ __forceinline__ void span_counts(const int* rows, const Span& sp, int* nrows,
                                            int* ntiles) {
  int nr = 0, nt = 0;
  for (int r = sp.r0; sp.r0 >= 0 && r <= sp.r1; ++r) {
    const Row rv = load_row(rows, r);
    const int tiles = row_tiles(rv);
    const int ja = (r == sp.r0) ? sp.t0 : 0;
    const int jb = (r == sp.r1) ? sp.t1 : (tiles > 0 ? tiles : 1);
    if (tiles > 0 && ja < jb) {
      ++nr;
      nt += jb - ja;
    }
  }
  *nrows = nr;
  *ntiles = nt;
}

template <bool kBf16, int kChunks, bool kTrace>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPThreads, 1)
    sas_pair_kernel(const FwdArgs args, const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_ori,
                    const __grid_constant__ CUtensorMap tm_cmp,
                    const __grid_constant__ CUtensorMap tm_ori8,
                    const __grid_constant__ CUtensorMap tm_cmp8) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ PairCtl ctl;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = (int)cluster_rank();
  const bool leader = (rank == 0);
  const int worker = blockIdx.x >> 1;
  const int group = rank;
  const int* plan = args.plan;
  const int* rows = plan + plan[H_ROWS_OFF];
  constexpr int nchunks = kChunks;
  int* err = args.err;
  // Diagnostic clock trace (trace instances only) of CTA 0 of worker
  // args.trace_cta: region 0 producer warp 4 per tile (3 t: before the
  // region wait, 3 t + 1: region free, 3 t + 2: loads issued); region 1 the
  // MMA issuer (4 t: QK group 0 issued, 4 t + 1: QK(t) complete in issue,
  // 4 t + 2: PV(t) issued; from 4096, 4 t + k: first time P own / P peer /
  // V own / V peer were seen ready); region 2 softmax thread 0 (4 t: S(t)
  // in, 4 t + 1: maximum exchanged, 4 t + 2: PV(t - 1) done, 4 t + 3: P(t)
  // released); region 3 mover warp 10 (4 t: start, 4 t + 1: rows in,
  // 4 t + 2: V buffer free, 4 t + 3: done).
  long long* tr = (kTrace && worker == args.trace_cta && rank == 0) ? args.trace : nullptr;

  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t sQ = base + kPSmemQ;
  const uint32_t sR0 = base + kPSmemR0;
  const uint32_t sV = base + kPSmemV;
  const uint32_t sP = base + kPSmemP;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumRegions; ++i) {
      for (int g = 0; g < 3; ++g) {
        // one arrival per producer warp (lane 0, arming the TMA bytes) and
        // one cp.async completion arrival per producer lane
        mbar_init(smem_addr(&ctl.kv_full[i][g]), 4 + kPProducerThreads);
      }
      // QK of the tile has read it (leader's commit) and every copy out of
      // it has landed (leader's arrival once both V buffers are complete)
      mbar_init(smem_addr(&ctl.kv_free[i]), 2);
      mbar_init(smem_addr(&ctl.m_kv_full[i]), 1);
    }
    for (int i = 0; i < kValidRing; ++i) {
      mbar_init(smem_addr(&ctl.vfull[i]), 4);
      mbar_init(smem_addr(&ctl.vfree[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_addr(&ctl.vin[i]), 1);
      mbar_init(smem_addr(&ctl.m_vin[i]), 1);
      mbar_init(smem_addr(&ctl.pv_done[i]), 1);
    }
    mbar_init(smem_addr(&ctl.p_full), kPSoftmaxThreads);
    mbar_init(smem_addr(&ctl.q_full), 1);
    mbar_init(smem_addr(&ctl.q_empty), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_addr(&ctl.s_full[i]), 1);
      mbar_init(smem_addr(&ctl.s_empty[i]), kPSoftmaxThreads);
      mbar_init(smem_addr(&ctl.xbar[i]), kPSoftmaxThreads);
      mbar_init(smem_addr(&ctl.fin_full[i]), kPSoftmaxThreads);
      mbar_init(smem_addr(&ctl.fin_free[i]), kPEpiThreads);
      mbar_init(smem_addr(&ctl.m_s_empty[i]), 4);
    }
    mbar_init(smem_addr(&ctl.o_full), 1);
    mbar_init(smem_addr(&ctl.o_free), kPEpiThreads);
    mbar_init(smem_addr(&ctl.drain), 2);  // one commit from each MMA issuer
    mbar_init(smem_addr(&ctl.m_p_full), 4);
    mbar_init(smem_addr(&ctl.m_q_full), 1);
    mbar_init(smem_addr(&ctl.m_o_free), 4);
    ctl.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kPMmaWarp) {
    // Both CTAs allocate from the same warp: the pair's columns are
    // allocated together (cta_group::2).
    asm volatile(
        "tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
            smem_addr(&ctl.tmem_base)),
        "r"(kPTmemCols)
        : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers are initialised before any remote arrival
  tc_fence_after();
  const uint32_t tmem = ctl.tmem_base;

  const Span span =
      (worker < plan[H_NUM_WORKERS]) ? load_span(plan, worker) : Span{-1, 0, -1, 0, 0};

  if (warp >= kPProducerWarp0 && warp < kPProducerWarp0 + 4) {
    // ======================= producers =======================
    const int pw = warp - kPProducerWarp0;
    const int D = args.head_dim;
    const uint32_t row_bytes = (uint32_t)D * 2u;
    const int gran = D >> 3;
    uint32_t free_par = (1u << kNumRegions) - 1u;  // bit = region (first use passes)
    int t = 0;                                     // tiles of the span so far
    bool ok = true;
    RowStream rs(rows, span.r0, span.r1);
    for (int r = span.r0; ok && span.r0 >= 0 && r <= span.r1; ++r) {
      const Row rv = rs.take(r);
      const int tiles = row_tiles(rv);
      const int ja = (r == span.r0) ? span.t0 : 0;
      const int jb = (r == span.r1) ? span.t1 : (tiles > 0 ? tiles : 1);
      if (tiles == 0 || ja >= jb) continue;
      QueryKeys qk;
      qk.window = rv.window;
      qk.win_lo = rv.win_lo;
      qk.cmp = rv.cmp;
      qk.thr = rv.thr;
      qk.cmp_len = 0;
      const int* idx_row = (args.scenario == SAS_SCENARIO_SCFA)
                               ? args.cmp_indices + (size_t)rv.token * args.topk
                               : nullptr;
      bool stopped = false;
      if (idx_row != nullptr && ja > 0) {
        // a -1 before this piece stops the scan: 512 indices per step
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
      TileRes nxt = resolve_pair_tile(args, rv, qk, idx_row, ja, pw, rank, lane, &stopped, err);
      for (int j = ja; j < jb; ++j, ++t) {
        const TileRes cur = nxt;
        if (j + 1 < jb) {
          nxt = resolve_pair_tile(args, rv, qk, idx_row, j + 1, pw, rank, lane, &stopped, err);
          prefetch_own_rows(args, nxt.src, lane, row_bytes);
        }
        if (args.slot_dump != nullptr && lane < 8)
          dump_slot(args, rv.token, j * kTileKeys + kOwnKeys * rank + 8 * pw + lane, cur.src);
        const int region = t % kNumRegions;
        const int vr = t % kValidRing;
        if (pw == 0 && lane == 0) trace(tr, 0, 3 * t);
        // valid bits: the softmax has read tile t - 4's from this entry
        if (t >= kValidRing &&
            !__all_sync(0xffffffffu, wait_bar(&ctl, &ctl.vfree[vr],
                                              (uint32_t)(((t / kValidRing) - 1) & 1), err, 70))) {
          ok = false;
          break;
        }
        if (lane == 0) {
          ctl.valid[vr][pw] = (uint16_t)cur.valid16;
          mbar_arrive(smem_addr(&ctl.vfull[vr]));
        }
        if (!__all_sync(0xffffffffu, wait_bar(&ctl, &ctl.kv_free[region],
                                             (free_par >> region) & 1u, err, 71))) {
          ok = false;
          break;
        }
        free_par ^= 1u << region;
        if (pw == 0 && lane == 0) trace(tr, 0, 3 * t + 1);
        uint32_t bar[3];
#pragma unroll
        for (int cg = 0; cg < 3; ++cg) bar[cg] = smem_addr(&ctl.kv_full[region][cg]);
        load_own_rows(args, cur.src, nchunks, sR0 + region * kRegionBytes, bar, pw, lane,
                      row_bytes, gran, &tm_ori, &tm_cmp, &tm_ori8, &tm_cmp8);
#pragma unroll
        for (int cg = 0; cg < 3; ++cg) cp_async_arrive_noinc(bar[cg]);
        if (pw == 0 && lane == 0) trace(tr, 0, 3 * t + 2);
      }
    }
    cp_async_wait_all();
  } else if (warp == kPMoverWarp0) {
    // ======================= mover =======================
    // Per tile t, once the CTA's 32 rows are in and PV(t - 2) has released
    // V buffer t % 2 of both CTAs: bulk copies (4 KB, one 64-column chunk of
    // the 32 rows each) of this CTA's d_v chunks into its own V buffer and of
    // the peer's d_v chunks into the peer's V buffer (rows 32 rank .. 32 rank
    // + 31 of each V chunk).  Each copy completes on the V barrier of the CTA
    // it writes; this CTA arms its own barrier with both halves' bytes.
    if (lane == 0) {
      const int peer = rank ^ 1;
      const uint32_t sV_peer = peer_addr(sV, (uint32_t)peer);
      int nrows = 0, ntiles = 0;
      span_counts(rows, span, &nrows, &ntiles);
      for (int t = 0; t < ntiles; ++t) {
        const int region = t % kNumRegions;
        const uint32_t kpar = (uint32_t)((t / kNumRegions) & 1);
        trace(tr, 3, 4 * t);
        bool w = true;
#pragma unroll
        for (int cg = 0; cg < 3; ++cg)
          w = w && wait_bar(&ctl, &ctl.kv_full[region][cg], kpar, err, 72);
        trace(tr, 3, 4 * t + 1);
        if (w && !leader)  // CTA 1's rows of the tile are in: tell the leader
          arrive_remote(peer_addr(smem_addr(&ctl.m_kv_full[region]), 0u));
        if (w && t >= 2)
          w = wait_bar(&ctl, &ctl.pv_done[t & 1], (uint32_t)(((t >> 1) - 1) & 1), err, 73);
        if (!w) break;
        trace(tr, 3, 4 * t + 2);
        const int vb = t & 1;
        const uint32_t reg = sR0 + region * kRegionBytes;
        const uint32_t dst_off = (uint32_t)(vb * kVBufBytes) + (uint32_t)(kOwnKeys * rank) * 128u;
        const uint32_t own_bar = smem_addr(&ctl.vin[vb]);
        const uint32_t peer_bar = peer_addr(own_bar, (uint32_t)peer);
        mbar_expect_tx(own_bar, 2u * 4u * (uint32_t)kSlotBytes);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t joff = dst_off + (uint32_t)(j * kVChunkBytes);
          bulk_s2s(sV + joff, reg + v_chunk_dims(rank, j) * kSlotBytes, kSlotBytes, own_bar);
          bulk_s2s(sV_peer + joff, reg + v_chunk_dims(peer, j) * kSlotBytes, kSlotBytes,
                   peer_bar);
        }
        trace(tr, 3, 4 * t + 3);
        const uint32_t vp = (uint32_t)((t >> 1) & 1);
        if (leader) {
          // Once both CTAs' V buffers hold the tile, every copy out of its
          // gather regions has landed: release them (QK's commit is their
          // other arrival).
          if (!wait_bar(&ctl, &ctl.vin[vb], vp, err, 79) ||
              !wait_mirror(&ctl, &ctl.m_vin[vb], vp, err, 79))
            break;
          const uint32_t fb = smem_addr(&ctl.kv_free[region]);
          mbar_arrive(fb);
          arrive_remote(peer_addr(fb, 1u));
        } else {
          // CTA 1's V buffer holds the tile (its own and the leader's copies)
          if (!wait_bar(&ctl, &ctl.vin[vb], vp, err, 79)) break;
          arrive_remote(peer_addr(smem_addr(&ctl.m_vin[vb]), 0u));
        }
      }
    }
    __syncwarp();
  } else if (warp == kPQWarp) {
    // ======================= Q loader =======================
    if (lane == 0) {
      const uint32_t q_bytes = (uint32_t)kHeadsPerCta * (uint32_t)args.head_dim * 2u;
      uint32_t q_empty_par = 1u;
      int q_loads = 0;
      int next = span.r0;
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
        for (next = max(next, r + 1); next <= span.r1; ++next) {
          int nq;
          if (qrow_of(next, &nq)) {
            for (int c = 0; c < nchunks; ++c) tma_prefetch_2d(&tm_q, c * 64, nq);
            ++next;
            break;
          }
        }
        if (!wait_bar(&ctl, &ctl.q_empty, q_empty_par, err, 74)) break;
        q_empty_par ^= 1u;
        mbar_expect_tx(smem_addr(&ctl.q_full), q_bytes);
        for (int c = 0; c < nchunks; ++c)
          tma_load_2d(sQ + c * kQChunkBytes, &tm_q, c * 64, qrow, smem_addr(&ctl.q_full));
        if (!leader) {
          // CTA 1's Q of the row is in: tell the leader
          if (!wait_bar(&ctl, &ctl.q_full, (uint32_t)(q_loads & 1), err, 74)) break;
          arrive_remote(peer_addr(smem_addr(&ctl.m_q_full), 0u));
        }
        ++q_loads;
      }
    }
    __syncwarp();
  } else if (warp == kPMmaWarp || warp == kPPvWarp) {
    const bool qk_role = (warp == kPMmaWarp);
    if (leader) {
      // ================= MMA issuers of the pair (CTA 0) =================
      // One thread issues the QKs, another the PVs; each waits (bounded) for
      // its inputs in both CTAs and issues in tile order.  The PV of tile t
      // follows its QK through P(t) (the softmax read S(t)); QK(t + 2) reuses
      // the S buffer of tile t after the softmax released it.
      if (lane == 0) {
        bool ok = true;
        if (qk_role) {
          const uint32_t idesc_qk = instr_desc(128, 64, kBf16, false, false);
          TileCursor qc(rows, span);
          int tq = 0, row_i = 0;
          while (ok && qc.valid) {
            const int sb = tq & 1;
            const int region = tq % kNumRegions;
            if (qc.first()) {
              const uint32_t qp = (uint32_t)(row_i & 1);
              ok = wait_bar(&ctl, &ctl.q_full, qp, err, 90) &&
                   wait_mirror(&ctl, &ctl.m_q_full, qp, err, 91);
            }
            if (ok && tq >= 2) {
              const uint32_t sp = (uint32_t)(((tq >> 1) - 1) & 1);
              ok = wait_bar(&ctl, &ctl.s_empty[sb], sp, err, 92) &&
                   wait_mirror(&ctl, &ctl.m_s_empty[sb], sp, err, 93);
            }
            const uint32_t kp = (uint32_t)((tq / kNumRegions) & 1);
            for (int g = 0; ok && g < 3; ++g) {
              ok = wait_bar(&ctl, &ctl.kv_full[region][g], kp, err, 94) &&
                   (g > 0 || wait_mirror(&ctl, &ctl.m_kv_full[region], kp, err, 95));
              if (!ok) break;
              tc_fence_after();
              if (g == 0) trace(tr, 1, 4 * tq);
              trace(tr, 3, 6144 + 8 * tq + 2 * g);
              issue_qk_pair<nchunks>(tmem + kPTmemS + 128u * sb, sQ,
                                     sR0 + region * kRegionBytes, idesc_qk, g);
              trace(tr, 3, 6145 + 8 * tq + 2 * g);
            }
            if (!ok) break;
            trace(tr, 1, 4 * tq + 1);
            commit_both(smem_addr(&ctl.s_full[sb]));
            commit_both(smem_addr(&ctl.kv_free[region]));
            if (qc.last()) {
              commit_both(smem_addr(&ctl.q_empty));
              ++row_i;
            }
            ++tq;
            qc.advance();
          }
        } else {
          const uint32_t idesc_pv = instr_desc(128, 256, kBf16, false, true);
          TileCursor pc(rows, span);
          int tp = 0, piece = 0;
          while (ok && pc.valid) {
            const int vb = tp & 1;
            const uint32_t vp = (uint32_t)((tp >> 1) & 1);
            const uint32_t pp = (uint32_t)(tp & 1);
            ok = wait_bar(&ctl, &ctl.vin[vb], vp, err, 96) &&
                 wait_mirror(&ctl, &ctl.m_vin[vb], vp, err, 97) &&
                 wait_bar(&ctl, &ctl.p_full, pp, err, 98) &&
                 wait_mirror(&ctl, &ctl.m_p_full, pp, err, 99);
            if (ok && pc.first() && piece > 0) {
              const uint32_t op = (uint32_t)((piece - 1) & 1);
              ok = wait_bar(&ctl, &ctl.o_free, op, err, 100) &&
                   wait_mirror(&ctl, &ctl.m_o_free, op, err, 101);
            }
            if (!ok) break;
            tc_fence_after();
            trace(tr, 1, 4 * tp + 2);
            issue_pv_pair(tmem + kPTmemO, sP, sV + vb * kVBufBytes, idesc_pv, pc.first());
            commit_both(smem_addr(&ctl.pv_done[vb]));
            if (pc.last()) {
              commit_both(smem_addr(&ctl.o_full));
              ++piece;
            }
            ++tp;
            pc.advance();
          }
        }
        // Drain (both issuers): completes in both CTAs once every MMA issued
        // above has finished, so neither CTA releases TMEM under an in-flight
        // MMA.
        commit_both(smem_addr(&ctl.drain));
        wait_bar(&ctl, &ctl.drain, 0u, err, 102);
      }
      __syncwarp();
    } else if (qk_role && lane == 0) {
      // CTA 1: the leader's last MMAs write this CTA's TMEM; wait for its
      // drain before the final cluster barrier and the release of TMEM.
      wait_bar(&ctl, &ctl.drain, 0u, err, 78);
    }
    __syncwarp();
  } else if (warp >= kPEpiWarp0) {
    // ======================= epilogue =======================
    const int ew = warp - kPEpiWarp0;
    const int half = ew >> 1;
    const int m0 = (ew & 1) * 32;
    const int m = m0 + lane;
    const int dv = args.head_dim_v;
    const uint32_t obase = tmem + ((uint32_t)(ew * 32) << 16) + kPTmemO;
    const int nlive = min(32, max(0, args.num_heads - (group * kHeadsPerCta + m0)));
    uint8_t* stg = ctl.epi[ew];
    int k = 0;
    RowStream rs(rows, span.r0, span.r1);
    for (int r = span.r0; span.r0 >= 0 && r <= span.r1; ++r) {
      const Row rv = rs.take(r);
      const int tiles = row_tiles(rv);
      const int ja = (r == span.r0) ? span.t0 : 0;
      const int jb = (r == span.r1) ? span.t1 : (tiles > 0 ? tiles : 1);
      if (tiles == 0 || ja >= jb) continue;
      const int fp = k & 1;
      if (!__all_sync(0xffffffffu, wait_bar(&ctl, &ctl.o_full, (uint32_t)(k & 1), err, 80)))
        break;
      if (!__all_sync(0xffffffffu,
                      wait_bar(&ctl, &ctl.fin_full[fp], (uint32_t)((k >> 1) & 1), err, 81)))
        break;
      tc_fence_after();
      const float m_run = ctl.fin_m[fp][m];
      const float l_tot = ctl.fin_l[fp][0][m] + ctl.fin_l[fp][1][m];
      mbar_arrive(smem_addr(&ctl.fin_free[fp]));
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
      __syncwarp();
      if (!leader && lane == 0) arrive_remote(peer_addr(smem_addr(&ctl.m_o_free), 0u));
      ++k;
    }
  } else if (warp < 4) {
    // ======================= softmax =======================
    const int L = threadIdx.x;
    const int m = L & (kHeadsPerCta - 1);
    const int half = L >> 6;
    const int head = group * kHeadsPerCta + m;
    const bool live = head < args.num_heads;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const float c2 = args.softmax_scale * kLog2e;
    const float sink = live ? __ldg(args.sinks + head) : -INFINITY;
    uint32_t xph = 0u;
    int xpar = 0, rows_done = 0;
    int t = 0;  // tiles of the span so far
    bool ok = true;
    const int dv = args.head_dim_v;
    for (int r = span.r0; ok && span.r0 >= 0 && r <= span.r1; ++r) {
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
      float m_run = first_piece ? sink * kLog2e : -INFINITY;
      float l_run = (first_piece && half == 0) ? 1.f : 0.f;
      for (int j = ja; j < jb; ++j, ++t) {
        const int sb = t & 1;
        const int vr = t % kValidRing;
        if (!__all_sync(0xffffffffu, wait_bar(&ctl, &ctl.s_full[sb], (uint32_t)((t >> 1) & 1),
                                             err, 82))) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (threadIdx.x == 0) trace(tr, 2, 4 * t);
        uint32_t sraw[32];
        {
          const uint32_t ts = tmem + lane_off + kPTmemS + 128u * sb;
          tmem_ld32(ts, sraw);
          tmem_wait_ld();
#pragma unroll
          for (int pp = 1; pp < kQkPartials; ++pp) {
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
        __syncwarp();
        if (!leader && lane == 0) arrive_remote(peer_addr(smem_addr(&ctl.m_s_empty[sb]), 0u));
        if (!__all_sync(0xffffffffu,
                        wait_bar(&ctl, &ctl.vfull[vr], (uint32_t)((t / kValidRing) & 1), err, 83))) {
          ok = false;
          break;
        }
        const uint32_t vb = (uint32_t)ctl.valid[vr][2 * half] |
                            ((uint32_t)ctl.valid[vr][2 * half + 1] << 16);
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
        const bool xw = wait_bar(&ctl, &ctl.xbar[xpar], (xph >> xpar) & 1u, err, 84);
        xph ^= 1u << xpar;
        if (!__all_sync(0xffffffffu, xw)) {
          ok = false;
          break;
        }
        // every softmax thread has read valid[vr]: the producers may reuse it
        if (threadIdx.x == 0) {
          mbar_arrive(smem_addr(&ctl.vfree[vr]));
          trace(tr, 2, 4 * t + 1);
        }
        mx = fmaxf(mx, ctl.red[xpar][half ^ 1][m]);
        xpar ^= 1;
        const float m_new = fmaxf(m_run, mx);
        const bool rescale = (m_new - m_run) > kRescaleThreshold;
        float alpha = 1.f;
        if (rescale) {
          alpha = exp2f(m_run - m_new);
          m_run = m_new;
          l_run *= alpha;
        }
        const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
        float lsum = 0.f;
        uint32_t pk[4][4];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int i = 8 * g + 2 * q;
            const float p0 = exp2f(x[i] - m_use);
            const float p1 = exp2f(x[i + 1] - m_use);
            lsum += p0 + p1;
            pk[g][q] = pack2<kBf16>(p0, p1);
          }
        }
        l_run += lsum;
        // The P buffer and O are free once PV of the previous tile is done.
        if (t > 0 && !__all_sync(0xffffffffu,
                                 wait_bar(&ctl, &ctl.pv_done[(t - 1) & 1],
                                         (uint32_t)(((t - 1) >> 1) & 1), err, 85))) {
          ok = false;
          break;
        }
        if (threadIdx.x == 0) trace(tr, 2, 4 * t + 2);
        uint8_t* prow = gbase + kPSmemP;
#pragma unroll
        for (int g = 0; g < 4; ++g)
          *reinterpret_cast<uint4*>(prow + swz(m, 4 * half + g)) =
              make_uint4(pk[g][0], pk[g][1], pk[g][2], pk[g][3]);
        fence_proxy_async();
        if (j > ja && __any_sync(0xffffffffu, rescale)) {
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < 16; ++c) {
            const uint32_t ta = tmem + lane_off + kPTmemO + 16u * c;
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
        mbar_arrive(smem_addr(&ctl.p_full));
        __syncwarp();
        if (!leader && lane == 0) arrive_remote(peer_addr(smem_addr(&ctl.m_p_full), 0u));
        if (threadIdx.x == 0) trace(tr, 2, 4 * t + 3);
      }
      if (!ok) break;
      const int fp = rows_done & 1;
      if (!__all_sync(0xffffffffu, wait_bar(&ctl, &ctl.fin_free[fp],
                                            (uint32_t)(((rows_done >> 1) & 1) ^ 1), err, 86)))
        break;
      if (half == 0) ctl.fin_m[fp][m] = m_run;
      ctl.fin_l[fp][half][m] = l_run;
      mbar_arrive(smem_addr(&ctl.fin_full[fp]));
      ++rows_done;
    }
  }

  tc_fence_before();
  __syncthreads();
  // Neither CTA leaves while the other may still read its shared memory or
  // arrive on its barriers.
  cluster_sync_all();
  if (warp == kPMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kPTmemCols)
                 : "memory");
  }
}

}  // namespace

// cuTensorMapEncodeTiled through the runtime's driver entry point.
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn_pair() {
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

static bool make_map_pair(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols,
                          uint32_t box_rows) {
  auto fn = encode_fn_pair();
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
static int launch_pair_one(const FwdArgs& args, int workers, cudaStream_t stream,
                           const CUtensorMap& tm_q, const CUtensorMap& tm_ori,
                           const CUtensorMap& tm_cmp, const CUtensorMap& tm_ori8,
                           const CUtensorMap& tm_cmp8) {
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(sas_pair_kernel<kBf16, kChunks, kTrace>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kPSmemDynamic) != cudaSuccess)
      return SAS_ERR_CUDA;
    configured = true;
  }
  sas_pair_kernel<kBf16, kChunks, kTrace><<<2 * workers, kPThreads, kPSmemDynamic, stream>>>(
      args, tm_q, tm_ori, tm_cmp, tm_ori8, tm_cmp8);
  return cudaGetLastError() == cudaSuccess ? SAS_OK : SAS_ERR_CUDA;
}

// The pair kernel for a plan with two head groups (65..128 heads); `workers`
// clusters of two CTAs.
int launch_fwd_pair(const FwdArgs& args, int workers, cudaStream_t stream) {
  const bool bf16 = args.dtype == SAS_DTYPE_BF16;
  if (args.head_dim != 576 && args.head_dim != 512) return SAS_ERR_UNSUPPORTED;
  alignas(64) CUtensorMap tm_q, tm_ori, tm_cmp, tm_ori8, tm_cmp8;
  const uint64_t D = (uint64_t)args.head_dim;
  if (!make_map_pair(&tm_q, args.q, (uint64_t)args.total_tokens * args.num_heads, D,
                     kHeadsPerCta))
    return SAS_ERR_CUDA;
  if (!make_map_pair(&tm_ori, args.ori_kv, (uint64_t)args.ori_rows, D, 1)) return SAS_ERR_CUDA;
  // A cache with fewer than 8 rows never takes the 8-row run path.
  const uint32_t ori_box = args.ori_rows < 8 ? (uint32_t)args.ori_rows : 8u;
  const uint32_t cmp_box = args.cmp_rows < 8 ? (uint32_t)args.cmp_rows : 8u;
  if (!make_map_pair(&tm_ori8, args.ori_kv, (uint64_t)args.ori_rows, D, ori_box))
    return SAS_ERR_CUDA;
  if (args.cmp_kv != nullptr && args.cmp_rows > 0) {
    if (!make_map_pair(&tm_cmp, args.cmp_kv, (uint64_t)args.cmp_rows, D, 1)) return SAS_ERR_CUDA;
    if (!make_map_pair(&tm_cmp8, args.cmp_kv, (uint64_t)args.cmp_rows, D, cmp_box))
      return SAS_ERR_CUDA;
  } else {
    tm_cmp = tm_ori;
    tm_cmp8 = tm_ori8;
  }
#define SAS_PAIR(B, C, T) \
  launch_pair_one<B, C, T>(args, workers, stream, tm_q, tm_ori, tm_cmp, tm_ori8, tm_cmp8)
  const bool t = args.trace != nullptr;
  if (args.head_dim == 576) {
    if (bf16) return t ? SAS_PAIR(true, 9, true) : SAS_PAIR(true, 9, false);
    return t ? SAS_PAIR(false, 9, true) : SAS_PAIR(false, 9, false);
  }
  if (bf16) return t ? SAS_PAIR(true, 8, true) : SAS_PAIR(true, 8, false);
  return t ? SAS_PAIR(false, 8, true) : SAS_PAIR(false, 8, false);
#undef SAS_PAIR
}

}  // namespace sas
