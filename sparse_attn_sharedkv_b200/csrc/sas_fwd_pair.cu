// Sparse shared-KV attention forward for calls with 65..128 query heads on
// B200 (sm_100a): a cluster of two CTAs on two SMs walks the worker's key
// slots in pair tiles of 128 and issues cta_group::2 MMAs (M = 128 heads,
// 64 per CTA; N = 128 keys, 64 gathered by each CTA).
//
// Per pair tile (slots 128 i .. 128 i + 127 of the worker's piece, golden.py
// tile order), CTA r gathers the rows of slots 64 r .. 64 r + 63 into a
// stage of nine 64-column chunk slots (64 rows x 128 B each):
//
//   QK   S = Q K^T, 36 x tcgen05.mma.cta_group::2 M128 N128 K16: A = the
//        CTA's 64 heads of Q, B = the CTA's 64 key rows (N split between the
//        CTAs), D = S[64 heads x 128 keys] in each CTA's TMEM (keys 0-63 on
//        lanes 0-63, keys 64-127 on lanes 64-127)
//   PV   O += P V, 16 x M128 N256 K16: A = the CTA's P[64 heads x 64 keys]
//        of one key half, B = V[64 keys x 128 d_v columns] of each CTA (N
//        split), so each CTA needs its d_v columns of all 128 keys.
//
// A CTA's d_v columns of the peer's 64 keys are gathered a second time from
// L2 once QK has read the stage, into the chunk slots of its own keys that
// only the peer's columns use (CTA 0: dims chunks 0, 1, 4, 5 of CTA 1's keys
// into slots 2, 3, 6, 7; CTA 1: dims chunks 2, 3, 6, 7 of CTA 0's keys into
// slots 0, 1, 4, 5), so both CTAs read V in place at the same shared-memory
// offsets and no key row crosses between the SMs.  Per SM and key this is
// 104 KB of gathered rows per 128 keys (72 KB + 32 KB) against 144 KB for
// one CTA per 64-head group, at twice the keys per QK instruction.
//
// Shared memory per CTA (227 KB, 1 KB aligned): Q 72 KB | two stages of
// 72 KB | P of key half 1 (8 KB; P of key half 0 goes into the rope slot 8
// of the tile's stage, which QK has read) | control.
//
// Every TMA load of both CTAs completes its bytes on the leader's barrier
// (.cta_group::2 loads, the barrier addressed in CTA 0), and each producer
// warp (per chunk group) and V warp (per tile) of either CTA arrives there
// once with the bytes it issued, so the leader's MMA issuers wait on local
// barriers only.  The
// leader's tcgen05.commit arrives on the barriers of both CTAs
// (.multicast::cluster).  CTA 1's softmax and epilogue warps signal P, the
// S release and the O release with relaxed remote arrivals on mirror
// barriers of the leader (each guards shared memory or TMEM already fenced
// before the arrival).
//
// Warp roles in each CTA (512 threads):
//   0-3    softmax: S from TMEM (thread: one head, one key half of 64 keys),
//          mask, maximum exchanged between warps w and w + 2 (the two key
//          halves of the same heads), online softmax seeded by the sink
//          (golden.py:156-196) in the exp2 domain, P into shared memory, lazy
//          O rescale in TMEM, statistics of each (row, piece)
//   4-7    producers: slot -> (cache, position) -> block table -> row
//          (golden.py:28-66, kernel.py:2606-2751), validity of the tile's
//          128 slots, TMA of the CTA's 64 rows (16-row boxes or
//          tile::gather4; cp.async for a 4-row group mixing the two caches);
//          the sources of the peer's rows go to the V warps
//   8      CTA 0: QK issuer; TMEM allocation in both CTAs
//   9      Q loader (TMA, next row's Q prefetched into L2)
//   10     CTA 0: PV issuer
//   12-15  V gather (the CTA's d_v columns of the peer's rows, once QK has
//          read the stage) and epilogue: O / l -> out (or fp32 split
//          partials) and the LSE
//
// Every wait is bounded: on timeout the thread records an error, raises its
// CTA's abort flag and leaves its loop; both CTAs then meet at the final
// cluster barrier.  No TMA load here uses .multicast::cluster, and no load
// reads another GPU's memory.

#include "sas_dev.cuh"

namespace sas {
namespace {

constexpr int kPThreads = 512;
constexpr int kPSoftmaxThreads = 128;
constexpr int kPProducerWarp0 = 4;
constexpr int kPQkWarp = 8;
constexpr int kPQWarp = 9;
constexpr int kPPvWarp = 10;
constexpr int kPEpiWarp0 = 12;
constexpr int kPEpiThreads = 128;

constexpr int kPairKeys = 128;                    // key slots per pair tile
constexpr int kOwnRows = kPairKeys / 2;           // key rows a CTA gathers per tile
constexpr int kSlotBytes = kOwnRows * 128;        // one 64-column chunk of 64 rows
constexpr int kStageBytes = 9 * kSlotBytes;       // 72 KB
constexpr int kQChunkBytes = kHeadsPerCta * 128;  // 64 heads x 64 columns
constexpr int kPSmemQ = 0;
constexpr int kPSmemK = kPSmemQ + 9 * kQChunkBytes;
constexpr int kPSmemPhi = kPSmemK + 2 * kStageBytes;
constexpr int kPSmemCtl = kPSmemPhi + kSlotBytes;
constexpr int kPSmemDynamic = 232448;             // the per-block opt-in maximum
constexpr int kValidRing = 4;                     // tiles whose valid bits are in flight
constexpr int kRopeSlot = 8;                      // slot of P's key half 0 once QK read it

// One S accumulator per tile: with 64 keys per thread the softmax reads S in
// one round of TMEM loads (measured faster than two partial sums).
constexpr int kPairQkPartials = 1;

constexpr uint32_t kPTmemCols = 512;
constexpr uint32_t kPTmemO = 0;    // O: 2 x 128 columns (N = 256 accumulators)
constexpr uint32_t kPTmemS = 256;  // S: 2 buffers of 128 columns (partial p at + 64 p)

struct PairCtl {
  // Leader only: all rows of stage s, chunk group g, of both CTAs landed.
  // Eight arrivals (each producer warp of each CTA, with the bytes of the
  // TMA loads it issued) plus the TMA transactions of both CTAs.
  uint64_t kv_full[2][3];
  uint64_t v_full[2];                // leader: both CTAs' re-gathered V columns (eight
                                     // arrivals: each V warp of each CTA, with its bytes)
  uint64_t qk_done[2];               // QK of the stage's tile complete (commit)
  uint64_t pv_done[2];               // PV of the stage's tile complete (commit)
  uint64_t vfull[kValidRing];        // valid bits of tile t in valid[t % 4]
  uint64_t vfree[kValidRing];        // the softmax has read them
  uint64_t p_full, m_p_full;         // P(t) written (local; mirror of CTA 1's)
  uint64_t q_full, q_empty;
  uint64_t s_full[2], s_empty[2], m_s_empty[2];
  uint64_t o_full, o_free, m_o_free, drain;
  uint64_t xbar[2][2];                // [parity][warp pair: warps w, w + 2 share heads]
  uint64_t fin_full[2], fin_free[2];
  uint64_t vsrc_full[2], vsrc_free[2];  // peer sources of a tile, producers -> V warps
  uint32_t tmem_base;
  volatile int abort;
  uint32_t valid[kValidRing][4];     // word w: slots 32 w .. 32 w + 31 of the tile
  float red[2][2][kHeadsPerCta];
  float fin_m[2][kHeadsPerCta];
  // Softmax sum of each head, both key halves added into it: two addends
  // from zero give the same float in either order.
  float fin_l[2][kHeadsPerCta];
  int32_t vsrc[2][kOwnRows];         // packed sources of the peer's rows of a tile
};
static_assert(kPSmemCtl + (int)sizeof(PairCtl) <= kPSmemDynamic, "shared memory budget");

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

// Arrival on a barrier of the other CTA of the pair (shared::cluster
// address).  Relaxed: every forwarded phase guards shared memory or TMEM that
// was complete before the arrival (generic stores fenced to the async proxy,
// TMEM stores waited), so the arrival only signals.
__device__ __forceinline__ void arrive_remote(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar)
               : "memory");
}

// Arrival with `bytes` of expected transactions on a barrier of the leader
// (shared::cluster address).  Release when the caller's own shared-memory
// writes (cp.async rows) must be visible before the phase completes.
__device__ __forceinline__ void arrive_tx_cluster(uint32_t cluster_bar, uint32_t bytes,
                                                  bool release) {
  if (release)
    asm volatile("mbarrier.arrive.expect_tx.release.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(
                     cluster_bar),
                 "r"(bytes)
                 : "memory");
  else
    asm volatile("mbarrier.arrive.expect_tx.relaxed.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(
                     cluster_bar),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// 2D tiled TMA load into this CTA's shared memory whose transactions complete
// on the barrier `bar` of the CTA pair's leader (shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y,
                                                 uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::"
      "bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// tile::gather4 of rows y0..y3 (column block x) into 4 consecutive 128-byte
// rows at dst, completing on the leader's barrier `bar`.
__device__ __forceinline__ void tma_gather4_pair(uint32_t dst, const CUtensorMap* map, int x,
                                                 int y0, int y1, int y2, int y3, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile::gather4.mbarrier::"
      "complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y0), "r"(y1), "r"(y2), "r"(y3), "r"(bar)
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

// Resolution of one pair tile (slots slot0 .. slot0 + 127, of which those at
// or past slot_end belong to another piece) for producer warp pw of CTA
// `rank`: the -1 scan of the whole tile (each warp scans all 128 slots, so
// the stop prefix needs no exchange), the valid bits of slots 32 pw .. 32 pw
// + 31, and the sources of the warp's gathered rows: lanes 0-15 slot 64 rank
// + 16 pw + lane (QK rows), lanes 16-31 slot 64 (1 - rank) + 16 pw + lane - 16
// (the peer's rows, whose d_v columns this CTA gathers again for PV).
struct TileRes {
  SlotSrc src;
  uint32_t valid32;
};

__device__ __forceinline__ TileRes resolve_pair_tile(const FwdArgs& a, const Row& rv,
                                                     const QueryKeys& qk, const int* idx_row,
                                                     int slot0, int slot_end, int pw, int rank,
                                                     int lane, bool* stopped, int* err) {
  uint32_t m1[4] = {0u, 0u, 0u, 0u};
  if (idx_row != nullptr) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int c = slot0 + 32 * u + lane - rv.window;
      const bool neg = (c >= 0 && c < qk.cmp) && (__ldg(idx_row + c) == -1);
      m1[u] = __ballot_sync(0xffffffffu, neg);
    }
  }
  auto blocked_before = [&](int k) {
    bool any = *stopped;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t below = (k >= 32 * (u + 1)) ? 0xffffffffu
                             : (k <= 32 * u)     ? 0u
                                                 : ((1u << (k - 32 * u)) - 1u);
      any = any || ((m1[u] & below) != 0u);
    }
    return any;
  };
  const int kv = 32 * pw + lane;
  const bool v = (slot0 + kv < slot_end) &&
                 slot_valid(rv, qk.thr, slot0 + kv, idx_row, blocked_before(kv));
  const int ks = (lane < 16 ? kOwnRows * rank : kOwnRows * (1 - rank)) + 16 * pw + (lane & 15);
  TileRes t;
  t.src = SlotSrc{-1, -1, false};
  if (slot0 + ks < slot_end)
    t.src = resolve_slot(a, rv, qk, slot0 + ks, idx_row, blocked_before(ks), err);
  t.valid32 = __ballot_sync(0xffffffffu, v);
  if ((m1[0] | m1[1] | m1[2] | m1[3]) != 0u) *stopped = true;
  return t;
}

__device__ __forceinline__ uint32_t group_chunks3(int cg, int nchunks) {
  return (uint32_t)max(0, min(3 * cg + 3, nchunks) - 3 * cg);
}

struct PairMaps {
  const CUtensorMap* ori;    // one-row box (tile::gather4)
  const CUtensorMap* cmp;
  const CUtensorMap* ori16;  // 16-row box
  const CUtensorMap* cmp16;
};

// Sixteen key rows of a tile into rows 16 pw .. 16 pw + 15 of chunk slots of
// a stage.  QK rows (v_part false): the sources in lanes 0-15, all `nchunks`
// chunks, chunk c into slot c, completing on bars[c / 3].  V rows (v_part
// true): the peer's rows in lanes 16-31, the four dims chunks 4 h + 2 rank + e
// that this CTA supplies to PV, into slots 4 h + 2 (1 - rank) + e, completing
// on bars[0].  One 16-row box per chunk when the rows are 16 consecutive rows
// of one cache, else tile::gather4 per 4-row group, or cp.async (16-byte
// copies, swizzled by hand) for a group that mixes the two caches; rows
// without a source read an out-of-range row, which TMA fills with zeros.  The
// warp then arrives once on each of its barriers with the TMA bytes it
// issued there (release, after its cp.async copies landed, when it issued
// any).
__device__ __forceinline__ void load_pair_rows(const FwdArgs& a, const SlotSrc& s, bool v_part,
                                               int rank, int pw, int lane, uint32_t stage,
                                               int nchunks, uint32_t bar0,
                                               const PairMaps& maps, uint32_t row_bytes,
                                               int gran) {
  const int l0 = v_part ? 16 : 0;
  const int nops = v_part ? 4 : nchunks;
  auto dims_of = [&](int k) { return v_part ? 4 * (k >> 1) + 2 * rank + (k & 1) : k; };
  auto slot_of = [&](int k) { return v_part ? 4 * (k >> 1) + 2 * (1 - rank) + (k & 1) : k; };
  // barriers of the chunk groups are consecutive in PairCtl::kv_full[s]
  auto bar_of = [&](int k) { return v_part ? bar0 : bar0 + 8u * (uint32_t)(k / 3); };
  const int li = l0 + (lane & 15);
  const int row_i = __shfl_sync(0xffffffffu, s.row, li);
  const int pool_i = __shfl_sync(0xffffffffu, s.pool, li);
  const int row0 = __shfl_sync(0xffffffffu, s.row, l0);
  const int pool0 = __shfl_sync(0xffffffffu, s.pool, l0);
  const bool run16 = __all_sync(0xffffffffu, pool0 >= 0 && row0 >= 0 && pool_i == pool0 &&
                                                 row_i == row0 + (lane & 15));
  const uint32_t rowoff = (uint32_t)(16 * pw) * 128u;
  uint32_t tma_rows = 16u;
  bool lsu = false;
  if (run16) {
    if (lane == 0) {
      const CUtensorMap* m = (pool0 == 1) ? maps.cmp16 : maps.ori16;
      for (int k = 0; k < nops; ++k)
        tma_load_2d_pair(stage + (uint32_t)(slot_of(k) * kSlotBytes) + rowoff, m, dims_of(k) * 64,
                         row0, bar_of(k));
    }
  } else {
    // lane q < 4: the 4-row group q
    const int q = lane & 3;
    int row[4], pool[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      row[i] = __shfl_sync(0xffffffffu, s.row, l0 + 4 * q + i);
      pool[i] = __shfl_sync(0xffffffffu, s.pool, l0 + 4 * q + i);
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
    const uint32_t mixed_mask = __ballot_sync(0xffffffffu, mixed && lane < 4) & 0xfu;
    tma_rows = 16u - 4u * (uint32_t)__popc(mixed_mask);
    if (lane < 4 && !mixed) {
      const CUtensorMap* m = (P == 1) ? maps.cmp : maps.ori;
      const int sentinel = (P == 1) ? a.cmp_rows : a.ori_rows;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (pool[i] < 0 || row[i] < 0) row[i] = sentinel;
      const uint32_t dst = stage + rowoff + (uint32_t)(4 * q) * 128u;
      for (int k = 0; k < nops; ++k)
        tma_gather4_pair(dst + (uint32_t)(slot_of(k) * kSlotBytes), m, dims_of(k) * 64, row[0],
                         row[1], row[2], row[3], bar_of(k));
    }
    // cp.async for the mixed groups: 4 rows x nops chunks x gran granules
    for (uint32_t mm = mixed_mask; mm != 0u; mm &= mm - 1u) {
      const int g = __ffs(mm) - 1;
      lsu = true;
      const int per_row = nops * 8;
      // sources of the group's rows, read by every lane
      int grow[4], gpool[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        grow[i] = __shfl_sync(0xffffffffu, s.row, l0 + 4 * g + i);
        gpool[i] = __shfl_sync(0xffffffffu, s.pool, l0 + 4 * g + i);
      }
      for (int o = lane; o < 4 * per_row; o += 32) {
        const int i = o / per_row;
        const int k = (o - i * per_row) >> 3;
        const int gr = o & 7;
        int rsel = grow[0], psel = gpool[0];
#pragma unroll
        for (int u = 1; u < 4; ++u)
          if (i == u) {
            rsel = grow[u];
            psel = gpool[u];
          }
        const bool has = (psel >= 0 && rsel >= 0 && dims_of(k) * 8 + gr < gran);
        const char* src = reinterpret_cast<const char*>(psel == 1 ? a.cmp_kv : a.ori_kv);
        if (has) src += (size_t)rsel * row_bytes + (size_t)(dims_of(k) * 8 + gr) * 16u;
        else src = reinterpret_cast<const char*>(a.ori_kv);
        cp_async_16(stage + (uint32_t)(slot_of(k) * kSlotBytes) + swz(16 * pw + 4 * g + i, gr),
                    src, has ? 16u : 0u);
      }
    }
  }
  if (lsu) {
    cp_async_wait_all();
    fence_proxy_async();
  }
  __syncwarp();
  if (lane == 0) {
    if (v_part) {
      arrive_tx_cluster(bar0, tma_rows * 128u * 4u, lsu);
    } else {
#pragma unroll
      for (int cg = 0; cg < 3; ++cg)
        arrive_tx_cluster(bar0 + 8u * (uint32_t)cg, tma_rows * 128u * group_chunks3(cg, nchunks),
                          lsu);
    }
  }
}

// Chunk group cg of S = Q K^T over the pair: chunk c of Q (64 heads) against
// chunk slot c of the CTA's 64 key rows, into partial c % kPairQkPartials (64
// TMEM columns each).
template <int kChunks>
__device__ __forceinline__ void issue_qk_pair(uint32_t d, uint32_t sQ, uint32_t stage,
                                              uint32_t idesc, int cg) {
  const uint64_t dq = smem_desc(sQ, 16, 1024);
  const uint64_t dk = smem_desc(stage, 16, 1024);
  const int c0 = 3 * cg;
  const int nc = min(3, kChunks - c0);
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      if (i < nc) {
        const int c = c0 + i;
        mma2(d + 64u * (c % kPairQkPartials), dq + (uint64_t)((c * kQChunkBytes + ks * 32) >> 4),
             dk + (uint64_t)((c * kSlotBytes + ks * 32) >> 4), idesc,
             (c < kPairQkPartials && ks == 0) ? 0u : 1u);
      }
    }
  }
}

// O (+)= P V over the pair: for key half kh (rows of CTA kh), A = P of that
// half (p_lo: keys 0-63, p_hi: keys 64-127), B = chunk slots 4 hv + 2 kh,
// 4 hv + 2 kh + 1 of the stage (MN-major, 64 rows): in place for the CTA's
// own keys, the re-gathered columns for the peer's.
__device__ __forceinline__ void issue_pv_pair(uint32_t o, uint32_t p_lo, uint32_t p_hi,
                                              uint32_t stage, uint32_t idesc, bool first) {
#pragma unroll
  for (int kh = 0; kh < 2; ++kh) {
    const uint64_t dp = smem_desc(kh ? p_hi : p_lo, 16, 1024);
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
      for (int hv = 0; hv < 2; ++hv) {
        const uint64_t dv =
            smem_desc(stage + (uint32_t)((4 * hv + 2 * kh) * kSlotBytes + ks * 2048), kSlotBytes,
                      1024);
        mma2(o + 128u * hv, dp + (uint64_t)((ks * 32) >> 4), dv, idesc,
             (first && kh == 0 && ks == 0) ? 0u : 1u);
      }
    }
  }
}

// A slot source in one int: 2 row + cache, -2 - cache for an unmapped page,
// -1 for a masked slot.
__device__ __forceinline__ int32_t pack_src(const SlotSrc& s) {
  if (s.pool < 0) return -1;
  return s.row >= 0 ? 2 * s.row + s.pool : -2 - s.pool;
}
__device__ __forceinline__ SlotSrc unpack_src(int32_t v) {
  if (v >= 0) return SlotSrc{v >> 1, v & 1, true};
  if (v == -1) return SlotSrc{-1, -1, false};
  return SlotSrc{-1, -2 - v, true};
}

// Walks the pair tiles of a worker span in plan order: tile j .. j + 1 of a
// (row, piece) [ja, jb), skipping rows without key tiles.  first / last: the
// pair tile opens / closes its (row, piece).
struct PairCursor {
  RowStream rs;
  Span span;
  Row row;
  int r, j, ja, jb;
  bool valid;
  __device__ __forceinline__ PairCursor(const int* rows, const Span& sp)
      : rs(rows, sp.r0, sp.r1), span(sp), r(sp.r0 - 1), j(0), ja(0), jb(0), valid(false) {
    next_row();
  }
  __device__ __forceinline__ void next_row() {
    valid = false;
    while (span.r0 >= 0 && ++r <= span.r1) {
      row = rs.take(r);
      const int tiles = row_tiles(row);
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
    j += 2;
    if (j >= jb) next_row();
  }
  __device__ __forceinline__ bool first() const { return j == ja; }
  __device__ __forceinline__ bool last() const { return j + 2 >= jb; }
};

// A mirror barrier of the leader (arrived remotely by CTA 1's roles), polled
// relaxed: it only orders the leader's MMA issue after CTA 1's shared memory
// or TMEM was complete (see arrive_remote).
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

// Epilogue of one 32-column block c of O (this thread's head row): scale by
// 1 / l and store, as bf16/fp16 into out or as fp32 into the split partials,
// straight from registers (each thread writes whole 32-byte sectors of its
// row).  Column block c is accumulator c / 4, dims (c / 4) * 256 + half * 128
// + (c % 4) * 32.  row_base: the thread's head row in out or the partials.
template <bool kBf16>
__device__ __forceinline__ void epi_direct(const uint32_t (&v)[32], int c, int half, float inv,
                                           bool split, char* row_base) {
  const int d0 = (c >> 2) * 256 + half * 128 + (c & 3) * 32;
  if (split) {
    uint4* dst = reinterpret_cast<uint4*>(row_base + (size_t)d0 * 4);
#pragma unroll
    for (int q = 0; q < 8; ++q)
      dst[q] = make_uint4(__float_as_uint(__uint_as_float(v[4 * q]) * inv),
                          __float_as_uint(__uint_as_float(v[4 * q + 1]) * inv),
                          __float_as_uint(__uint_as_float(v[4 * q + 2]) * inv),
                          __float_as_uint(__uint_as_float(v[4 * q + 3]) * inv));
  } else {
    uint4* dst = reinterpret_cast<uint4*>(row_base + (size_t)d0 * 2);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int i = 8 * q;
      dst[q] = make_uint4(
          pack2<kBf16>(__uint_as_float(v[i]) * inv, __uint_as_float(v[i + 1]) * inv),
          pack2<kBf16>(__uint_as_float(v[i + 2]) * inv, __uint_as_float(v[i + 3]) * inv),
          pack2<kBf16>(__uint_as_float(v[i + 4]) * inv, __uint_as_float(v[i + 5]) * inv),
          pack2<kBf16>(__uint_as_float(v[i + 6]) * inv, __uint_as_float(v[i + 7]) * inv));
    }
  }
}

template <bool kBf16, int kChunks, bool kTrace>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPThreads, 1)
    sas_pair_kernel(const FwdArgs args, const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_ori,
                    const __grid_constant__ CUtensorMap tm_cmp,
                    const __grid_constant__ CUtensorMap tm_ori16,
                    const __grid_constant__ CUtensorMap tm_cmp16) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t base = smem_addr(smem_raw);
  int* err = args.err;
  if ((base & 1023u) != 0u) {
    // the 128-byte swizzled chunks need a 1 KB aligned base (same in both
    // CTAs, so both leave here)
    if (threadIdx.x == 0) record_error(err, SAS_ERR_DEVICE, 119, (int)base);
    return;
  }
  PairCtl& ctl = *reinterpret_cast<PairCtl*>(smem_raw + kPSmemCtl);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = (int)cluster_rank();
  const bool leader = (rank == 0);
  const int worker = blockIdx.x >> 1;
  const int group = rank;
  const int* plan = args.plan;
  const int* rows = plan + plan[H_ROWS_OFF];
  constexpr int nchunks = kChunks;
  // Diagnostic clock trace (trace instances only) of CTA 0 of worker
  // args.trace_cta: region 0 producer warp 4 per tile (3 t: before the stage
  // wait, 3 t + 1: stage free, 3 t + 2: rows issued), [4096, 6144) 2 t: V
  // gather of tile t issued; region 1 the QK issuer (4 t: start, 4 t + 1:
  // issued) and the PV issuer (4 t + 2: inputs seen, 4 t + 3: issued);
  // region 2 softmax thread 0 ([0, 4000) 4 t: S seen, 4 t + 1: maximum
  // exchanged, 4 t + 2: P written, 4 t + 3: released; [4000, 6000) 2 t: S
  // in registers, 2 t + 1: valid bits seen), [6144, 8192) every CTA's start
  // / end (global timer); region 3 [0, 3072) chunk group g of tile t seen by
  // the QK issuer (3 t + g), [3072, 4096) softmax thread 96 at its maximum
  // exchange (t), [4096, 6144) the PV issuer's V (2 t) and P (2 t + 1) seen,
  // [6144, 8192) QK(t) seen complete by V warp 12 (t).
  long long* tr = (kTrace && worker == args.trace_cta && rank == 0) ? args.trace : nullptr;
  if (kTrace && args.trace != nullptr && threadIdx.x == 0 && blockIdx.x < 1024)
    args.trace[2 * kTraceRegion + 6144 + 2 * blockIdx.x] = (long long)global_ns();

  const uint32_t sQ = base + kPSmemQ;
  const uint32_t sK = base + kPSmemK;
  const uint32_t sPhi = base + kPSmemPhi;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      for (int g = 0; g < 3; ++g) mbar_init(smem_addr(&ctl.kv_full[i][g]), 8);
      mbar_init(smem_addr(&ctl.v_full[i]), 8);
      mbar_init(smem_addr(&ctl.qk_done[i]), 1);
      mbar_init(smem_addr(&ctl.pv_done[i]), 1);
      mbar_init(smem_addr(&ctl.s_full[i]), 1);
      mbar_init(smem_addr(&ctl.s_empty[i]), kPSoftmaxThreads);
      mbar_init(smem_addr(&ctl.m_s_empty[i]), 4);
      mbar_init(smem_addr(&ctl.xbar[i][0]), 64);
      mbar_init(smem_addr(&ctl.xbar[i][1]), 64);
      mbar_init(smem_addr(&ctl.fin_full[i]), kPSoftmaxThreads);
      mbar_init(smem_addr(&ctl.fin_free[i]), kPEpiThreads);
    }
    for (int i = 0; i < kValidRing; ++i) {
      mbar_init(smem_addr(&ctl.vfull[i]), 4);
      mbar_init(smem_addr(&ctl.vfree[i]), 2);  // after each warp pair's exchange
    }
    mbar_init(smem_addr(&ctl.p_full), kPSoftmaxThreads);
    mbar_init(smem_addr(&ctl.m_p_full), 4);
    mbar_init(smem_addr(&ctl.q_full), 2);  // one arrival per CTA, with its Q bytes
    mbar_init(smem_addr(&ctl.q_empty), 1);
    mbar_init(smem_addr(&ctl.o_full), 1);
    mbar_init(smem_addr(&ctl.o_free), kPEpiThreads);
    mbar_init(smem_addr(&ctl.m_o_free), 4);
    mbar_init(smem_addr(&ctl.drain), 2);  // one commit from each MMA issuer
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_addr(&ctl.vsrc_full[i]), 4);
      mbar_init(smem_addr(&ctl.vsrc_free[i]), 4);
      for (int h = 0; h < kHeadsPerCta; ++h) ctl.fin_l[i][h] = 0.f;
    }
    ctl.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kPQkWarp) {
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
    // Per pair tile t (stage t % 2): valid bits, the peer's sources for the V
    // warps, then, once PV(t - 2) has released the stage, the CTA's 64 rows.
    const int pw = warp - kPProducerWarp0;
    const int D = args.head_dim;
    const uint32_t row_bytes = (uint32_t)D * 2u;
    const int gran = D >> 3;
    const PairMaps maps{&tm_ori, &tm_cmp, &tm_ori16, &tm_cmp16};
    // the leader's barriers (shared::cluster addresses)
    auto kbar = [&](int s) { return peer_addr(smem_addr(&ctl.kv_full[s][0]), 0u); };
    int t = 0;  // pair tiles of the span so far
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
      const int slot_end = jb * kTileKeys;
      TileRes nxt = resolve_pair_tile(args, rv, qk, idx_row, ja * kTileKeys, slot_end, pw, rank,
                                      lane, &stopped, err);
      for (int j = ja; j < jb; j += 2, ++t) {
        const TileRes cur = nxt;
        if (j + 2 < jb)
          nxt = resolve_pair_tile(args, rv, qk, idx_row, (j + 2) * kTileKeys, slot_end, pw, rank,
                                  lane, &stopped, err);
        // the index lines of the tile after next into L1, so that its
        // resolve (one iteration later) reads L1 rather than L2
        if (idx_row != nullptr && j + 4 < jb && lane < 5) {
          const int c = (j + 4) * kTileKeys - rv.window + 32 * lane;
          if (c >= 0 && c < qk.cmp)
            asm volatile("prefetch.global.L1 [%0];" ::"l"(idx_row + c) : "memory");
        }
        const int own_slot = j * kTileKeys + kOwnRows * rank + 16 * pw + lane;
        if (args.slot_dump != nullptr && lane < 16 && own_slot < slot_end)
          dump_slot(args, rv.token, own_slot, cur.src);
        const int s = t & 1;
        const int vr = t % kValidRing;
        if (pw == 0 && lane == 0) trace_in(tr, 0, 0, 3 * t, 4096);
        // valid bits: the softmax has read tile t - 4's from this entry
        if (t >= kValidRing &&
            !__all_sync(0xffffffffu, wait_bar(&ctl, &ctl.vfree[vr],
                                              (uint32_t)(((t / kValidRing) - 1) & 1), err, 70))) {
          ok = false;
          break;
        }
        if (lane == 0) {
          ctl.valid[vr][pw] = cur.valid32;
          mbar_arrive(smem_addr(&ctl.vfull[vr]));
        }
        // the peer's sources of tile t for the V warps (vsrc[s] is free once
        // they have read tile t - 2's)
        if (t >= 2 && !__all_sync(0xffffffffu, wait_bar(&ctl, &ctl.vsrc_free[s],
                                                        (uint32_t)(((t >> 1) - 1) & 1), err, 75))) {
          ok = false;
          break;
        }
        if (lane >= 16) ctl.vsrc[s][16 * pw + lane - 16] = pack_src(cur.src);
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(&ctl.vsrc_full[s]));
        // the stage: PV(t - 2) has read it
        if (t >= 2 && !__all_sync(0xffffffffu, wait_bar(&ctl, &ctl.pv_done[s],
                                                        (uint32_t)(((t >> 1) - 1) & 1), err, 71))) {
          ok = false;
          break;
        }
        if (pw == 0 && lane == 0) trace_in(tr, 0, 0, 3 * t + 1, 4096);
        load_pair_rows(args, cur.src, false, rank, pw, lane, sK + s * kStageBytes, nchunks,
                       kbar(s), maps, row_bytes, gran);
        if (pw == 0 && lane == 0) trace_in(tr, 0, 0, 3 * t + 2, 4096);
      }
    }
    cp_async_wait_all();
  } else if (warp == kPQWarp) {
    // ======================= Q loader =======================
    // Q of a row (the CTA's 64 heads) once the last QK of the previous row
    // has released the Q buffer, completing on the leader's q_full; the next
    // row's Q is prefetched into L2 meanwhile.
    if (lane == 0) {
      const uint32_t q_bytes = (uint32_t)kHeadsPerCta * (uint32_t)args.head_dim * 2u;
      const uint32_t qbar = peer_addr(smem_addr(&ctl.q_full), 0u);
      uint32_t q_empty_par = 1u;
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
        arrive_tx_cluster(qbar, q_bytes, false);
        for (int c = 0; c < nchunks; ++c)
          tma_load_2d_pair(sQ + c * kQChunkBytes, &tm_q, c * 64, qrow, qbar);
      }
    }
    __syncwarp();
  } else if (warp == kPQkWarp || warp == kPPvWarp) {
    const bool qk_role = (warp == kPQkWarp);
    if (leader) {
      // ================= MMA issuers of the pair (CTA 0) =================
      // One thread issues the QKs, another the PVs; each waits (bounded) for
      // its inputs in both CTAs and issues in tile order.  The PV of tile t
      // follows its QK through P(t) (the softmax read S(t)) and the V columns
      // gathered after QK(t); QK(t + 2) reuses the S buffer of tile t after
      // the softmax released it.
      if (lane == 0) {
        bool ok = true;
        if (qk_role) {
          const uint32_t idesc_qk = instr_desc(128, 128, kBf16, false, false);
          PairCursor qc(rows, span);
          int tq = 0, row_i = 0;
          while (ok && qc.valid) {
            const int sb = tq & 1;
            if (qc.first()) ok = wait_bar(&ctl, &ctl.q_full, (uint32_t)(row_i & 1), err, 90);
            if (ok && tq >= 2) {
              const uint32_t sp = (uint32_t)(((tq >> 1) - 1) & 1);
              ok = wait_bar(&ctl, &ctl.s_empty[sb], sp, err, 92) &&
                   wait_mirror(&ctl, &ctl.m_s_empty[sb], sp, err, 93);
            }
            trace_in(tr, 1, 0, 4 * tq, 8192);
            const uint32_t kp = (uint32_t)((tq >> 1) & 1);
            for (int g = 0; ok && g < 3; ++g) {
              ok = wait_bar(&ctl, &ctl.kv_full[sb][g], kp, err, 94);
              if (!ok) break;
              trace_in(tr, 3, 0, 3 * tq + g, 3072);
              tc_fence_after();
              issue_qk_pair<nchunks>(tmem + kPTmemS + 128u * sb, sQ, sK + sb * kStageBytes,
                                     idesc_qk, g);
            }
            if (!ok) break;
            trace_in(tr, 1, 0, 4 * tq + 1, 8192);
            commit_both(smem_addr(&ctl.s_full[sb]));
            commit_both(smem_addr(&ctl.qk_done[sb]));
            if (qc.last()) {
              commit_both(smem_addr(&ctl.q_empty));
              ++row_i;
            }
            ++tq;
            qc.advance();
          }
        } else {
          const uint32_t idesc_pv = instr_desc(128, 256, kBf16, false, true);
          PairCursor pc(rows, span);
          int tp = 0, piece = 0;
          while (ok && pc.valid) {
            const int s = tp & 1;
            const uint32_t pp = (uint32_t)(tp & 1);
            ok = wait_bar(&ctl, &ctl.v_full[s], (uint32_t)((tp >> 1) & 1), err, 96);
            trace_in(tr, 3, 4096, 2 * tp, 2048);
            ok = ok && wait_bar(&ctl, &ctl.p_full, pp, err, 98) &&
                 wait_mirror(&ctl, &ctl.m_p_full, pp, err, 99);
            trace_in(tr, 3, 4096, 2 * tp + 1, 2048);
            if (ok && pc.first() && piece > 0) {
              const uint32_t op = (uint32_t)((piece - 1) & 1);
              ok = wait_bar(&ctl, &ctl.o_free, op, err, 100) &&
                   wait_mirror(&ctl, &ctl.m_o_free, op, err, 101);
            }
            if (!ok) break;
            tc_fence_after();
            trace_in(tr, 1, 0, 4 * tp + 2, 8192);
            const uint32_t stage = sK + s * kStageBytes;
            issue_pv_pair(tmem + kPTmemO, stage + kRopeSlot * kSlotBytes, sPhi, stage, idesc_pv,
                          pc.first());
            trace_in(tr, 1, 0, 4 * tp + 3, 8192);
            commit_both(smem_addr(&ctl.pv_done[s]));
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
    // ================= V gather and epilogue =================
    // Per pair tile t, epilogue warp ew gathers the d_v columns this CTA
    // supplies to PV of the peer's rows 16 ew .. 16 ew + 15 (sources from the
    // producers), once QK(t) has read stage t % 2; after the last tile of a
    // (row, piece), once its PV is done: O / l -> out (or the fp32 split
    // partials) and the LSE.
    const int ew = warp - kPEpiWarp0;
    const int half = ew >> 1;
    const int m0 = (ew & 1) * 32;
    const int m = m0 + lane;
    const int dv = args.head_dim_v;
    const uint32_t obase = tmem + ((uint32_t)(ew * 32) << 16) + kPTmemO;
    const bool live = group * kHeadsPerCta + m < args.num_heads;
    const PairMaps maps{&tm_ori, &tm_cmp, &tm_ori16, &tm_cmp16};
    const uint32_t row_bytes = (uint32_t)args.head_dim * 2u;
    const int gran = args.head_dim >> 3;
    PairCursor ec(rows, span);
    int t = 0, k = 0;
    while (ec.valid) {
      const int s = t & 1;
      const uint32_t tp = (uint32_t)((t >> 1) & 1);
      if (!__all_sync(0xffffffffu, wait_bar(&ctl, &ctl.vsrc_full[s], tp, err, 87))) break;
      SlotSrc src{-1, -1, false};
      if (lane >= 16) src = unpack_src(ctl.vsrc[s][16 * ew + lane - 16]);
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&ctl.vsrc_free[s]));
      if (!__all_sync(0xffffffffu, wait_bar(&ctl, &ctl.qk_done[s], tp, err, 72))) break;
      if (ew == 0 && lane == 0) trace_in(tr, 3, 6144, t, 2048);
      load_pair_rows(args, src, true, rank, ew, lane, sK + s * kStageBytes, nchunks,
                     peer_addr(smem_addr(&ctl.v_full[s]), 0u), maps, row_bytes, gran);
      if (ew == 0 && lane == 0) trace_in(tr, 0, 4096, 2 * t, 2048);
      if (ec.last()) {
        const Row& rv = ec.row;
        const int fp = k & 1;
        if (!__all_sync(0xffffffffu, wait_bar(&ctl, &ctl.o_full, (uint32_t)(k & 1), err, 80)))
          break;
        if (!__all_sync(0xffffffffu,
                        wait_bar(&ctl, &ctl.fin_full[fp], (uint32_t)((k >> 1) & 1), err, 81)))
          break;
        tc_fence_after();
        const float m_run = ctl.fin_m[fp][m];
        const float l_tot = ctl.fin_l[fp][m];
        // both epilogue threads of head m have read the sum: clear it for the
        // row after next
        asm volatile("bar.sync 1, %0;" ::"r"(kPEpiThreads) : "memory");
        if (half == 0) ctl.fin_l[fp][m] = 0.f;
        mbar_arrive(smem_addr(&ctl.fin_free[fp]));
        const float inv = (l_tot > 0.f) ? 1.f / l_tot : 0.f;
        const float lse = (m_run + log2f(l_tot)) * kLn2;
        const bool split = rv.partial_base >= 0;
        const int piece = (ec.r == span.r0) ? span.piece0 : 0;
        const size_t hrow = split ? (size_t)(rv.partial_base + piece) * args.num_heads +
                                        group * kHeadsPerCta + m
                                  : (size_t)rv.token * args.num_heads + group * kHeadsPerCta + m;
        char* row_base = split ? reinterpret_cast<char*>(args.o_partial + hrow * dv)
                               : reinterpret_cast<char*>(args.out) + hrow * dv * 2;
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
          uint32_t v[32];
          tmem_ld32(obase + 32u * c, v);
          tmem_wait_ld();
          if (live) epi_direct<kBf16>(v, c, half, inv, split, row_base);
        }
        if (half == 0 && live) {
          if (split)
            args.lse_partial[hrow] = lse;
          else
            args.lse[hrow] = lse;
        }
        tc_fence_before();
        mbar_arrive(smem_addr(&ctl.o_free));
        __syncwarp();
        if (!leader && lane == 0) arrive_remote(peer_addr(smem_addr(&ctl.m_o_free), 0u));
        ++k;
      }
      ++t;
      ec.advance();
    }
    cp_async_wait_all();
  } else if (warp < 4) {
    // ======================= softmax =======================
    // Thread L: head m = L % 64 of the CTA, key half L / 64 (keys 64 half ..
    // 64 half + 63 of each pair tile, TMEM lane L).
    const int L = threadIdx.x;
    const int m = L & (kHeadsPerCta - 1);
    const int half = L >> 6;
    const int head = group * kHeadsPerCta + m;
    const bool live = head < args.num_heads;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const float c2 = args.softmax_scale * kLog2e;
    const float sink = live ? __ldg(args.sinks + head) : -INFINITY;
    const uint32_t m_p_full = peer_addr(smem_addr(&ctl.m_p_full), 0u);
    uint32_t xph = 0u;
    int xpar = 0, rows_done = 0;
    int t = 0;  // pair tiles of the span so far
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
      for (int j = ja; j < jb; j += 2, ++t) {
        const int sb = t & 1;
        const int vr = t % kValidRing;
        if (!__all_sync(0xffffffffu, wait_bar(&ctl, &ctl.s_full[sb], (uint32_t)((t >> 1) & 1),
                                             err, 82))) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (threadIdx.x == 0) trace_in(tr, 2, 0, 4 * t, 4000);
        float x[64];
        {
          const uint32_t ts = tmem + lane_off + kPTmemS + 128u * sb;
          if constexpr (kPairQkPartials == 1) {
            // both 32-column halves in flight, one wait
            uint32_t a0[32], a1[32];
            tmem_ld32(ts, a0);
            tmem_ld32(ts + 32u, a1);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              x[i] = __uint_as_float(a0[i]);
              x[32 + i] = __uint_as_float(a1[i]);
            }
          } else {
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
              uint32_t a0[32], a1[32];
              tmem_ld32(ts + 32u * h2, a0);
              tmem_ld32(ts + 64u + 32u * h2, a1);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i)
                x[32 * h2 + i] = __uint_as_float(a0[i]) + __uint_as_float(a1[i]);
            }
          }
        }
        if (threadIdx.x == 0) trace_in(tr, 2, 4000, 2 * t, 2000);
        tc_fence_before();
        mbar_arrive(smem_addr(&ctl.s_empty[sb]));
        __syncwarp();
        if (!leader && lane == 0) arrive_remote(peer_addr(smem_addr(&ctl.m_s_empty[sb]), 0u));
        if (!__all_sync(0xffffffffu,
                        wait_bar(&ctl, &ctl.vfull[vr], (uint32_t)((t / kValidRing) & 1), err, 83))) {
          ok = false;
          break;
        }
        if (threadIdx.x == 0) trace_in(tr, 2, 4000, 2 * t + 1, 2000);
        const uint32_t va = ctl.valid[vr][2 * half];
        const uint32_t vb = ctl.valid[vr][2 * half + 1];
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const uint32_t w = (i < 32) ? (va >> i) : (vb >> (i - 32));
          const float v = (w & 1u) ? x[i] * c2 : -INFINITY;
          x[i] = v;
          mx = fmaxf(mx, v);
        }
        ctl.red[xpar][half][m] = mx;
        if (threadIdx.x == 96) trace_in(tr, 3, 3072, t, 1024);
        // the maximum is exchanged only between the two warps of the same
        // heads (warps w and w + 2)
        mbar_arrive(smem_addr(&ctl.xbar[xpar][warp & 1]));
        const bool xw = wait_bar(&ctl, &ctl.xbar[xpar][warp & 1], (xph >> xpar) & 1u, err, 84);
        xph ^= 1u << xpar;
        if (!__all_sync(0xffffffffu, xw)) {
          ok = false;
          break;
        }
        // both warps of each pair have read valid[vr]: the producers may
        // reuse it once both pairs arrived
        if (threadIdx.x < 64 && lane == 0) mbar_arrive(smem_addr(&ctl.vfree[vr]));
        if (threadIdx.x == 0) {
          trace_in(tr, 2, 0, 4 * t + 1, 4000);
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
        const bool rescale_o = (j > ja) && __any_sync(0xffffffffu, rescale);
        // P of key half 1 and O are free once PV(t - 1) is done; P of key
        // half 0 goes into the rope slot of this tile's stage, read by QK(t).
        if (t > 0 && (half == 1 || rescale_o) &&
            !__all_sync(0xffffffffu, wait_bar(&ctl, &ctl.pv_done[(t - 1) & 1],
                                              (uint32_t)(((t - 1) >> 1) & 1), err, 85))) {
          ok = false;
          break;
        }
        uint8_t* prow = half ? smem_raw + kPSmemPhi
                             : smem_raw + kPSmemK + sb * kStageBytes + kRopeSlot * kSlotBytes;
        float lsum = 0.f;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          uint32_t pk[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int i = 8 * g + 2 * q;
            const float p0 = ex2_approx(x[i] - m_use);
            const float p1 = ex2_approx(x[i + 1] - m_use);
            lsum += p0 + p1;
            pk[q] = pack2<kBf16>(p0, p1);
          }
          *reinterpret_cast<uint4*>(prow + swz(m, g)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
        l_run += lsum;
        fence_proxy_async();
        if (threadIdx.x == 0) trace_in(tr, 2, 0, 4 * t + 2, 4000);
        if (rescale_o) {
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
        if (!leader && lane == 0) arrive_remote(m_p_full);
        if (threadIdx.x == 0) trace_in(tr, 2, 0, 4 * t + 3, 4000);
      }
      if (!ok) break;
      const int fp = rows_done & 1;
      if (!__all_sync(0xffffffffu, wait_bar(&ctl, &ctl.fin_free[fp],
                                            (uint32_t)(((rows_done >> 1) & 1) ^ 1), err, 86)))
        break;
      if (half == 0) ctl.fin_m[fp][m] = m_run;
      atomicAdd(&ctl.fin_l[fp][m], l_run);
      mbar_arrive(smem_addr(&ctl.fin_full[fp]));
      ++rows_done;
    }
  }

  tc_fence_before();
  __syncthreads();
  // Neither CTA leaves while the other may still read its shared memory or
  // arrive on its barriers.
  cluster_sync_all();
  if (kTrace && args.trace != nullptr && threadIdx.x == 0 && blockIdx.x < 1024)
    args.trace[2 * kTraceRegion + 6144 + 2 * blockIdx.x + 1] = (long long)global_ns();
  if (warp == kPQkWarp) {
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
                           const CUtensorMap& tm_cmp, const CUtensorMap& tm_ori16,
                           const CUtensorMap& tm_cmp16) {
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(sas_pair_kernel<kBf16, kChunks, kTrace>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kPSmemDynamic) != cudaSuccess)
      return SAS_ERR_CUDA;
    configured = true;
  }
  sas_pair_kernel<kBf16, kChunks, kTrace><<<2 * workers, kPThreads, kPSmemDynamic, stream>>>(
      args, tm_q, tm_ori, tm_cmp, tm_ori16, tm_cmp16);
  return cudaGetLastError() == cudaSuccess ? SAS_OK : SAS_ERR_CUDA;
}

// The pair kernel for a plan with two head groups (65..128 heads); `workers`
// clusters of two CTAs.
int launch_fwd_pair(const FwdArgs& args, int workers, cudaStream_t stream) {
  const bool bf16 = args.dtype == SAS_DTYPE_BF16;
  if (args.head_dim != 576 && args.head_dim != 512) return SAS_ERR_UNSUPPORTED;
  alignas(64) CUtensorMap tm_q, tm_ori, tm_cmp, tm_ori16, tm_cmp16;
  const uint64_t D = (uint64_t)args.head_dim;
  if (!make_map_pair(&tm_q, args.q, (uint64_t)args.total_tokens * args.num_heads, D,
                     kHeadsPerCta))
    return SAS_ERR_CUDA;
  if (!make_map_pair(&tm_ori, args.ori_kv, (uint64_t)args.ori_rows, D, 1)) return SAS_ERR_CUDA;
  // A cache with fewer than 16 rows never takes the 16-row box path.
  const uint32_t ori_box = args.ori_rows < 16 ? (uint32_t)args.ori_rows : 16u;
  const uint32_t cmp_box = args.cmp_rows < 16 ? (uint32_t)args.cmp_rows : 16u;
  if (!make_map_pair(&tm_ori16, args.ori_kv, (uint64_t)args.ori_rows, D, ori_box))
    return SAS_ERR_CUDA;
  if (args.cmp_kv != nullptr && args.cmp_rows > 0) {
    if (!make_map_pair(&tm_cmp, args.cmp_kv, (uint64_t)args.cmp_rows, D, 1)) return SAS_ERR_CUDA;
    if (!make_map_pair(&tm_cmp16, args.cmp_kv, (uint64_t)args.cmp_rows, D, cmp_box))
      return SAS_ERR_CUDA;
  } else {
    tm_cmp = tm_ori;
    tm_cmp16 = tm_ori16;
  }
#define SAS_PAIR(B, C, T) \
  launch_pair_one<B, C, T>(args, workers, stream, tm_q, tm_ori, tm_cmp, tm_ori16, tm_cmp16)
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
