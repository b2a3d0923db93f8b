// Internal layout shared by the host planner (sas_plan.cpp), the C ABI
// (sas_capi.cu) and the kernels (sas_fwd.cu, sas_combine.cu).
#pragma once

#include <stdint.h>

#include "sas.h"

namespace sas {

// Geometry of the attention kernel.
constexpr int kHeadsPerCta = 64;   // query heads of one CTA (M of the .ws MMAs)
constexpr int kTileKeys = 64;      // key slots per pipeline tile (N of QK)
constexpr int kMaxHeadGroups = 2;  // H <= 128

// Serialised plan (int32), all sections 64-element aligned:
//   header[kHeaderInts]
//   rows[num_rows][kRowInts]      one per query token (incl. padded BSND rows),
//                                 with its key bounds (query_keys) precomputed
//   workers[num_workers][kWorkerInts]  begin_row, begin_tile, end_row, end_tile,
//                                 piece ordinal of begin_row (0 if begin_tile = 0)
//   split[num_split_rows][4]      token, pieces, partial_base, pad
//   batch: act_q[B] then (64-aligned) act_kv[B]
constexpr int kHeaderInts = 16;
constexpr int kRowInts = 12;
constexpr int kWorkerInts = 8;
enum HeaderField {
  H_MAGIC = 0, H_NUM_ROWS, H_NUM_WORKERS, H_HEAD_GROUPS, H_NUM_SPLIT, H_NUM_PARTIALS,
  H_ROWS_OFF, H_WORKERS_OFF, H_SPLIT_OFF, H_TOTAL_INTS, H_BATCH, H_ACTQ_OFF, H_ACTKV_OFF
};
enum RowField {
  R_TOKEN = 0,     // flat token id (row of q / out)
  R_BATCH,         // b
  R_POS,           // s: query index inside the batch
  R_SLOTS,         // key slots: window + compressed (before masking)
  R_FLAGS,         // bit0: padded BSND slot (write zeros); bit1: ring row
  R_FIRST_WORKER,  // first worker that processes a tile of this row (diagnostic)
  R_PARTIAL_BASE,  // partial slot of piece 0, or -1 when the row is not split
  R_WINDOW,        // window slots W (slots [0, W) are window keys)
  R_WIN_LO,        // first logical window position
  R_CMP,           // compressed slots scanned
  R_THR,           // causal threshold of the compressed positions
  R_PAD            // unused
};
constexpr int kRowPadded = 1;
// bit1: ring row.  A pure sliding window of at most kRingKeys keys is kept
// in the two K stages as a ring over cache positions (position p at stage
// half (p >> 6) & 1, row p & 63), so that the next query of the sequence
// reuses every key but one.  Ring rows always span two 64-key tiles.
constexpr int kRowRing = 2;
constexpr int32_t kRingKeys = 128;
constexpr int32_t kPlanMagic = 0x53415331;  // "SAS1"

inline int64_t align64(int64_t x) { return (x + 63) / 64 * 64; }

// Work accounting of one query (identical on host and device).
struct QueryKeys {
  int32_t window;   // W: keys of the sliding window
  int32_t win_lo;   // first logical window position
  int32_t cmp;      // compressed slots scanned (before -1 / filter masks)
  int32_t thr;      // causal threshold of the compressed branch
  int32_t cmp_len;  // floor(act_kv / ratio)
};

#if defined(__CUDACC__)
#define SAS_HD __host__ __device__
#else
#define SAS_HD
#endif

SAS_HD inline int32_t floordiv(int64_t a, int64_t b) {
  int64_t q = a / b;
  if ((a % b != 0) && ((a < 0) != (b < 0))) --q;
  return (int32_t)q;
}

// Key slots of query s of a batch with act_q queries over act_kv keys
// (golden.py:125-150): the window [max(s_g - left, 0), s_g] and the
// compressed slots min(K, threshold) (SCFA) or threshold (CFA).
SAS_HD inline QueryKeys query_keys(int32_t scenario, int32_t act_q, int32_t act_kv, int32_t s,
                                   int32_t win_left, int32_t ratio, int32_t topk) {
  QueryKeys k;
  int64_t s_g = (int64_t)act_kv - act_q + s;
  int64_t lo = s_g - win_left;
  if (lo < 0) lo = 0;
  int64_t hi = s_g + 1;
  k.window = hi > lo ? (int32_t)(hi - lo) : 0;
  k.win_lo = (int32_t)lo;
  k.cmp = 0;
  k.thr = 0;
  k.cmp_len = 0;
  if (scenario >= SAS_SCENARIO_CFA && ratio > 0) {
    k.thr = floordiv((int64_t)act_kv - act_q + s + 1, ratio);
    k.cmp_len = floordiv(act_kv, ratio);
    int32_t c = k.thr > 0 ? k.thr : 0;
    if (scenario == SAS_SCENARIO_SCFA && c > topk) c = topk;
    k.cmp = c;
  }
  return k;
}

// Cost axis of the work plan (both planners): 1 unit per row (Q load,
// epilogue) + 1 per 64-key tile.  Rows of at most kSnapTiles key tiles are
// never split between workers: all their units take the row's midpoint, so
// the worker whose share holds that point runs the whole row (no fp32
// partials to write and combine, and ring rows stay on the warm path).
// Longer rows are cut at tile granularity.
constexpr int64_t kSnapTiles = 4;

// Cost of a row's key tiles: one unit per 64-key tile; with two head groups
// (the CTA-pair kernel walks 128-key pair tiles) whole pairs, a half-used
// last pair costing as much as a full one.
SAS_HD inline int64_t tiles_cost(int64_t tiles, int32_t head_groups) {
  return head_groups == 2 ? 2 * ((tiles + 1) / 2) : tiles;
}

// Point of unit j of a row that starts at `start` on the cost axis and has
// `tiles` key tiles, doubled to stay integral; a row without tiles is one
// unit.  With two head groups both tiles of a pair take the pair's
// midpoint, so pieces of a split row start at even tiles (whole pair tiles).
SAS_HD inline int64_t unit_mid2(int64_t start, int64_t tiles, int64_t j, int32_t head_groups) {
  if (tiles <= 0) return 2 * start + 1;
  if (tiles <= kSnapTiles) return 2 * start + 1 + tiles_cost(tiles, head_groups);
  if (head_groups == 2) return 2 * (start + 1 + 2 * (j >> 1)) + 2;
  return 2 * (start + 1 + j) + 1;
}

// Windows of 65..128 keys with no compressed branch run as ring rows when
// the call has one head group (at most 64 heads); the two-CTA kernel used
// for more heads walks such windows as ordinary two-tile rows.
SAS_HD inline bool ring_window(int32_t scenario, int32_t win_left, int32_t num_heads) {
  return scenario == SAS_SCENARIO_SWA && win_left >= 64 && win_left < kRingKeys &&
         num_heads <= kHeadsPerCta;
}

// Key slots of a query row and its flags (both planners).
SAS_HD inline int32_t row_slots(const QueryKeys& k, int32_t scenario, int32_t win_left,
                                int32_t num_heads, int32_t* flags) {
  if (ring_window(scenario, win_left, num_heads) && k.window > 0) {
    *flags = kRowRing;
    return kRingKeys;
  }
  *flags = 0;
  return k.window + k.cmp;
}

}  // namespace sas
