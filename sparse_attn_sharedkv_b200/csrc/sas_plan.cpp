// B200 work plan: splits the (query token, 64-key tile) work of one forward
// call over the persistent workers (one CTA per SM, or a pair of CTAs per
// worker when the call has more than 64 query heads).
//
// This is the role the reference gives its metadata table (per-core
// (bn2, m, s2) ranges plus flash-decode reduce tasks, metadata.py:795-827,
// 974-1009), rebuilt for 148 SMs: every query token is a row with
// `window + compressed` key slots (golden.py:125-150); rows are laid out in
// token order on a cost axis (a fixed per-row cost for the Q load and output
// store, plus one unit per 64-key tile, rounded up to whole 128-key pair
// tiles with two head groups) and cut into `num_workers` equal spans at tile
// granularity (pair-tile granularity with two head groups; rows of at most
// sas::kSnapTiles tiles whole).  A row whose tiles land on several workers is a
// split row: each worker writes an fp32 partial (normalised O + LSE) and the
// combine kernel merges them (the flash-decode reduction the reference plans
// but never runs).

#include <cstdint>
#include <cstring>
#include <vector>

#include "sas.h"
#include "sas_internal.h"

namespace {

using sas::kRowInts;

constexpr int64_t kRowCost = 1;   // Q load + epilogue, in tile units (sas::unit_mid2)
constexpr int64_t kTileCost = 1;

struct Row {
  int32_t token, b, s, slots, flags, window, win_lo, cmp, thr;
};

int collect_rows(const SasProblem& p, std::vector<Row>* rows) {
  if (p.batch <= 0 || p.num_heads <= 0 || p.num_heads > sas::kHeadsPerCta * sas::kMaxHeadGroups)
    return SAS_ERR_INVALID;
  if (!p.q_start || !p.q_len || !p.kv_len) return SAS_ERR_INVALID;
  if (p.layout_q != SAS_LAYOUT_TND && p.layout_q != SAS_LAYOUT_BSND) return SAS_ERR_INVALID;
  if (p.scenario < SAS_SCENARIO_SWA || p.scenario > SAS_SCENARIO_SCFA) return SAS_ERR_INVALID;
  if (p.scenario >= SAS_SCENARIO_CFA && p.cmp_ratio <= 0) return SAS_ERR_INVALID;
  if (p.scenario == SAS_SCENARIO_SCFA && p.topk <= 0) return SAS_ERR_INVALID;
  if (p.ori_win_left < -1) return SAS_ERR_INVALID;
  rows->clear();
  rows->reserve(p.total_tokens);
  for (int32_t b = 0; b < p.batch; ++b) {
    int32_t start = p.q_start[b], len = p.q_len[b], kv = p.kv_len[b];
    if (len < 0 || kv < 0 || start < 0) return SAS_ERR_INVALID;
    int32_t span = len;
    if (p.layout_q == SAS_LAYOUT_BSND) {
      if (len > p.max_q_len || start != b * p.max_q_len) return SAS_ERR_INVALID;
      span = p.max_q_len;  // slots past act_q are padded rows (zeros)
    }
    if ((int64_t)start + span > p.total_tokens) return SAS_ERR_INVALID;
    for (int32_t s = 0; s < span; ++s) {
      Row r{start + s, b, s, 0, 0, 0, 0, 0, 0};
      if (s >= len) {
        r.flags = sas::kRowPadded;
      } else {
        sas::QueryKeys k = sas::query_keys(p.scenario, len, kv, s, p.ori_win_left, p.cmp_ratio,
                                           p.topk);
        r.window = k.window;
        r.slots = sas::row_slots(k, p.scenario, p.ori_win_left, p.num_heads, &r.flags);
        r.win_lo = k.win_lo;
        r.cmp = k.cmp;
        r.thr = k.thr;
      }
      rows->push_back(r);
    }
  }
  return SAS_OK;
}

struct Built {
  std::vector<int32_t> plan;
  SasPlanInfo info;
};

int build(const SasProblem& p, int32_t num_sms, bool fill, Built* out) {
  std::vector<Row> rows;
  int rc = collect_rows(p, &rows);
  if (rc != SAS_OK) return rc;
  if (num_sms <= 0) return SAS_ERR_INVALID;
  const int32_t hg = (p.num_heads + sas::kHeadsPerCta - 1) / sas::kHeadsPerCta;
  const int64_t R = (int64_t)rows.size();

  // Cost axis.
  std::vector<int64_t> tiles(R), start(R + 1, 0);
  int64_t total_tiles = 0;
  for (int64_t r = 0; r < R; ++r) {
    tiles[r] = (rows[r].slots + sas::kTileKeys - 1) / sas::kTileKeys;
    total_tiles += tiles[r];
    start[r + 1] = start[r] + kRowCost + sas::tiles_cost(tiles[r], hg) * kTileCost;
  }
  const int64_t total = start[R];
  int64_t nw = num_sms / hg;
  if (nw < 1) nw = 1;
  if (R == 0) nw = 0;

  // Worker of a point on the cost axis (midpoints, doubled to stay integral).
  auto owner = [&](int64_t mid2) -> int64_t {
    int64_t w = (int64_t)(((__int128)mid2 * nw) / (2 * (__int128)total));
    return w >= nw ? nw - 1 : w;
  };

  std::vector<int32_t> wbeg_row(nw, -1), wbeg_tile(nw, 0), wend_row(nw, 0), wend_tile(nw, 0);
  std::vector<int32_t> wbeg_piece(nw, 0);  // piece ordinal of the worker's first row
  std::vector<int32_t> first_w(R, 0), partial_base(R, -1);
  std::vector<int32_t> split_token, split_pieces, split_base;
  int64_t partials = 0;
  for (int64_t r = 0; r < R; ++r) {
    int64_t units = tiles[r] > 0 ? tiles[r] : 1;
    int64_t w_first = -1, w_last = -1, pieces = 0;
    for (int64_t j = 0; j < units; ++j) {
      const int64_t mid2 = sas::unit_mid2(start[r], tiles[r], j, hg);
      int64_t w = owner(mid2);
      if (w_first < 0) w_first = w;
      if (w != w_last) {
        if (wbeg_row[w] < 0) {
          wbeg_row[w] = (int32_t)r;
          wbeg_tile[w] = (int32_t)j;
          wbeg_piece[w] = (int32_t)pieces;
        }
        w_last = w;
        ++pieces;
      }
      wend_row[w] = (int32_t)r;
      wend_tile[w] = (int32_t)(j + 1);
    }
    first_w[r] = (int32_t)w_first;
    if (pieces > 1) {
      partial_base[r] = (int32_t)partials;
      split_token.push_back(rows[r].token);
      split_pieces.push_back((int32_t)pieces);
      split_base.push_back((int32_t)partials);
      partials += pieces;
    }
  }

  const int64_t ns = (int64_t)split_token.size();
  const int64_t rows_off = sas::kHeaderInts;
  const int64_t workers_off = rows_off + sas::align64(R * kRowInts);
  const int64_t split_off = workers_off + sas::align64(nw * sas::kWorkerInts);
  const int64_t actq_off = split_off + sas::align64(ns * 4);
  const int64_t actkv_off = actq_off + sas::align64(p.batch);
  const int64_t total_ints = actkv_off + sas::align64(p.batch);

  out->info.num_rows = (int32_t)R;
  out->info.num_workers = (int32_t)nw;
  out->info.head_groups = hg;
  out->info.num_split_rows = (int32_t)ns;
  out->info.num_partials = (int32_t)partials;
  out->info.total_tiles = total_tiles;
  out->info.plan_ints = total_ints;
  out->info.split_off = split_off;
  out->info.actq_off = actq_off;
  out->info.actkv_off = actkv_off;
  if (!fill) return SAS_OK;

  std::vector<int32_t>& pl = out->plan;
  pl.assign(total_ints, 0);
  pl[sas::H_MAGIC] = sas::kPlanMagic;
  pl[sas::H_NUM_ROWS] = (int32_t)R;
  pl[sas::H_NUM_WORKERS] = (int32_t)nw;
  pl[sas::H_HEAD_GROUPS] = hg;
  pl[sas::H_NUM_SPLIT] = (int32_t)ns;
  pl[sas::H_NUM_PARTIALS] = (int32_t)partials;
  pl[sas::H_ROWS_OFF] = (int32_t)rows_off;
  pl[sas::H_WORKERS_OFF] = (int32_t)workers_off;
  pl[sas::H_SPLIT_OFF] = (int32_t)split_off;
  pl[sas::H_TOTAL_INTS] = (int32_t)total_ints;
  pl[sas::H_BATCH] = p.batch;
  pl[sas::H_ACTQ_OFF] = (int32_t)actq_off;
  pl[sas::H_ACTKV_OFF] = (int32_t)actkv_off;
  for (int32_t b = 0; b < p.batch; ++b) {
    pl[actq_off + b] = p.q_len[b];
    pl[actkv_off + b] = p.kv_len[b];
  }
  for (int64_t r = 0; r < R; ++r) {
    int32_t* e = &pl[rows_off + r * kRowInts];
    e[sas::R_TOKEN] = rows[r].token;
    e[sas::R_BATCH] = rows[r].b;
    e[sas::R_POS] = rows[r].s;
    e[sas::R_SLOTS] = rows[r].slots;
    e[sas::R_FLAGS] = rows[r].flags;
    e[sas::R_FIRST_WORKER] = first_w[r];
    e[sas::R_PARTIAL_BASE] = partial_base[r];
    e[sas::R_WINDOW] = rows[r].window;
    e[sas::R_WIN_LO] = rows[r].win_lo;
    e[sas::R_CMP] = rows[r].cmp;
    e[sas::R_THR] = rows[r].thr;
    e[sas::R_PAD] = 0;
  }
  for (int64_t w = 0; w < nw; ++w) {
    int32_t* e = &pl[workers_off + w * sas::kWorkerInts];
    if (wbeg_row[w] < 0) {  // idle worker: begin_row = -1
      e[0] = -1; e[1] = 0; e[2] = -1; e[3] = 0; e[4] = 0;
    } else {
      e[0] = wbeg_row[w]; e[1] = wbeg_tile[w]; e[2] = wend_row[w]; e[3] = wend_tile[w];
      e[4] = wbeg_piece[w];
    }
  }
  for (int64_t i = 0; i < ns; ++i) {
    int32_t* e = &pl[split_off + i * 4];
    e[0] = split_token[i]; e[1] = split_pieces[i]; e[2] = split_base[i]; e[3] = 0;
  }
  return SAS_OK;
}

}  // namespace

// Exposed to sas_capi.cu.
namespace sas {
int plan_build(const SasProblem& p, int32_t num_sms, std::vector<int32_t>* plan,
               SasPlanInfo* info) {
  Built b;
  int rc = build(p, num_sms, true, &b);
  if (rc != SAS_OK) return rc;
  *info = b.info;
  plan->swap(b.plan);
  return SAS_OK;
}
}  // namespace sas

extern "C" int sas_plan_size(const SasProblem* prob, int32_t num_sms, SasPlanInfo* info) {
  if (!prob || !info) return SAS_ERR_INVALID;
  Built b;
  int rc = build(*prob, num_sms, false, &b);
  if (rc != SAS_OK) return rc;
  *info = b.info;
  return SAS_OK;
}

extern "C" int sas_plan(const SasProblem* prob, int32_t num_sms, int32_t* plan, int64_t plan_len,
                        SasPlanInfo* info) {
  if (!prob || !plan || !info) return SAS_ERR_INVALID;
  Built b;
  int rc = build(*prob, num_sms, true, &b);
  if (rc != SAS_OK) return rc;
  if (plan_len < b.info.plan_ints) return SAS_ERR_INVALID;
  std::memcpy(plan, b.plan.data(), sizeof(int32_t) * b.info.plan_ints);
  *info = b.info;
  return SAS_OK;
}
