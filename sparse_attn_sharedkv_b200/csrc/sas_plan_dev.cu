// Device-side work plan: the plan of sas_plan.cpp built on the GPU from
// device-resident sequence lengths, so a forward call needs no host read of
// cu_seqlens_q / seqused_kv (the reference syncs on them, api.py:210, 260,
// 336) and its launches can be recorded in a CUDA graph.
//
// Same rows, workers, split rows and partial bases as the host planner for
// the same lengths (rows carry the same key bounds; the cost axis is 1 per
// row + 1 per 64-key tile, whole pair tiles with two head groups,
// sas::tiles_cost; the owner of a unit is the worker whose share of the cost
// axis holds the unit's midpoint, sas::unit_mid2).  Only the section offsets differ:
// they are fixed by host-known bounds (rows = total_tokens, split rows <=
// workers - 1, partial slots <= 2 (workers - 1)); the unused split entries
// carry zero pieces.
//
// One CTA of 1024 threads, three passes over the rows, each thread owning a
// contiguous chunk of rows; two block-wide scans (cost axis, split rows).
// Worker entries are written by the unique row where ownership changes, so
// no atomics.  Invalid lengths (negative, a TND batch outside the token
// range, act_q > S in BSND, TND lengths that do not cover total_tokens) are
// recorded in the error word (site 60) and leave every worker idle.

#include <cuda_runtime.h>
#include <stdint.h>

#include "sas.h"
#include "sas_internal.h"

namespace {

constexpr int kThreads = 1024;
constexpr int64_t kRowCost = 1;
constexpr int64_t kTileCost = 1;

struct DevLayout {
  int64_t rows_off, workers_off, split_off, actq_off, actkv_off, start_off, pieces_off, total;
  int64_t ns_max, partials_max;
};

DevLayout dev_layout(int64_t R, int64_t nw, int64_t B) {
  DevLayout L{};
  L.ns_max = nw > 1 ? nw - 1 : 0;
  L.partials_max = 2 * L.ns_max;
  L.rows_off = sas::kHeaderInts;
  L.workers_off = L.rows_off + sas::align64(R * sas::kRowInts);
  L.split_off = L.workers_off + sas::align64(nw * sas::kWorkerInts);
  L.actq_off = L.split_off + sas::align64(L.ns_max * 4);
  L.actkv_off = L.actq_off + sas::align64(B);
  // Scratch after the plan proper: int64 cost-axis starts, int32 pieces.
  L.start_off = L.actkv_off + sas::align64(B);
  L.pieces_off = L.start_off + sas::align64(2 * R);
  L.total = L.pieces_off + sas::align64(R);
  return L;
}

// Exclusive block scan of one int64 per thread; returns the block total.
__device__ int64_t block_exclusive_scan(int64_t v, int64_t* out, int64_t* smem) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int64_t x = v;
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) smem[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int64_t w = lane < kThreads / 32 ? smem[lane] : 0;
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    smem[lane] = w;  // inclusive per warp
  }
  __syncthreads();
  const int64_t warp_off = warp > 0 ? smem[warp - 1] : 0;
  *out = warp_off + x - v;
  const int64_t total = smem[kThreads / 32 - 1];
  __syncthreads();
  return total;
}

__device__ __forceinline__ int64_t owner_of(int64_t mid2, int64_t nw, int64_t total) {
  const int64_t w = (mid2 * nw) / (2 * total);
  return w >= nw ? nw - 1 : w;
}

using sas::unit_mid2;

__device__ void record(int32_t* err, int detail) {
  if (err != nullptr && atomicCAS(err, 0, SAS_ERR_DEVICE) == 0) {
    err[1] = 60;
    err[2] = detail;
    err[3] = 0;
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    plan_dev_kernel(int32_t* __restrict__ plan, DevLayout L, int32_t batch, int32_t layout_q,
                    int32_t max_q_len, int32_t R, int32_t nw, int32_t hg, int32_t scenario,
                    int32_t win_left, int32_t ratio, int32_t topk,
                    const int32_t* __restrict__ q_start, const int32_t* __restrict__ q_len,
                    const int32_t* __restrict__ kv_len, int32_t* err) {
  __shared__ int64_t scan_smem[32];
  __shared__ int bad;
  const int tid = threadIdx.x;
  if (tid == 0) bad = 0;
  __syncthreads();
  int32_t* rows = plan + L.rows_off;
  int32_t* workers = plan + L.workers_off;
  int32_t* split = plan + L.split_off;
  int64_t* start = reinterpret_cast<int64_t*>(plan + L.start_off);
  int32_t* pieces = plan + L.pieces_off;
  const int per = (R + kThreads - 1) / kThreads;
  const int r_lo = min(R, tid * per), r_hi = min(R, r_lo + per);

  // ---- validation, batch arrays, idle workers ----
  int64_t qsum = 0;
  for (int b = tid; b < batch; b += kThreads) {
    const int32_t st = q_start[b], ql = q_len[b], kv = kv_len[b];
    plan[L.actq_off + b] = ql;
    plan[L.actkv_off + b] = kv;
    bool ok = st >= 0 && ql >= 0 && kv >= 0;
    if (layout_q == SAS_LAYOUT_BSND) ok = ok && ql <= max_q_len && st == b * max_q_len;
    else ok = ok && (int64_t)st + ql <= R && (b == 0 ? st == 0 : st == q_start[b - 1] + q_len[b - 1]);
    if (!ok) { bad = 1; record(err, b); }
    qsum += ql;
  }
  int64_t qsum_excl;
  const int64_t qtotal = block_exclusive_scan(qsum, &qsum_excl, scan_smem);
  if (tid == 0 && layout_q != SAS_LAYOUT_BSND && qtotal != R) { bad = 1; record(err, -1); }
  for (int w = tid; w < nw; w += kThreads) {
    int32_t* e = workers + (int64_t)w * sas::kWorkerInts;
    e[0] = -1; e[1] = 0; e[2] = -1; e[3] = 0; e[4] = 0; e[5] = 0; e[6] = 0; e[7] = 0;
  }
  __syncthreads();
  const bool invalid = bad != 0;

  // ---- pass 1: rows, key bounds, cost ----
  int64_t my_cost = 0;
  for (int r = r_lo; r < r_hi; ++r) {
    int b, s;
    if (layout_q == SAS_LAYOUT_BSND) {
      b = r / max_q_len;
      s = r - b * max_q_len;
    } else {
      int lo = 0, hi = batch - 1;  // last b with q_start[b] <= r
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (q_start[mid] <= r) lo = mid; else hi = mid - 1;
      }
      b = lo;
      s = r - q_start[b];
    }
    int32_t* e = rows + (int64_t)r * sas::kRowInts;
    const int32_t ql = invalid ? 0 : q_len[b];
    e[sas::R_TOKEN] = r;
    e[sas::R_BATCH] = b;
    e[sas::R_POS] = s;
    e[sas::R_FIRST_WORKER] = 0;
    e[sas::R_PARTIAL_BASE] = -1;
    e[sas::R_PAD] = 0;
    int32_t slots = 0;
    if (s >= ql) {
      e[sas::R_FLAGS] = sas::kRowPadded;
      e[sas::R_WINDOW] = 0; e[sas::R_WIN_LO] = 0; e[sas::R_CMP] = 0; e[sas::R_THR] = 0;
    } else {
      const sas::QueryKeys k = sas::query_keys(scenario, ql, kv_len[b], s, win_left, ratio, topk);
      int32_t flags = 0;
      slots = sas::row_slots(k, scenario, win_left, hg * sas::kHeadsPerCta, &flags);
      e[sas::R_FLAGS] = flags;
      e[sas::R_WINDOW] = k.window; e[sas::R_WIN_LO] = k.win_lo;
      e[sas::R_CMP] = k.cmp; e[sas::R_THR] = k.thr;
    }
    e[sas::R_SLOTS] = slots;
    my_cost += kRowCost +
               sas::tiles_cost((slots + sas::kTileKeys - 1) / sas::kTileKeys, hg) * kTileCost;
  }
  int64_t my_start;
  const int64_t total = block_exclusive_scan(my_cost, &my_start, scan_smem);
  {
    int64_t st = my_start;
    for (int r = r_lo; r < r_hi; ++r) {
      start[r] = st;
      const int32_t slots = rows[(int64_t)r * sas::kRowInts + sas::R_SLOTS];
      st += kRowCost +
            sas::tiles_cost((slots + sas::kTileKeys - 1) / sas::kTileKeys, hg) * kTileCost;
    }
  }
  __syncthreads();

  // ---- pass 2: owners of every unit, worker spans, pieces per row ----
  auto tiles_of = [&](int r) -> int64_t {
    const int32_t slots = rows[(int64_t)r * sas::kRowInts + sas::R_SLOTS];
    return (slots + sas::kTileKeys - 1) / sas::kTileKeys;
  };
  for (int r = r_lo; r < r_hi && !invalid; ++r) {
    const int64_t tiles = tiles_of(r);
    const int64_t units = tiles > 0 ? tiles : 1;
    int64_t prev_owner = -1;  // owner of the previous row's last unit
    if (r > 0) {
      const int64_t pt = tiles_of(r - 1);
      prev_owner = owner_of(unit_mid2(start[r - 1], pt, (pt > 0 ? pt : 1) - 1, hg), nw, total);
    }
    int64_t next_owner = -1;  // owner of the next row's first unit
    if (r + 1 < R) next_owner = owner_of(unit_mid2(start[r + 1], tiles_of(r + 1), 0, hg), nw, total);
    int64_t w_prev = -1, npieces = 0, w_first = -1;
    for (int64_t j = 0; j < units; ++j) {
      const int64_t w = owner_of(unit_mid2(start[r], tiles, j, hg), nw, total);
      if (j == 0) w_first = w;
      const bool new_global = (j == 0) ? (w != prev_owner) : (w != w_prev);
      if (w != w_prev) {
        if (new_global) {
          int32_t* e = workers + w * sas::kWorkerInts;
          e[0] = r; e[1] = (int32_t)j; e[4] = (int32_t)npieces;
        }
        ++npieces;
      }
      const int64_t wn = (j + 1 < units) ? owner_of(unit_mid2(start[r], tiles, j + 1, hg), nw, total)
                                         : next_owner;
      if (wn != w) {
        int32_t* e = workers + w * sas::kWorkerInts;
        e[2] = r; e[3] = (int32_t)(j + 1);
      }
      w_prev = w;
    }
    rows[(int64_t)r * sas::kRowInts + sas::R_FIRST_WORKER] = (int32_t)w_first;
    pieces[r] = (int32_t)npieces;
  }
  __syncthreads();

  // ---- pass 3: split rows and partial bases ----
  int64_t my_split = 0, my_parts = 0;
  for (int r = r_lo; r < r_hi && !invalid; ++r) {
    if (pieces[r] > 1) { ++my_split; my_parts += pieces[r]; }
  }
  int64_t split0, parts0;
  const int64_t ns = block_exclusive_scan(my_split, &split0, scan_smem);
  const int64_t np = block_exclusive_scan(my_parts, &parts0, scan_smem);
  for (int r = r_lo; r < r_hi && !invalid; ++r) {
    const int32_t pc = pieces[r];
    if (pc > 1) {
      rows[(int64_t)r * sas::kRowInts + sas::R_PARTIAL_BASE] = (int32_t)parts0;
      int32_t* e = split + split0 * 4;
      e[0] = r; e[1] = pc; e[2] = (int32_t)parts0; e[3] = 0;
      ++split0;
      parts0 += pc;
    }
  }
  for (int64_t i = (invalid ? 0 : ns) + tid; i < L.ns_max; i += kThreads) {
    int32_t* e = split + i * 4;
    e[0] = 0; e[1] = 0; e[2] = 0; e[3] = 0;
  }
  if (tid == 0) {
    plan[sas::H_MAGIC] = sas::kPlanMagic;
    plan[sas::H_NUM_ROWS] = R;
    plan[sas::H_NUM_WORKERS] = nw;
    plan[sas::H_HEAD_GROUPS] = hg;
    plan[sas::H_NUM_SPLIT] = invalid ? 0 : (int32_t)ns;
    plan[sas::H_NUM_PARTIALS] = invalid ? 0 : (int32_t)np;
    plan[sas::H_ROWS_OFF] = (int32_t)L.rows_off;
    plan[sas::H_WORKERS_OFF] = (int32_t)L.workers_off;
    plan[sas::H_SPLIT_OFF] = (int32_t)L.split_off;
    plan[sas::H_TOTAL_INTS] = (int32_t)L.total;
    plan[sas::H_BATCH] = batch;
    plan[sas::H_ACTQ_OFF] = (int32_t)L.actq_off;
    plan[sas::H_ACTKV_OFF] = (int32_t)L.actkv_off;
    for (int i = 13; i < sas::kHeaderInts; ++i) plan[i] = 0;
  }
}

}  // namespace

namespace sas {

// Info of a device-built plan: upper bounds where the host cannot know the
// value (split rows, partial slots), exact otherwise.
int plan_dev_info(const SasProblem& p, int32_t num_sms, SasPlanInfo* info) {
  if (p.batch <= 0 || p.num_heads <= 0 || p.num_heads > kHeadsPerCta * kMaxHeadGroups)
    return SAS_ERR_INVALID;
  if (p.layout_q != SAS_LAYOUT_TND && p.layout_q != SAS_LAYOUT_BSND) return SAS_ERR_INVALID;
  if (p.scenario < SAS_SCENARIO_SWA || p.scenario > SAS_SCENARIO_SCFA) return SAS_ERR_INVALID;
  if (p.scenario >= SAS_SCENARIO_CFA && p.cmp_ratio <= 0) return SAS_ERR_INVALID;
  if (p.scenario == SAS_SCENARIO_SCFA && p.topk <= 0) return SAS_ERR_INVALID;
  if (p.ori_win_left < -1 || p.total_tokens < 0 || num_sms <= 0) return SAS_ERR_INVALID;
  if (p.layout_q == SAS_LAYOUT_BSND &&
      (p.max_q_len <= 0 || (int64_t)p.batch * p.max_q_len != p.total_tokens))
    return SAS_ERR_INVALID;
  const int32_t hg = (p.num_heads + kHeadsPerCta - 1) / kHeadsPerCta;
  const int64_t R = p.total_tokens;
  int64_t nw = num_sms / hg;
  if (nw < 1) nw = 1;
  if (R == 0) nw = 0;
  const DevLayout L = dev_layout(R, nw, p.batch);
  info->num_rows = (int32_t)R;
  info->num_workers = (int32_t)nw;
  info->head_groups = hg;
  info->num_split_rows = (int32_t)L.ns_max;
  info->num_partials = (int32_t)L.partials_max;
  info->total_tiles = -1;
  info->plan_ints = L.total;
  info->split_off = L.split_off;
  info->actq_off = L.actq_off;
  info->actkv_off = L.actkv_off;
  return SAS_OK;
}

int plan_dev_launch(const SasProblem& p, const SasPlanInfo& info, int32_t* dplan, int32_t* err,
                    cudaStream_t stream) {
  if (info.num_rows == 0) return SAS_OK;
  const DevLayout L = dev_layout(info.num_rows, info.num_workers, p.batch);
  plan_dev_kernel<<<1, kThreads, 0, stream>>>(dplan, L, p.batch, p.layout_q, p.max_q_len,
                                              info.num_rows, info.num_workers, info.head_groups,
                                              p.scenario, p.ori_win_left, p.cmp_ratio, p.topk,
                                              p.q_start, p.q_len, p.kv_len, err);
  return cudaGetLastError() == cudaSuccess ? SAS_OK : SAS_ERR_CUDA;
}

}  // namespace sas
