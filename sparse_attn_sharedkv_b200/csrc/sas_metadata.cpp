// Host scheduler of the SparseAttnSharedkvMetadata operator, in C++.
//
// Bit-exact restatement of the reference's Python port of the aicpu
// `BalanceSchedule` (metadata.py:258-1015): per-(batch, kv-head, query-row
// group, 512-key block) cost model `6*ceil(m/16) + 10*ceil(s2/64)`
// (metadata.py:428-438), greedy assignment of work to cores batch -> row ->
// block with a tolerance of half the last block's cost (metadata.py:718-793),
// flash-decode (split-KV) bookkeeping (metadata.py:795-827, 925-954; dormant
// because `supportFd` is false, metadata.py:320-325) and serialisation into
// int32[1024] = faMetadata[36][8] + fdMetadata[72][8] (metadata.py:974-1009).
//
// The step order and state updates follow the reference one for one, because
// the output is compared bit for bit; the arithmetic is written in 128-bit
// integers where the reference relies on Python's unbounded ints
// (pre-token = INT64_MAX windows, metadata.py:362-374, 409-412).
//
// One divergence, documented: the reference's row walk
// (`_assign_by_row`, metadata.py:759-763) loops forever when no later query
// row has a key block (a window of 0 with no compressed branch).  Here the
// walk is bounded and the call returns SAS_ERR_SCHEDULE instead of hanging.

#include <cstdint>
#include <cstring>
#include <vector>

#include "sas.h"

namespace {

using i64 = long long;
using i128 = __int128;

constexpr i64 kInt64Max = 0x7fffffffffffffffLL;
constexpr int kToleranceRatio = 2;  // FA_TOLERANCE_RATIO, metadata.py:80

enum BlockType { WIN_NORMAL = 0, WIN_TAIL = 1, CMP_NORMAL = 2, CMP_TAIL = 3, BLOCK_TYPES = 4 };
enum MaskMode { DEFAULT_MASK = 0, ALL_MASK = 1, LEFT_UP_CAUSAL = 2, RIGHT_DOWN_CAUSAL = 3,
                BAND = 4 };

struct BatchCache {
  i64 b_idx = 0, s1_size = 0, s2_size = 0;
  i128 pre_left_up = 0, next_left_up = 0;
};

struct RowCache {  // S1GCache, metadata.py:154-177
  i64 b_idx = 0, s1g_idx = 0, s2_start = 0, s2_end = 0;
  i64 win_s2_start = 0, win_s2_end = 0, cmp_s2_start = 0, cmp_s2_end = 0;
  i64 cost = 0, last_block_cost = 0, block = 0, normal_block_cost = 0;
  i64 win_block = 0, win_cost = 0, win_last_block_cost = 0, win_normal_block_cost = 0;
  i64 cmp_block = 0, cmp_cost = 0, cmp_last_block_cost = 0, cmp_normal_block_cost = 0;
  i64 cmp_tail = 0, win_tail = 0;
};

struct CoreCache { i64 cost_limit = 0, cost = 0, block = 0; };

struct Assign {  // AssignContext, metadata.py:187-203
  i64 b = 0, bn2 = 0, s1g = 0, s2 = 0, core = 0, unassigned = 0, used_cores = 0;
  i64 kv_split_part = 1, fd_data_num = 1, bn2_cost = 0, bn2_block = 0;
  bool finished = false;
  BatchCache bc;
  RowCache rc;
  CoreCache cc;
};

struct Split {  // SplitInfo + CostInfo
  std::vector<i64> s1g_num, s2_num, s1g_tail, s2_tail;
  bool all_zero = true;
  std::vector<i64> bn2_cost, bn2_block, bn2_last_block_cost;
  i64 total_block = 0, total_cost = 0, max_row_cost = 0;
};

struct Result {  // SplitResult + FlashDecodeResult
  i64 used_cores = 0, max_cost = 0, fd_heads = 0, max_split = 0, fd_used_vec = 0;
  std::vector<i64> bn2_end, s1g_end, s2_end, first_fd_ws;
  std::vector<i64> fd_bn2, fd_m, fd_ws, fd_split, fd_msize, fd_idx, fd_mstart, fd_mnum;
};

bool within(i64 limit, i64 tol, i64 value) { return (i128)limit + tol >= value; }
i64 cost_of(i64 m, i64 s2) { return 6 * ((m + 15) >> 4) + 10 * ((s2 + 63) >> 6); }

class Scheduler {
 public:
  explicit Scheduler(const SasMetaParams& p) : p_(p) {}

  int run(int32_t* out) {
    init();
    Result r;
    r.bn2_end.assign(aic_, 0); r.s1g_end.assign(aic_, 0); r.s2_end.assign(aic_, 0);
    r.first_fd_ws.assign(aic_, 0);
    r.fd_bn2.assign(aic_, 0); r.fd_m.assign(aic_, 0); r.fd_ws.assign(aic_, 0);
    r.fd_split.assign(aic_, 0); r.fd_msize.assign(aic_, 0);
    r.fd_idx.assign(aiv_, 0); r.fd_mstart.assign(aiv_, 0); r.fd_mnum.assign(aiv_, 0);
    int rc = balance(r);
    if (rc != SAS_OK) return rc;
    emit(r, out);
    return SAS_OK;
  }

 private:
  const SasMetaParams& p_;
  i64 batch_ = 0, group_ = 0, mbase_ = 0, s2base_ = 512, aic_ = 0, aiv_ = 0;
  i128 pre_ = 0, next_ = 0;
  int attention_mode_ = 1;
  bool s1g_layout_ = true, cfa_ = false, scfa_ = false;
  static constexpr bool kSupportFd = false;  // metadata.py:325
  i64 type_cost_[BLOCK_TYPES][BLOCK_TYPES] = {};

  bool tnd_q() const { return p_.layout_q == SAS_LAYOUT_TND; }
  bool tnd_kv() const { return p_.layout_kv == SAS_LAYOUT_TND; }

  i64 query_batch() const {
    if (p_.n_seqused_q > 0) return p_.n_seqused_q;
    if (tnd_q() && p_.n_cu_seqlens_q > 0) return p_.n_cu_seqlens_q - 1;
    return p_.batch_size;
  }
  i64 s1_size(i64 b) const {
    if (p_.n_seqused_q > 0) return p_.seqused_q[b];
    if (tnd_q() && p_.n_cu_seqlens_q > 0) return p_.cu_seqlens_q[b + 1] - p_.cu_seqlens_q[b];
    return p_.max_seqlen_q;
  }
  i64 s2_size(i64 b) const {
    if (p_.n_seqused_kv > 0) return p_.seqused_kv[b];
    if (tnd_kv() && p_.n_cu_seqlens_ori_kv > 0)
      return p_.cu_seqlens_ori_kv[b + 1] - p_.cu_seqlens_ori_kv[b];
    return p_.max_seqlen_kv;
  }

  void init() {  // _params_init, metadata.py:359-389
    batch_ = query_batch();
    aic_ = p_.aic_core_num;
    aiv_ = p_.aiv_core_num;
    switch (p_.ori_mask_mode) {
      case DEFAULT_MASK: pre_ = kInt64Max; next_ = kInt64Max; attention_mode_ = 0; break;
      case RIGHT_DOWN_CAUSAL: pre_ = kInt64Max; next_ = 0; attention_mode_ = 1; break;
      default:
        pre_ = p_.ori_win_left > -1 ? (i128)p_.ori_win_left : (i128)kInt64Max;
        next_ = 0; attention_mode_ = 1; break;
    }
    s1g_layout_ = p_.layout_q == SAS_LAYOUT_BSND || p_.layout_q == SAS_LAYOUT_BSH ||
                  p_.layout_q == SAS_LAYOUT_TND;
    group_ = p_.num_heads_kv == 0 ? 0 : p_.num_heads_q / p_.num_heads_kv;
    if (p_.has_cmp_kv) {
      if (p_.cmp_topk > 0) scfa_ = true; else cfa_ = true;
    }
    mbase_ = group_;
    s2base_ = 512;
  }

  i128 pre_left_up(i64 s1, i64 s2) const {
    return p_.ori_mask_mode == BAND ? (i128)s1 - s2 + pre_ : pre_;
  }
  i128 next_left_up(i64 s1, i64 s2) const {
    switch (p_.ori_mask_mode) {
      case DEFAULT_MASK: case ALL_MASK: case LEFT_UP_CAUSAL: return next_;
      case RIGHT_DOWN_CAUSAL: return (i128)s2 - s1;
      case BAND: return (i128)s2 - s1 + next_;
      default: return next_;
    }
  }

  void cost_table(i64 s1n, i64 s2n, i64 s1t, i64 wt, i64 ct) {  // metadata.py:440-477
    auto& tc = type_cost_;
    tc[WIN_NORMAL][WIN_NORMAL] = cost_of(s1n, s2n);
    tc[WIN_TAIL][WIN_NORMAL] = s1t == 0 ? 0 : cost_of(s1t, s2n);
    tc[WIN_NORMAL][WIN_TAIL] = wt == 0 ? 0 : cost_of(s1n, wt);
    tc[WIN_TAIL][WIN_TAIL] = (s1t == 0 || wt == 0) ? 0 : cost_of(s1t, wt);
    if (p_.has_cmp_kv) {
      tc[CMP_NORMAL][CMP_NORMAL] = cost_of(s1n, s2n);
      tc[CMP_TAIL][CMP_NORMAL] = s1t == 0 ? 0 : cost_of(s1t, s2n);
      tc[CMP_NORMAL][CMP_TAIL] = ct == 0 ? 0 : cost_of(s1n, ct);
      tc[CMP_TAIL][CMP_TAIL] = (s1t == 0 || ct == 0) ? 0 : cost_of(s1t, ct);
    }
  }

  // Key range of one query-row group (metadata.py:479-501); 128-bit because
  // the window edges may sit at +-INT64_MAX.
  void s2_token_range(i64 s1g, const BatchCache& bc, i128* first, i128* last) const {
    if (bc.s1_size == 0 || bc.s2_size == 0) { *first = 0; *last = 0; return; }
    if (!attention_mode_) { *first = 0; *last = bc.s2_size - 1; return; }
    i64 g_first = s1g * mbase_;
    i64 g_last = (g_first + mbase_ < bc.s1_size * group_ ? g_first + mbase_
                                                          : bc.s1_size * group_) - 1;
    i64 q_first, q_last;
    if (s1g_layout_) {
      q_first = pydiv(g_first, group_);
      q_last = pydiv(g_last, group_);
    } else if (pydiv(g_first, bc.s1_size) == pydiv(g_last, bc.s1_size)) {
      q_first = pymod(g_first, bc.s1_size);
      q_last = pymod(g_last, bc.s1_size);
    } else {
      q_first = 0;
      q_last = bc.s1_size;
    }
    *first = (i128)q_first - bc.pre_left_up;
    *last = (i128)q_last + bc.next_left_up;
  }

  static i64 pydiv(i64 a, i64 b) { i64 q = a / b; if ((a % b != 0) && ((a < 0) != (b < 0))) --q; return q; }
  static i64 pymod(i64 a, i64 b) { i64 m = a % b; if (m != 0 && ((m < 0) != (b < 0))) m += b; return m; }

  void batch_cache(i64 b, BatchCache* bc) const {  // metadata.py:505-510
    bc->b_idx = b;
    bc->s1_size = s1_size(b);
    bc->s2_size = s2_size(b);
    bc->pre_left_up = pre_left_up(bc->s1_size, bc->s2_size);
    bc->next_left_up = next_left_up(bc->s1_size, bc->s2_size);
  }

  void block_range(i128 first, i128 last, const BatchCache& bc, RowCache* rc) const {
    // metadata.py:512-547
    i64 f, l;
    if (first >= bc.s2_size || last < 0 || last < first) {
      f = 0; l = 0;
      rc->win_s2_start = 0; rc->win_s2_end = 0; rc->win_tail = 0;
    } else {
      f = (i64)(first < 0 ? 0 : (first > bc.s2_size - 1 ? bc.s2_size - 1 : first));
      l = (i64)(last < 0 ? 0 : (last > bc.s2_size - 1 ? bc.s2_size - 1 : last));
      rc->win_s2_start = 0;
      rc->win_s2_end = (l - f) / s2base_ + 1;
      rc->win_tail = (l - f + 1) % s2base_;
    }
    rc->cmp_s2_start = rc->win_s2_end;
    i64 cmp_last_size = (p_.has_cmp_kv && p_.cmp_ratio > 0) ? (l + 1) / p_.cmp_ratio : 0;
    i64 act = 0;
    if (cfa_) act = cmp_last_size;
    else if (scfa_) act = cmp_last_size < p_.cmp_topk ? cmp_last_size : p_.cmp_topk;
    rc->cmp_s2_end = act == 0 ? rc->cmp_s2_start : rc->cmp_s2_start + (act - 1) / s2base_ + 1;
    rc->cmp_tail = act % s2base_;
  }

  void win_row(RowCache* rc, const Split& sp) const {  // metadata.py:549-584
    const auto& tc = type_cost_;
    if (rc->win_s2_start >= rc->win_s2_end) {
      rc->win_block = 0; rc->win_cost = 0; rc->win_last_block_cost = 0;
      rc->win_normal_block_cost = 0;
      return;
    }
    rc->win_block = rc->win_s2_end - rc->win_s2_start;
    i64 tail = rc->win_tail != 0 ? 1 : 0;
    i64 normal = rc->win_block - tail;
    if (rc->s1g_idx == sp.s1g_num[rc->b_idx] - 1 && sp.s1g_tail[rc->b_idx] != 0) {
      rc->win_cost = tc[WIN_TAIL][WIN_NORMAL] * normal + tc[WIN_TAIL][WIN_TAIL] * tail;
      rc->win_last_block_cost = tail > 0 ? tc[WIN_TAIL][WIN_TAIL] : tc[WIN_TAIL][WIN_NORMAL];
      rc->win_normal_block_cost = tc[WIN_TAIL][WIN_NORMAL];
    } else {
      rc->win_cost = tc[WIN_NORMAL][WIN_NORMAL] * normal + tc[WIN_NORMAL][WIN_TAIL] * tail;
      rc->win_last_block_cost = tail > 0 ? tc[WIN_NORMAL][WIN_TAIL] : tc[WIN_NORMAL][WIN_NORMAL];
      rc->win_normal_block_cost = tc[WIN_NORMAL][WIN_NORMAL];
    }
  }

  void cmp_row(RowCache* rc, const Split& sp) const {  // metadata.py:586-621
    const auto& tc = type_cost_;
    if (rc->cmp_s2_start >= rc->cmp_s2_end) {
      rc->cmp_block = 0; rc->cmp_cost = 0; rc->cmp_last_block_cost = 0;
      rc->cmp_normal_block_cost = 0;
      return;
    }
    rc->cmp_block = rc->cmp_s2_end - rc->cmp_s2_start;
    i64 tail = rc->cmp_tail != 0 ? 1 : 0;
    i64 normal = rc->cmp_block - tail;
    if (rc->s1g_idx == sp.s1g_num[rc->b_idx] - 1 && sp.s1g_tail[rc->b_idx] != 0) {
      rc->cmp_cost = tc[CMP_TAIL][CMP_NORMAL] * normal + tc[CMP_TAIL][CMP_TAIL] * tail;
      rc->cmp_last_block_cost = tail > 0 ? tc[CMP_TAIL][CMP_TAIL] : tc[CMP_TAIL][CMP_NORMAL];
      rc->cmp_normal_block_cost = tc[CMP_TAIL][CMP_NORMAL];
    } else {
      rc->cmp_cost = tc[CMP_NORMAL][CMP_NORMAL] * normal + tc[CMP_NORMAL][CMP_TAIL] * tail;
      rc->cmp_last_block_cost = tail > 0 ? tc[CMP_NORMAL][CMP_TAIL] : tc[CMP_NORMAL][CMP_NORMAL];
      rc->cmp_normal_block_cost = tc[CMP_NORMAL][CMP_NORMAL];
    }
  }

  void row_cache(i64 s1g, const Split& sp, const BatchCache& bc, RowCache* rc) {
    // _calc_s1g_cache, metadata.py:634-667
    if (sp.s1g_num[bc.b_idx] == 0) {
      rc->cost = 0; rc->last_block_cost = 0; rc->win_normal_block_cost = 0;
      rc->win_last_block_cost = 0; rc->cmp_normal_block_cost = 0; rc->cmp_last_block_cost = 0;
      rc->block = 0; rc->s2_start = 0; rc->cmp_s2_start = 0; rc->s2_end = 0;
      return;
    }
    rc->b_idx = bc.b_idx;
    rc->s1g_idx = s1g;
    i128 f, l;
    s2_token_range(s1g, bc, &f, &l);
    block_range(f, l, bc, rc);
    cost_table(mbase_, s2base_, sp.s1g_tail[rc->b_idx], rc->win_tail, rc->cmp_tail);
    win_row(rc, sp);
    cmp_row(rc, sp);
    rc->s2_start = rc->win_block > 0 ? rc->win_s2_start : rc->cmp_s2_start;  // metadata.py:623-632
    if (rc->cmp_block > 0) {
      rc->last_block_cost = rc->cmp_last_block_cost;
      rc->s2_end = rc->cmp_s2_end;
    } else {
      rc->last_block_cost = rc->win_last_block_cost;
      rc->s2_end = rc->win_s2_end;
    }
    rc->block = rc->win_block + rc->cmp_block;
    rc->cost = rc->win_cost + rc->cmp_cost;
  }

  void split_info(Split* sp) {  // metadata.py:671-683
    sp->s1g_num.assign(batch_, 0); sp->s2_num.assign(batch_, 0);
    sp->s1g_tail.assign(batch_, 0); sp->s2_tail.assign(batch_, 0);
    for (i64 b = 0; b < batch_; ++b) {
      i64 s1 = s1_size(b), s2 = s2_size(b);
      sp->s1g_num[b] = pydiv(s1 * group_ + mbase_ - 1, mbase_);
      sp->s1g_tail[b] = pymod(s1 * group_, mbase_);
      sp->s2_num[b] = pydiv(s2 + s2base_ - 1, s2base_);
      sp->s2_tail[b] = pymod(s2, s2base_);
      if (sp->s1g_num[b] != 0 && sp->s2_num[b] != 0) sp->all_zero = false;
    }
  }

  void cost_info(Split* sp) {  // metadata.py:685-714
    sp->bn2_cost.assign(batch_, 0); sp->bn2_block.assign(batch_, 0);
    sp->bn2_last_block_cost.assign(batch_, 0);
    if (sp->all_zero) { sp->total_cost = 0; sp->total_block = 0; return; }
    for (i64 b = 0; b < batch_; ++b) {
      sp->bn2_cost[b] = 0; sp->bn2_block[b] = 0; sp->bn2_last_block_cost[b] = 0;
      if (s1_size(b) != 0 && s2_size(b) != 0) {
        BatchCache bc;
        RowCache rc;
        batch_cache(b, &bc);
        for (i64 r = 0; r < sp->s1g_num[b]; ++r) {
          row_cache(r, *sp, bc, &rc);
          sp->bn2_cost[b] += rc.cost;
          sp->bn2_block[b] += rc.block;
          if (rc.cost > sp->max_row_cost) sp->max_row_cost = rc.cost;
          if (rc.block > 0) sp->bn2_last_block_cost[b] = rc.last_block_cost;
        }
      }
      sp->total_cost += sp->bn2_cost[b] * p_.num_heads_kv;
      sp->total_block += sp->bn2_block[b] * p_.num_heads_kv;
    }
  }

  void by_batch(Split& sp, Assign& a) {  // metadata.py:718-745
    if (a.finished) return;
    while (a.bn2_cost == 0 ||
           within(a.cc.cost_limit, sp.bn2_last_block_cost[a.b] / kToleranceRatio,
                  a.cc.cost + a.bn2_cost)) {
      a.cc.cost += a.bn2_cost;
      a.cc.block += a.bn2_block;
      a.bn2 += 1;
      if (a.bn2 == batch_ * p_.num_heads_kv) {
        a.s1g = 0; a.s2 = 0; a.finished = true;
        return;
      }
      if (a.bn2 / p_.num_heads_kv != a.b) {
        a.b = a.bn2 / p_.num_heads_kv;
        batch_cache(a.b, &a.bc);
      }
      a.bn2_cost = sp.bn2_cost[a.b];
      a.bn2_block = sp.bn2_block[a.b];
      a.s1g = 0;
      row_cache(a.s1g, sp, a.bc, &a.rc);
      a.s2 = a.rc.s2_start;
    }
  }

  bool by_row(Split& sp, Assign& a) {  // metadata.py:747-764
    if (a.finished) return true;
    while (within(a.cc.cost_limit, a.rc.last_block_cost / kToleranceRatio, a.cc.cost + a.rc.cost)) {
      a.cc.cost += a.rc.cost;
      a.cc.block += a.rc.block;
      a.bn2_cost = a.bn2_cost - a.rc.cost > 0 ? a.bn2_cost - a.rc.cost : 0;
      a.bn2_block = a.bn2_block - a.rc.block > 0 ? a.bn2_block - a.rc.block : 0;
      i64 steps = 0;
      while (true) {
        a.s1g += 1;
        row_cache(a.s1g, sp, a.bc, &a.rc);
        if (a.rc.block != 0) break;
        if (++steps > (1LL << 22)) return false;  // reference would spin forever
      }
      a.s2 = a.rc.s2_start;
    }
    return true;
  }

  i64 cur_block_cost(const Assign& a) const {  // metadata.py:766-775
    i64 c;
    if (a.s2 < a.rc.cmp_s2_start) {
      c = a.rc.win_normal_block_cost;
      if (a.s2 == a.rc.cmp_s2_start - 1) c = a.rc.win_last_block_cost;
    } else {
      c = a.rc.cmp_normal_block_cost;
      if (a.s2 == a.rc.s2_end - 1) c = a.rc.cmp_last_block_cost;
    }
    return c;
  }

  void by_block(Split& sp, Assign& a) {  // metadata.py:777-793 (dormant: supportFd=false)
    (void)sp;
    if (a.finished || !kSupportFd) return;
    i64 c = cur_block_cost(a);
    while (within(a.cc.cost_limit, c / kToleranceRatio, a.cc.cost + c)) {
      a.cc.cost += c; a.cc.block += 1; a.s2 += 1;
      a.bn2_cost -= c; a.rc.cost -= c; a.bn2_block -= 1; a.rc.block -= 1;
      c = cur_block_cost(a);
    }
  }

  bool need_record_fd(const Assign& a, const Result& r) const {  // metadata.py:795-805
    if (a.core == 0) return false;
    if (a.kv_split_part <= 1) return false;
    if (a.bn2 == r.bn2_end[a.core - 1] && a.s1g == r.s1g_end[a.core - 1]) return false;
    return true;
  }

  void record_fd(Split& sp, Assign& a, Result& r) {  // metadata.py:807-827
    i64 sb = r.bn2_end[a.core - 1] / p_.num_heads_kv;
    i64 ss = r.s1g_end[a.core - 1];
    i64 s1 = s1_size(sb);
    i64 msize = ss == sp.s1g_num[sb] - 1 ? s1 * group_ - ss * mbase_ : mbase_;
    if (a.kv_split_part > r.max_split) r.max_split = a.kv_split_part;
    i64 h = r.fd_heads;
    r.fd_bn2[h] = r.bn2_end[a.core - 1];
    r.fd_m[h] = r.s1g_end[a.core - 1];
    r.fd_ws[h] = a.fd_data_num - a.kv_split_part;
    r.fd_split[h] = a.kv_split_part;
    r.fd_msize[h] = msize;
    r.fd_heads += 1;
  }

  bool assign_core(Split& sp, Assign& a, Result& r) {  // metadata.py:872-896
    i64 avg = pydiv(a.unassigned, aic_ - a.core > 1 ? aic_ - a.core : 1);
    a.cc = CoreCache();
    a.cc.cost_limit = kSupportFd ? avg : (avg > sp.max_row_cost ? avg : sp.max_row_cost);
    by_batch(sp, a);
    if (!by_row(sp, a)) return false;
    by_block(sp, a);
    // _force_assign (metadata.py:859-870) only runs with supportFd.
    r.bn2_end[a.core] = a.bn2;
    r.s1g_end[a.core] = a.s1g;
    r.s2_end[a.core] = a.s2;
    if (a.cc.cost > r.max_cost) r.max_cost = a.cc.cost;
    a.unassigned -= a.cc.cost;
    if (need_record_fd(a, r)) {
      record_fd(sp, a, r);
      a.kv_split_part = 1;
    }
    if (a.rc.s2_start < a.s2 && a.s2 <= a.rc.s2_end) a.kv_split_part += 1;
    return true;
  }

  bool split_plan(i64 cost_limit, Split& sp, Result& r) {  // metadata.py:898-923
    if (aic_ == 0) return true;
    r.max_cost = 0;
    r.used_cores = 0;
    Assign a;
    a.b = 0;
    a.s1g = 0;
    a.unassigned = sp.total_cost;
    a.bn2_cost = sp.bn2_cost[a.b];
    a.bn2_block = sp.bn2_block[a.b];
    batch_cache(a.b, &a.bc);
    row_cache(a.s1g, sp, a.bc, &a.rc);
    a.s2 = a.rc.s2_start;
    for (i64 i = 0; i < aic_; ++i) {
      if (r.max_cost > cost_limit) return true;
      if (a.finished || a.unassigned <= 0) break;
      a.core = i;
      if (!assign_core(sp, a, r)) return false;
    }
    r.used_cores = a.core + 1;
    return true;
  }

  void split_fd(Result& r) {  // metadata.py:925-954
    i64 total = 0;
    for (i64 i = 0; i < r.fd_heads; ++i) total += r.fd_split[i] * r.fd_msize[i];
    if (aiv_ == 0) return;
    i64 avg = total / aiv_;
    if (avg == 0) return;
    i64 cur = 0;
    for (i64 i = 0; i < r.fd_heads; ++i) {
      i64 nvec = r.fd_split[i] * r.fd_msize[i] / avg;
      if (nvec == 0) continue;
      i64 mavg = r.fd_msize[i] / nvec;
      for (i64 v = 0; v < nvec; ++v) {
        if (cur >= (i64)r.fd_idx.size()) break;
        r.fd_idx[cur] = i;
        r.fd_mstart[cur] = v * mavg;
        r.fd_mnum[cur] = v < nvec - 1 ? mavg : r.fd_msize[i] - v * mavg;
        ++cur;
      }
    }
    r.fd_used_vec = cur;
  }

  int balance(Result& r) {  // metadata.py:956-972
    if (batch_ <= 0) return SAS_ERR_INVALID;
    Split sp;
    split_info(&sp);
    if (sp.all_zero) {
      r.used_cores = 1;
      if (aic_ > 0) {
        r.bn2_end[0] = batch_ * p_.num_heads_kv;
        r.s1g_end[0] = 0;
        r.s2_end[0] = 0;
      }
      return SAS_OK;
    }
    cost_info(&sp);
    r.max_cost = kInt64Max;
    r.used_cores = 1;
    if (!split_plan(r.max_cost, sp, r)) return SAS_ERR_SCHEDULE;
    if (r.fd_heads > 0) split_fd(r);
    if (r.used_cores < 1) r.used_cores = 1;
    return SAS_OK;
  }

  void emit(const Result& r, int32_t* out) const {  // metadata.py:974-1009
    std::memset(out, 0, sizeof(int32_t) * SAS_META_SIZE);
    for (i64 i = 0; i < SAS_AIC_CORE_NUM; ++i) {
      int32_t* row = out + i * SAS_FA_METADATA_SIZE;
      if (i >= r.used_cores || i >= aic_) continue;
      row[0] = 1;
      row[1] = (int32_t)(i == 0 ? 0 : r.bn2_end[i - 1]);
      row[2] = (int32_t)(i == 0 ? 0 : r.s1g_end[i - 1]);
      row[3] = (int32_t)(i == 0 ? 0 : r.s2_end[i - 1]);
      row[4] = (int32_t)r.bn2_end[i];
      row[5] = (int32_t)r.s1g_end[i];
      row[6] = (int32_t)r.s2_end[i];
      row[7] = (int32_t)r.first_fd_ws[i];
    }
    int32_t* fd = out + SAS_AIC_CORE_NUM * SAS_FA_METADATA_SIZE;
    for (i64 i = 0; i < SAS_AIV_CORE_NUM; ++i) {
      int32_t* row = fd + i * SAS_FD_METADATA_SIZE;
      if (i >= r.fd_used_vec || i >= aiv_) continue;
      i64 f = r.fd_idx[i];
      row[0] = 1;
      row[1] = (int32_t)r.fd_bn2[f];
      row[2] = (int32_t)r.fd_m[f];
      row[3] = (int32_t)r.fd_ws[f];
      row[4] = (int32_t)r.fd_split[f];
      row[5] = (int32_t)r.fd_mstart[i];
      row[6] = (int32_t)r.fd_mnum[i];
    }
  }
};

}  // namespace

extern "C" int sas_metadata(const SasMetaParams* params, int32_t* out, size_t out_len) {
  if (params == nullptr || out == nullptr) return SAS_ERR_INVALID;
  if (out_len < (size_t)SAS_META_SIZE) return SAS_ERR_INVALID;
  const SasMetaParams& p = *params;
  if (p.aic_core_num < 0 || p.aiv_core_num < 0 || p.num_heads_q < 0 || p.num_heads_kv < 0)
    return SAS_ERR_INVALID;
  if (p.num_heads_kv == 0) return SAS_ERR_INVALID;  // the reference divides by it
  if (p.num_heads_q / p.num_heads_kv == 0) return SAS_ERR_INVALID;
  if ((p.n_seqused_q > 0 && p.seqused_q == nullptr) ||
      (p.n_seqused_kv > 0 && p.seqused_kv == nullptr) ||
      (p.n_cu_seqlens_q > 0 && p.cu_seqlens_q == nullptr) ||
      (p.n_cu_seqlens_ori_kv > 0 && p.cu_seqlens_ori_kv == nullptr))
    return SAS_ERR_INVALID;
  // Every batch index the scheduler reads must be backed by the arrays (the
  // reference raises IndexError in these cases).
  int64_t qb = p.n_seqused_q > 0 ? p.n_seqused_q
               : (p.layout_q == SAS_LAYOUT_TND && p.n_cu_seqlens_q > 0 ? p.n_cu_seqlens_q - 1
                                                                        : p.batch_size);
  if (qb < 0) return SAS_ERR_INVALID;
  if (p.n_seqused_kv > 0 && p.n_seqused_kv < qb) return SAS_ERR_INVALID;
  if (p.n_seqused_kv == 0 && p.layout_kv == SAS_LAYOUT_TND && p.n_cu_seqlens_ori_kv > 0 &&
      p.n_cu_seqlens_ori_kv < qb + 1)
    return SAS_ERR_INVALID;
  Scheduler s(p);
  return s.run(out);
}
