"""The B200 work plan (``sas_plan``) and the kernel's slot logic, on CPU.

* coverage: every (row, tile) unit of every query row is owned by exactly one
  worker, worker spans are contiguous, split rows get unique partial slots;
* slot semantics: a Python mirror of the producer warps' per-tile slot ->
  (cache, position) mapping, including the ``-1`` stop prefix carried across
  tiles and pieces, reproduces the oracle's attended key list
  (golden.py:28-66 via ``oracle.sas_oracle``).
"""

import ctypes as C

import numpy as np
import pytest
import torch

from oracle import sas_oracle as O
from sparse_attn_sharedkv_b200 import _lib
from tests import workloads as W

HDR = dict(magic=0, rows=1, workers=2, hg=3, nsplit=4, npart=5, rows_off=6, workers_off=7,
           split_off=8, total=9, batch=10, actq_off=11, actkv_off=12)


def make_problem(layout, q_start, q_len, kv_len, H, scenario, win_left, ratio, topk, S=0,
                 total=None):
    p = _lib.SasProblem()
    p.batch = len(q_len)
    p.layout_q = _lib.LAYOUTS[layout]
    p.max_q_len = S
    p.total_tokens = total if total is not None else (sum(q_len) if layout == "TND"
                                                      else S * len(q_len))
    keep = [(C.c_int32 * len(v))(*v) for v in (q_start, q_len, kv_len)]
    p.q_start, p.q_len, p.kv_len = [C.cast(k, C.POINTER(C.c_int32)) for k in keep]
    p.num_heads, p.scenario, p.ori_win_left = H, scenario, win_left
    p.cmp_ratio, p.topk = ratio, topk
    return p, keep


def build_plan(p, sms):
    info = _lib.SasPlanInfo()
    L = _lib.lib()
    _lib.check("sas_plan_size", L.sas_plan_size(C.byref(p), sms, C.byref(info)))
    buf = (C.c_int32 * info.plan_ints)()
    _lib.check("sas_plan", L.sas_plan(C.byref(p), sms, buf, info.plan_ints, C.byref(info)))
    return np.frombuffer(buf, dtype=np.int32).copy(), info


ROW_INTS = 12  # token, b, s, slots, flags, first_worker, partial_base, window, win_lo, cmp, thr, pad
RING = 2  # flags bit: pure sliding window kept as a 128-position ring (two tiles)


def rows_of(plan):
    n = plan[HDR["rows"]]
    off = plan[HDR["rows_off"]]
    return plan[off: off + ROW_INTS * n].reshape(n, ROW_INTS)


def segments(plan):
    """Yield (worker, row, ja, jb) exactly like the kernel's span walk."""
    rows = rows_of(plan)
    nw = plan[HDR["workers"]]
    woff = plan[HDR["workers_off"]]
    for w in range(nw):
        r0, t0, r1, t1, piece0 = plan[woff + 8 * w: woff + 8 * w + 5]
        if r0 < 0:
            continue
        for r in range(r0, r1 + 1):
            tiles = (rows[r][3] + 63) // 64
            ja = t0 if r == r0 else 0
            jb = t1 if r == r1 else max(tiles, 1)
            if ja < jb:
                yield w, r, ja, jb, (piece0 if r == r0 else 0)


CASES = [
    ("TND", [0, 5], [5, 3], [300, 700], 64, 3, 127, 4, 96, 0),
    ("TND", [0, 5], [5, 3], [300, 700], 128, 1, 127, 4, 0, 0),
    ("BSND", [0, 6], [4, 6], [400, 520], 64, 3, 127, 4, 48, 6),
    ("BSND", [0, 1, 2, 3], [1, 1, 1, 1], [9000, 20000, 8192, 32768], 128, 3, -1, 1, 2048, 1),
    ("TND", [0, 4096], [4096, 4096], [4096, 4096], 128, 3, -1, 1, 2048, 0),
    ("TND", [0, 1], [1, 0], [5, 7], 16, 2, 127, 16, 0, 0),
]


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("sms", [1, 7, 148])
def test_plan_covers_every_tile_once(case, sms):
    layout, qs, ql, kvl, H, scen, wl, ratio, K, S = case
    p, keep = make_problem(layout, qs, ql, kvl, H, scen, wl, ratio, K, S)
    plan, info = build_plan(p, sms)
    assert plan[0] == 0x53415331
    rows = rows_of(plan)
    hg = (H + 63) // 64
    assert info.head_groups == hg and info.num_workers == max(1, sms // hg)
    seen = {}
    pieces = {}
    for w, r, ja, jb, piece in segments(plan):
        for j in range(ja, jb):
            assert (r, j) not in seen
            seen[(r, j)] = w
        pieces.setdefault(r, []).append((w, piece))
        if hg == 2:
            # the CTA-pair kernel walks 128-key pair tiles: pieces are cut at
            # whole pairs (even first tile; even end tile unless the row ends)
            tiles_r = max((rows[r][3] + 63) // 64, 1)
            assert ja % 2 == 0 and (jb % 2 == 0 or jb == tiles_r), (r, ja, jb)
    for r, row in enumerate(rows):
        units = max((row[3] + 63) // 64, 1)
        assert all((r, j) in seen for j in range(units)), r
        ws = [w for w, _ in pieces[r]]
        assert ws == sorted(ws) and len(set(ws)) == len(ws)
        if units <= 4:
            assert len(ws) == 1, r  # rows of at most 4 tiles run whole on one worker
        assert [pc for _, pc in pieces[r]] == list(range(len(ws)))  # piece ordinals
        assert row[5] == ws[0]
        if len(ws) > 1:
            assert row[6] >= 0
        else:
            assert row[6] == -1
    bases = [row[6] + k for row in rows if row[6] >= 0
             for k in range(len(pieces[list(rows[:, 0]).index(row[0])]))]
    assert sorted(bases) == list(range(info.num_partials))
    # batch section
    B = plan[HDR["batch"]]
    assert list(plan[plan[HDR["actq_off"]]: plan[HDR["actq_off"]] + B]) == ql
    assert list(plan[plan[HDR["actkv_off"]]: plan[HDR["actkv_off"]] + B]) == kvl


def kernel_slot_positions(case, plan):
    """Mirror of the producer warps: per (row, piece) the attended
    (branch, logical position) list in slot order."""
    rows = rows_of(plan)
    cu_start = {}
    out = {}
    qlen = case.cu_seqlens_q
    idx = case.cmp_sparse_indices
    if idx is not None:
        idx = idx.reshape(-1, idx.shape[-1]).numpy()
    K = idx.shape[1] if idx is not None else 0
    for w, r, ja, jb, piece in segments(plan):
        t, b, s, slots, flags, _, _, Wn, row_lo, row_cmp, row_thr, _ = rows[r]
        if flags & 1 or slots == 0:
            continue
        aq = int(case.meta["q_len"][b])
        akv = int(case.seqused_kv[b])
        scen = case.meta["scenario"]
        s_g = akv - aq + s
        lo = max(s_g - case.ori_win_left, 0)
        thr = (akv - aq + s + 1) // case.cmp_ratio if scen >= 2 else 0
        ncmp = min(max(thr, 0), K) if scen == 3 else max(thr, 0)
        # the key bounds the planner precomputes for the kernel
        assert (row_lo, row_cmp, row_thr) == (lo, ncmp, thr), (r, row_lo, row_cmp, row_thr)
        stopped = False
        if scen == 3 and ja > 0:
            lim = min(ja * 64 - Wn, ncmp)
            stopped = any(idx[t, c] == -1 for c in range(max(lim, 0)))
        got = out.setdefault(r, [])
        if flags & RING:
            assert scen == 1 and slots == 128 and 64 <= case.ori_win_left < 128 and Wn > 0
            if (ja, jb) == (0, 2):
                # ring slot (half, row) holds position p = 64 half + row (mod 128)
                # of [hi - 127, hi]; attended when p >= lo
                hi = row_lo + Wn - 1
                for i in range(128):
                    p = hi - ((hi - i) % 128)
                    if p >= row_lo:
                        got.append(("ori", p))
                continue
        for j in range(ja, jb):
            m1 = 0
            if scen == 3:
                for key in range(64):
                    c = j * 64 + key - Wn
                    if 0 <= c < ncmp and idx[t, c] == -1:
                        m1 |= 1 << key
            for key in range(64):
                slot = j * 64 + key
                if slot < Wn:
                    got.append(("ori", lo + slot))
                elif slot < Wn + row_cmp:
                    c = slot - Wn
                    if scen == 3:
                        pos = int(idx[t, c])
                        before = stopped or (m1 & ((1 << key) - 1)) != 0
                        if not before and 0 <= pos < thr:
                            got.append(("cmp", pos))
                    else:
                        got.append(("cmp", c))
            if m1:
                stopped = True
    return out


SLOT_CASES = [
    dict(seed=1, layout_q="TND", scenario=3, idx_mode="dirty", K=200, q_lens=(5, 3),
         kv_lens=(900, 700)),
    dict(seed=2, layout_q="TND", scenario=3, idx_mode="perm", K=96),
    dict(seed=3, layout_q="BSND", B=2, scenario=3, idx_mode="dirty", K=300, q_lens=(3, 2),
         kv_lens=(1300, 1500)),
    dict(seed=4, layout_q="TND", scenario=2, ratio=8, q_lens=(6, 2), kv_lens=(1400, 600)),
    dict(seed=5, layout_q="TND", scenario=1, q_lens=(70, 3), kv_lens=(100, 3)),
    dict(seed=7, layout_q="TND", scenario=1, q_lens=(300, 2, 64), kv_lens=(1000, 130, 64)),
    dict(seed=8, layout_q="BSND", B=2, scenario=1, win_left=100, q_lens=(5, 9),
         kv_lens=(700, 9)),
    dict(seed=9, layout_q="TND", scenario=1, win_left=300, q_lens=(40, 3), kv_lens=(900, 50)),
    dict(seed=6, layout_q="TND", scenario=3, ratio=1, win_left=-1, K=256, idx_mode="dirty",
         q_lens=(4, 4), kv_lens=(600, 300)),
]


@pytest.mark.parametrize("kw", SLOT_CASES)
@pytest.mark.parametrize("sms", [3, 64])
def test_kernel_slot_logic_matches_oracle(kw, sms):
    case = W.random_case(**kw)
    B = case.batch
    if case.layout_q == "TND":
        cu = case.cu_seqlens_q.tolist()
        qs, ql, S = cu[:-1], [cu[i + 1] - cu[i] for i in range(B)], 0
    else:
        S = case.q.shape[1]
        qs = [b * S for b in range(B)]
        ql = ([int(x) for x in (case.cu_seqlens_q[1:] - case.cu_seqlens_q[:-1])]
              if case.cu_seqlens_q is not None else [S] * B)
    case.meta["q_len"] = ql
    H = case.q.shape[-2]
    scen = case.meta["scenario"]
    K = case.cmp_sparse_indices.shape[-1] if case.cmp_sparse_indices is not None else 0
    p, keep = make_problem(case.layout_q, qs, ql, case.seqused_kv.tolist(), H, scen,
                           case.ori_win_left, case.cmp_ratio or 4, K, S)
    plan, _ = build_plan(p, sms)
    got = kernel_slot_positions(case, plan)
    rows = rows_of(plan)
    idx = (case.cmp_sparse_indices.reshape(-1, K).numpy() if K else None)
    for r, row in enumerate(rows):
        t, b, s = row[0], row[1], row[2]
        if row[4] & 1:
            continue
        aq, akv = ql[b], int(case.seqused_kv[b])
        lo, hi = O.window_positions(akv, aq, s, case.ori_win_left)
        exp = [("ori", x) for x in range(lo, hi)]
        if scen == 3:
            exp += [("cmp", x) for x in O.scfa_positions(idx[t], akv, aq, s, case.cmp_ratio)]
        elif scen == 2:
            exp += [("cmp", x) for x in range(max(O.cmp_threshold(akv, aq, s, case.cmp_ratio), 0))]
        if row[4] & RING:
            assert sorted(got.get(r, [])) == sorted(exp), (r, t)
        else:
            assert got.get(r, []) == exp, (r, t)


# Decode rows of exactly 4 key tiles (256 keys: kept whole) and 5 tiles
# (257..320 keys: cut at tile granularity) side by side.
SNAP_KV = [256, 257, 256, 320, 193, 257, 256, 300, 256, 256, 257, 320]


def _snap_problem():
    B = len(SNAP_KV)
    return make_problem("BSND", list(range(B)), [1] * B, SNAP_KV, 64, 3, -1, 1, 512, 1)


@pytest.mark.parametrize("sms", range(2, 30))
def test_short_rows_whole_next_to_worker_boundaries(sms):
    p, keep = _snap_problem()
    plan, info = build_plan(p, sms)
    rows = rows_of(plan)
    owners = {}
    for w, r, ja, jb, piece in segments(plan):
        owners.setdefault(r, []).append(w)
    for r, row in enumerate(rows):
        if (row[3] + 63) // 64 <= 4:
            assert len(owners[r]) == 1, (sms, r)


def test_snap_sweep_exercises_both_sides_of_the_rule():
    """Across the worker counts above, some worker boundary falls inside a
    4-tile row (kept whole) and some 5-tile row is split (cut as usual)."""
    p, keep = _snap_problem()
    cut4 = split5 = False
    for sms in range(2, 30):
        plan, info = build_plan(p, sms)
        starts = np.cumsum([0] + [1 + (k + 63) // 64 for k in SNAP_KV])
        total = starts[-1]
        bounds = [total * w / sms for w in range(1, sms)]
        for r, k in enumerate(SNAP_KV):
            tiles = (k + 63) // 64
            inside = any(starts[r] < x < starts[r + 1] for x in bounds)
            if tiles == 4 and inside:
                cut4 = True
        owners = {}
        for w, r, ja, jb, piece in segments(plan):
            owners.setdefault(r, []).append(w)
        split5 |= any(len(v) > 1 and (SNAP_KV[r] + 63) // 64 == 5 for r, v in owners.items())
    assert cut4 and split5


def test_plan_rejects_bad_problems():
    p, keep = make_problem("TND", [0], [1], [5], 200, 1, 127, 4, 0)
    info = _lib.SasPlanInfo()
    assert _lib.lib().sas_plan_size(C.byref(p), 148, C.byref(info)) == 1
    p, keep = make_problem("TND", [0], [4], [5], 64, 3, 127, 4, 0)  # SCFA without K
    assert _lib.lib().sas_plan_size(C.byref(p), 148, C.byref(info)) == 1
    p, keep = make_problem("TND", [0], [4], [5], 64, 1, 127, 4, 0, total=2)  # rows overflow
    assert _lib.lib().sas_plan_size(C.byref(p), 148, C.byref(info)) == 1
