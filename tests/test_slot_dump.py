"""Index handling of the kernels themselves, compared exactly on the GPU.

Every forward can record, per query row and key slot, the key source its
producer warps resolved (``SasFwdParams.slot_dump``): the pool row and cache
of each attended slot, ``-2 - cache`` for an attended position whose page is
unmapped (read as a zero row), ``-1`` for a masked slot.  This test checks
that record against a restatement of the reference's index rules
(golden.py:28-66 for the top-k branch: scan the first min(K, threshold)
entries, stop at the first -1, skip ids that are negative or at / past the
causal threshold; golden.py:125-150 for the window and the dense compressed
branch) mapped through the block tables — slot for slot, bit-exact.

Cases cover dirty indices (-1 in the middle, out-of-range, duplicates and
other negatives), unmapped pages, split rows (forced worker counts), ring
rows (one head group, 65..128-key windows: checked as a set, since ring
slots hold the window in ring order), the dense compressed branch, D = 512,
and both the one-CTA kernel (<= 64 heads) and the CTA-pair kernel (65..128
heads)."""

import ctypes as C

import numpy as np
import pytest
import torch

from oracle import sas_oracle as O
from sparse_attn_sharedkv_b200 import _lib
from sparse_attn_sharedkv_b200.api import build_call
from tests import workloads as W

pytestmark = pytest.mark.gpu

UNSET = -7  # never written by the kernels


def _slots_expected(case: W.Case):
    """{flat token: (list of per-slot values in golden order, ring?)}."""
    B = case.batch
    H = case.q.shape[-2]
    scen = 1 if case.cmp_kv is None else (3 if case.cmp_sparse_indices is not None else 2)
    ratio = case.cmp_ratio or 4
    wl = case.ori_win_left
    ori_bs = case.ori_kv.shape[1]
    ori_t = case.ori_block_table.cpu().numpy()
    cmp_bs = case.cmp_kv.shape[1] if case.cmp_kv is not None else 1
    cmp_t = case.cmp_block_table.cpu().numpy() if case.cmp_block_table is not None else None
    if case.layout_q == "TND":
        cu = case.cu_seqlens_q.tolist()
        starts, lens = cu[:-1], [cu[i + 1] - cu[i] for i in range(B)]
    else:
        S = case.q.shape[1]
        starts = [b * S for b in range(B)]
        lens = ([int(x) for x in (case.cu_seqlens_q[1:] - case.cu_seqlens_q[:-1])]
                if case.cu_seqlens_q is not None else [S] * B)
    idx = None
    if scen == 3:
        idx = case.cmp_sparse_indices.reshape(-1, case.cmp_sparse_indices.shape[-1]).numpy()

    def src(table, bs, b, pos, cache):
        lb = pos // bs
        blk = int(table[b, lb]) if lb < table.shape[1] else -1
        return 2 * (blk * bs + pos % bs) + cache if blk >= 0 else -2 - cache

    ring = scen == 1 and 64 <= wl < 128 and H <= 64
    out = {}
    for b in range(B):
        akv = int(case.seqused_kv[b])
        for s in range(lens[b]):
            t = starts[b] + s
            lo, hi = O.window_positions(akv, lens[b], s, wl)
            vals = [src(ori_t, ori_bs, b, p, 0) for p in range(lo, hi)]
            if scen == 2:
                thr = O.cmp_threshold(akv, lens[b], s, ratio)
                vals += [src(cmp_t, cmp_bs, b, c, 1) for c in range(max(thr, 0))]
            elif scen == 3:
                thr = O.cmp_threshold(akv, lens[b], s, ratio)
                stopped = False
                for c in range(max(min(idx.shape[1], thr), 0)):
                    tid = int(idx[t, c])
                    if tid == -1:
                        stopped = True
                    ok = (not stopped) and 0 <= tid < thr
                    vals.append(src(cmp_t, cmp_bs, b, tid, 1) if ok else -1)
            out[t] = (vals, ring and hi > lo)
    return out


def _run_dump(case: W.Case, num_sms=None):
    c = case.to("cuda")
    call = build_call(c.q, num_sms=num_sms, **c.kwargs())
    T = call.total
    K = c.cmp_sparse_indices.shape[-1] if c.cmp_sparse_indices is not None else 0
    cap = 128 + max(K, 0) + 4 * 64
    if c.cmp_kv is not None and c.cmp_sparse_indices is None:
        cap += int(c.seqused_kv.max()) // (c.cmp_ratio or 4)
    dump = torch.full((T, cap), UNSET, dtype=torch.int32, device="cuda")
    call.fp.slot_dump = dump.data_ptr()
    call.fp.slot_dump_cap = cap
    L = _lib.lib()
    n = C.c_size_t(0)
    _lib.check("ws", L.sas_fwd_workspace_size(C.byref(call.prob), call.fp.num_sms, C.byref(n)))
    ws = torch.empty(max(n.value, 256), dtype=torch.uint8, device="cuda")
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    call.fp.err = err.data_ptr()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check("sas_fwd", L.sas_fwd(C.byref(call.prob), C.byref(call.fp), ws.data_ptr(),
                                    n.value, stream))
    torch.cuda.synchronize()
    assert err.tolist()[0] == 0, err.tolist()
    return dump.cpu().numpy()


def _unmap_page(case: W.Case, b: int, logical_block: int) -> W.Case:
    """The same case with one page of batch b's window table unmapped (-1)."""
    t = case.ori_block_table.clone()
    t[b, logical_block] = -1
    case.ori_block_table = t
    if case.cmp_kv is case.ori_kv or (case.cmp_block_table is not None and
                                      case.cmp_block_table.data_ptr() ==
                                      case.ori_block_table.data_ptr()):
        case.cmp_block_table = t
    return case


CASES = [
    # top-k with dirty indices (one CTA per 64 heads / CTA pair for 128)
    (dict(seed=401, layout_q="TND", H=64, scenario=3, idx_mode="dirty", K=200, q_lens=(5, 3),
          kv_lens=(900, 700)), None, None),
    (dict(seed=402, layout_q="TND", H=128, scenario=3, idx_mode="dirty", K=200,
          q_lens=(5, 3), kv_lens=(900, 700)), None, None),
    # split rows: few workers, long rows
    (dict(seed=403, layout_q="BSND", B=2, H=128, scenario=3, idx_mode="dirty", K=700,
          q_lens=(1, 1), kv_lens=(3000, 2500), ratio=1, win_left=-1), 5, None),
    (dict(seed=404, layout_q="TND", H=64, scenario=3, idx_mode="dirty", K=700, q_lens=(2, 3),
          kv_lens=(3000, 2500)), 37, None),
    # unmapped page inside the window
    (dict(seed=405, layout_q="TND", H=64, scenario=3, K=96, q_lens=(4, 3),
          kv_lens=(600, 400)), None, (0, 8)),
    (dict(seed=406, layout_q="TND", H=128, scenario=3, K=96, q_lens=(4, 3),
          kv_lens=(600, 400)), None, (1, 5)),
    # dense compressed branch
    (dict(seed=407, layout_q="TND", H=128, scenario=2, ratio=8, q_lens=(6, 2),
          kv_lens=(1400, 600)), None, None),
    (dict(seed=408, layout_q="TND", H=64, scenario=2, ratio=8, q_lens=(6, 2),
          kv_lens=(1400, 600)), 7, None),
    # sliding windows: ring rows (64 heads) and plain windows (128 heads)
    (dict(seed=409, layout_q="TND", H=64, scenario=1, q_lens=(70, 3), kv_lens=(300, 3)),
     None, None),
    (dict(seed=410, layout_q="TND", H=128, scenario=1, q_lens=(70, 3), kv_lens=(300, 3)),
     None, None),
    (dict(seed=411, layout_q="BSND", B=2, H=64, scenario=1, win_left=100, q_lens=(5, 9),
          kv_lens=(700, 9)), 3, None),
    # d_qk 512 and BSND padding
    (dict(seed=412, layout_q="BSND", B=2, H=96, D=512, d_v=None, scenario=3, K=128,
          q_lens=(3, 1), kv_lens=(700, 900)), None, None),
    # short windows: the 4-row group at the window / compressed boundary mixes the caches
    (dict(seed=413, layout_q="TND", H=128, scenario=3, K=32, q_lens=(3, 2),
          kv_lens=(31, 45)), None, None),
    (dict(seed=414, layout_q="TND", H=64, scenario=3, K=32, q_lens=(3, 2),
          kv_lens=(31, 45)), None, None),
]


@pytest.mark.parametrize("kw,sms,unmap", CASES)
def test_kernel_slot_sources_match_golden_rules(kw, sms, unmap):
    case = W.random_case(**kw)
    if unmap is not None:
        case = _unmap_page(case, *unmap)
    dump = _run_dump(case, sms)
    exp = _slots_expected(case)
    assert exp, "case has no query rows"
    checked_unmapped = 0
    for t, (vals, ring) in exp.items():
        got = dump[t]
        if ring:
            # ring slots: the 128 ring entries hold the window in ring order
            ring_got = sorted(int(v) for v in got[:128] if v != -1)
            assert ring_got == sorted(vals), t
        else:
            n = len(vals)
            assert list(got[:n]) == vals, (t, [(i, int(got[i]), vals[i]) for i in range(n)
                                                if got[i] != vals[i]][:5])
        checked_unmapped += sum(1 for v in vals if v <= -2)
    if unmap is not None:
        assert checked_unmapped > 0
