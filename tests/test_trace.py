"""The diagnostic clock trace (``SasFwdParams.trace``) of both attention kernels.

A forward launched with a trace buffer runs the trace instance of the
kernel.  It must give bit-identical outputs to the untraced launch, record
every CTA's start and end, and keep each event stream inside its own
sub-range of the 4 x 8192 buffer: the events of the traced CTA are ordered
as the pipeline orders them (a tile's QK starts before it is issued, its
chunk groups are seen in order, P is written after the S of the tile is
seen) and entries past a stream's capacity stay unwritten.  The one-CTA
kernel is traced on 16 and 128 heads (SAS_FWD_KERNEL=single), the CTA-pair
kernel (the default for 65..128 heads) on 128."""

import ctypes as C

import numpy as np
import pytest
import torch

from sparse_attn_sharedkv_b200 import _lib
from sparse_attn_sharedkv_b200.api import build_call
from tests import workloads as W

pytestmark = pytest.mark.gpu

REGION = 8192


def _launch(call, trace=None):
    L = _lib.lib()
    n = C.c_size_t(0)
    _lib.check("ws", L.sas_fwd_workspace_size(C.byref(call.prob), call.fp.num_sms, C.byref(n)))
    ws = torch.empty(max(n.value, 256), dtype=torch.uint8, device="cuda")
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    call.fp.err = err.data_ptr()
    call.fp.trace = trace.data_ptr() if trace is not None else None
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check("sas_fwd", L.sas_fwd(C.byref(call.prob), C.byref(call.fp), ws.data_ptr(),
                                    n.value, stream))
    torch.cuda.synchronize()
    assert err.tolist()[0] == 0, err.tolist()


# (benchmark config, workers): few workers, so the traced CTA 0 owns tiles
@pytest.mark.parametrize("cfg,sms", [(0, 4), (2, 16)])
def test_trace_instance_matches_and_records_in_order(cfg, sms, monkeypatch):
    monkeypatch.setenv("SAS_FWD_KERNEL", "single")
    monkeypatch.setenv("SAS_TRACE_CTA", "0")
    case = W.baseline_case(cfg, device="cuda", scale_down=1 if cfg == 0 else 4)
    call = build_call(case.q, num_sms=sms, **case.kwargs())
    _launch(call)
    out_ref, lse_ref = call.out.clone(), call.lse.clone()
    tr = torch.zeros(4 * REGION, dtype=torch.int64, device="cuda")
    _launch(call, tr)
    assert torch.equal(call.out, out_ref)
    assert torch.equal(call.lse, lse_ref)

    t = tr.cpu().numpy().reshape(4, REGION)
    workers, groups_per_worker = _plan_shape(call)
    grid = workers * groups_per_worker
    spans = t[2][6144:8192].reshape(-1, 2)[:grid]
    assert (spans[:, 0] > 0).all() and (spans[:, 1] >= spans[:, 0]).all()

    mma, smx, r3 = t[1], t[2], t[3]
    tiles = int((mma[0:REGION:4] > 0).sum())
    assert tiles > 0
    n = min(tiles, 600)
    qk_start, qk_end = mma[0:4 * n:4], mma[1:4 * n:4]
    assert (qk_end >= qk_start).all()
    groups = r3[2048:2048 + 3 * n].reshape(n, 3)
    assert (np.diff(groups, axis=1) >= 0).all()
    assert (groups[:, 0] >= qk_start).all() and (groups[:, 2] <= qk_end).all()
    s_seen, p_done = smx[3:4 * n:4], smx[2:4 * n:4]
    assert (p_done >= s_seen).all()
    # entries past the softmax stream's 6144 slots hold only CTA spans
    assert (t[2][2 * grid + 6144:] == 0).all()


def test_pair_trace_instance_matches_and_records_in_order(monkeypatch):
    monkeypatch.delenv("SAS_FWD_KERNEL", raising=False)
    monkeypatch.setenv("SAS_TRACE_CTA", "0")
    case = W.baseline_case(2, device="cuda", scale_down=4)  # 128 heads: the pair kernel
    call = build_call(case.q, num_sms=16, **case.kwargs())
    _launch(call)
    out_ref, lse_ref = call.out.clone(), call.lse.clone()
    tr = torch.zeros(4 * REGION, dtype=torch.int64, device="cuda")
    _launch(call, tr)
    assert torch.equal(call.out, out_ref)
    assert torch.equal(call.lse, lse_ref)

    t = tr.cpu().numpy().reshape(4, REGION)
    workers, groups_per_worker = _plan_shape(call)
    grid = workers * groups_per_worker  # two CTAs per worker
    spans = t[2][6144:8192].reshape(-1, 2)[:grid]
    assert (spans[:, 0] > 0).all() and (spans[:, 1] >= spans[:, 0]).all()

    prod, mma, smx, r3 = t
    tiles = int((mma[0:4000:4] > 0).sum())
    assert tiles > 0
    n = min(tiles, 900)
    qk_start, qk_end = mma[0:4 * n:4], mma[1:4 * n:4]
    pv_end = mma[3:4 * n:4]
    assert (qk_end >= qk_start).all()
    groups = r3[0:3 * n].reshape(n, 3)
    assert (np.diff(groups, axis=1) >= 0).all()
    assert (groups[:, 0] >= qk_start).all() and (groups[:, 2] <= qk_end).all()
    # producer: stage wait <= stage free <= rows issued
    p3 = prod[0:3 * n].reshape(n, 3)
    assert (np.diff(p3, axis=1) >= 0).all()
    # softmax: S seen <= maximum exchanged <= P written <= released
    s4 = smx[0:4 * n].reshape(n, 4)
    assert (np.diff(s4, axis=1) >= 0).all()
    # PV(t): V seen, then P seen (after this CTA wrote P(t)), then issued
    v_seen, p_seen = r3[4096:4096 + 2 * n:2], r3[4097:4097 + 2 * n:2]
    assert (p_seen >= v_seen).all() and (pv_end >= p_seen).all()
    assert (p_seen >= s4[:, 2]).all()
    # the V gather of tile t follows QK(t): seen complete after QK(t) was issued
    assert (r3[6144:6144 + n] >= qk_end).all()
    # nothing between the softmax streams and the CTA spans
    assert (t[2][6000:6144] == 0).all()


def _plan_shape(call):
    """(workers, CTAs per worker) of the call's plan: the launch grid."""
    info = _lib.SasPlanInfo()
    L = _lib.lib()
    _lib.check("plan", L.sas_plan_size(C.byref(call.prob), call.fp.num_sms, C.byref(info)))
    return int(info.num_workers), int(info.head_groups)
