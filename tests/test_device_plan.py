"""Device-built work plan (sas_fwd_prepare_device): the same plan as the host
planner, the same outputs bit for bit, no host read of the lengths (the call
is recorded in a CUDA graph and replayed with new lengths), and invalid
lengths reported through the error word."""

import ctypes as C

import numpy as np
import pytest
import torch

from sparse_attn_sharedkv_b200 import _lib
from tests import workloads as W
from sparse_attn_sharedkv_b200.api import build_call, sparse_attn_sharedkv

pytestmark = pytest.mark.gpu

ROW_INTS, WORKER_INTS = 12, 8
H = dict(rows=1, workers=2, nsplit=4, npart=5, rows_off=6, workers_off=7, split_off=8,
         batch=10, actq_off=11, actkv_off=12)


def _sections(plan):
    R, nw, ns = plan[H["rows"]], plan[H["workers"]], plan[H["nsplit"]]
    rows = plan[plan[H["rows_off"]]: plan[H["rows_off"]] + R * ROW_INTS].reshape(R, ROW_INTS)
    workers = plan[plan[H["workers_off"]]: plan[H["workers_off"]] + nw * WORKER_INTS]
    split = plan[plan[H["split_off"]]: plan[H["split_off"]] + ns * 4]
    B = plan[H["batch"]]
    acts = (plan[plan[H["actq_off"]]: plan[H["actq_off"]] + B],
            plan[plan[H["actkv_off"]]: plan[H["actkv_off"]] + B])
    return dict(rows=rows, workers=workers.reshape(nw, WORKER_INTS), split=split.reshape(ns, 4),
                counts=(R, nw, ns, plan[H["npart"]]), acts=acts)


def _host_plan(case, num_sms):
    c = case.to("cuda")
    call = build_call(c.q, num_sms=num_sms, **c.kwargs())
    info = _lib.SasPlanInfo()
    L = _lib.lib()
    _lib.check("sas_plan_size", L.sas_plan_size(C.byref(call.prob), num_sms, C.byref(info)))
    buf = (C.c_int32 * info.plan_ints)()
    _lib.check("sas_plan", L.sas_plan(C.byref(call.prob), num_sms, buf, info.plan_ints,
                                      C.byref(info)))
    return np.frombuffer(buf, dtype=np.int32).copy()


def _device_plan(case, num_sms, err=None):
    c = case.to("cuda")
    call = build_call(c.q, num_sms=num_sms, device_plan=True, err=err, **c.kwargs())
    L = _lib.lib()
    n = C.c_size_t(0)
    _lib.check("ws", L.sas_fwd_workspace_size_device(C.byref(call.prob), num_sms, C.byref(n)))
    ws = torch.zeros(n.value, dtype=torch.uint8, device="cuda")
    info = _lib.SasPlanInfo()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check("prep", L.sas_fwd_prepare_device(C.byref(call.prob), C.byref(call.fp),
                                                ws.data_ptr(), n.value, stream, C.byref(info)))
    torch.cuda.synchronize()
    return ws[: info.plan_ints * 4].view(torch.int32).cpu().numpy().copy(), info


CASES = [
    (dict(seed=301, layout_q="TND", B=3, H=64, q_lens=(5, 64, 130), kv_lens=(900, 64, 4000),
          K=512, scenario=3), 148),
    (dict(seed=302, layout_q="TND", B=2, H=128, q_lens=(2, 3), kv_lens=(3000, 2500), K=700,
          scenario=3), 37),
    (dict(seed=303, layout_q="BSND", B=4, H=16, q_lens=(3, 1, 3, 2), kv_lens=(500, 40, 300, 9),
          K=96, scenario=3), 148),
    (dict(seed=304, layout_q="TND", B=2, H=64, q_lens=(300, 1), kv_lens=(300, 800),
          scenario=1), 148),
    (dict(seed=305, layout_q="TND", B=2, H=64, q_lens=(40, 70), kv_lens=(400, 90), scenario=2,
          ratio=4), 5),
    (dict(seed=306, layout_q="BSND", B=6, H=128, q_lens=(1,) * 6,
          kv_lens=(9000, 40, 7000, 64, 128, 3000), K=2048, ratio=1, win_left=-1, scenario=3), 296),
    (dict(seed=307, layout_q="TND", B=1, H=64, q_lens=(1,), kv_lens=(100,), K=64,
          scenario=3), 1),
    # rows of 4 tiles (kept whole) and 5 tiles (cut) next to worker boundaries
    (dict(seed=308, layout_q="BSND", B=12, H=64, q_lens=(1,) * 12,
          kv_lens=(256, 257, 256, 320, 193, 257, 256, 300, 256, 256, 257, 320), K=512,
          ratio=1, win_left=-1, scenario=3), 7),
    (dict(seed=308, layout_q="BSND", B=12, H=64, q_lens=(1,) * 12,
          kv_lens=(256, 257, 256, 320, 193, 257, 256, 300, 256, 256, 257, 320), K=512,
          ratio=1, win_left=-1, scenario=3), 11),
]


@pytest.mark.parametrize("kw,sms", CASES)
def test_device_plan_equals_host_plan(kw, sms):
    case = W.random_case(**kw)
    hp = _sections(_host_plan(case, sms))
    dp_raw, info = _device_plan(case, sms)
    dp = _sections(dp_raw)
    assert hp["counts"] == dp["counts"]
    assert np.array_equal(hp["rows"], dp["rows"])
    assert np.array_equal(hp["workers"], dp["workers"])
    assert np.array_equal(hp["split"], dp["split"])
    assert np.array_equal(hp["acts"][0], dp["acts"][0]) and np.array_equal(hp["acts"][1],
                                                                          dp["acts"][1])
    # the section sizes are worst-case bounds
    assert info.num_split_rows >= dp["counts"][2] and info.num_partials >= dp["counts"][3]


@pytest.mark.parametrize("kw,sms", CASES[:3] + CASES[5:6])
def test_device_plan_forward_is_bitwise_the_host_forward(kw, sms):
    c = W.random_case(**kw).to("cuda")
    a = sparse_attn_sharedkv(c.q, return_softmax_lse=True, num_sms=sms, **c.kwargs())
    b = sparse_attn_sharedkv(c.q, return_softmax_lse=True, num_sms=sms, device_plan=True,
                             **c.kwargs())
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_cuda_graph_replay_with_new_lengths():
    # Same shapes, different lengths: the graph re-plans on the GPU at replay.
    kw = dict(seed=311, layout_q="BSND", B=4, H=64, q_lens=(1,) * 4,
              kv_lens=(3000, 2000, 900, 4000), K=512, scenario=3)
    c = W.random_case(**kw).to("cuda")
    args = c.kwargs()
    seq = args["seqused_kv"].clone()
    args["seqused_kv"] = seq
    sparse_attn_sharedkv(c.q, return_softmax_lse=True, device_plan=True, **args)  # warm-up
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out_g, lse_g = sparse_attn_sharedkv(c.q, return_softmax_lse=True, device_plan=True,
                                            **args)
    for new in ([3000, 2000, 900, 4000], [1200, 4000, 64, 2500], [9, 700, 3999, 1]):
        seq.copy_(torch.tensor(new, dtype=seq.dtype))
        g.replay()
        torch.cuda.synchronize()
        ref = sparse_attn_sharedkv(c.q, return_softmax_lse=True, **args)
        assert torch.equal(out_g, ref[0]) and torch.equal(lse_g, ref[1])


def test_invalid_lengths_are_reported():
    kw = dict(seed=312, layout_q="TND", B=2, H=64, q_lens=(3, 2), kv_lens=(300, 200), K=64,
              scenario=3)
    case = W.random_case(**kw)
    case.seqused_kv = torch.tensor([300, -5], dtype=torch.int32)
    err = torch.zeros(4, dtype=torch.int32, device="cuda")
    _device_plan(case, 148, err=err)
    e = err.tolist()
    assert e[0] == 6 and e[1] == 60
