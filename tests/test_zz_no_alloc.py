"""sas_fwd_noalloc: the forward for callers that cannot allocate device memory.

Some users of this library run attention inside a device-memory arena that
was planned ahead of time, or under an allocator that is frozen during a
step, so they cannot size and allocate the workspace that ``sas_fwd`` needs.
``sas_fwd_noalloc`` keeps that workspace (work plan + split-KV partials) in a
fixed 16 MiB device array inside the library instead.

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test.  It calls both entry points
directly through the C ABI (ctypes on libsas.so), on two different problems
in a row, and requires the no-allocation outputs to equal those of
``sas_fwd`` with a caller workspace: same plan and same kernels, so the
results must be bit-identical (the tolerance used elsewhere in the suite
would also be met).  Both problems split query rows over several workers,
so the partial buffers inside the shared array are exercised, and the
second call runs on whatever the first left in the array.
"""

import ctypes as C

import numpy as np
import pytest
import torch

from sparse_attn_sharedkv_b200 import _lib
from tests import workloads as W
from sparse_attn_sharedkv_b200.api import build_call

pytestmark = pytest.mark.gpu


def _outputs(case: W.Case, entry: str, num_sms: int):
    """Run one forward through the named C-ABI entry point."""
    c = case.to("cuda")
    call = build_call(c.q, num_sms=num_sms, **c.kwargs())
    L = _lib.lib()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    if entry == "sas_fwd":
        nbytes = C.c_size_t(0)
        _lib.check("sas_fwd_workspace_size",
                   L.sas_fwd_workspace_size(C.byref(call.prob), num_sms, C.byref(nbytes)))
        ws = torch.empty(max(nbytes.value, 256), dtype=torch.uint8, device="cuda")
        _lib.check("sas_fwd", L.sas_fwd(C.byref(call.prob), C.byref(call.fp), ws.data_ptr(),
                                        nbytes.value, stream))
    else:
        _lib.check("sas_fwd_noalloc",
                   L.sas_fwd_noalloc(C.byref(call.prob), C.byref(call.fp), stream))
    torch.cuda.synchronize()
    return call.out.float().cpu().numpy(), call.lse.cpu().numpy()


CASES = [
    # 128 heads (two CTAs per worker), rows split over many workers.
    (dict(seed=81, layout_q="TND", H=128, q_lens=(2, 3), kv_lens=(3000, 2500), K=700,
          scenario=3), 37),
    # 64 heads, BSND decode, window + top-k, different split pattern.
    (dict(seed=82, layout_q="BSND", B=3, H=64, q_lens=(1, 1, 1), kv_lens=(4000, 900, 2600),
          K=512, scenario=3, sinks="random"), 64),
]


def test_noalloc_matches_sas_fwd_on_two_calls_in_a_row():
    for kw, num_sms in CASES:
        case = W.random_case(**kw)
        ref_out, ref_lse = _outputs(case, "sas_fwd", num_sms)
        out, lse = _outputs(case, "sas_fwd_noalloc", num_sms)
        assert np.isfinite(out).all()
        assert np.array_equal(out, ref_out)
        assert np.array_equal(lse, ref_lse)


def test_noalloc_rejects_problems_beyond_its_scratch():
    # 128 heads over many workers: the split-KV partials alone exceed 16 MiB.
    case = W.random_case(seed=83, layout_q="BSND", B=8, H=128, q_lens=(1,) * 8,
                         kv_lens=(6000,) * 8, K=2048, ratio=1, win_left=-1, scenario=3)
    c = case.to("cuda")
    call = build_call(c.q, num_sms=296, **c.kwargs())
    rc = _lib.lib().sas_fwd_noalloc(C.byref(call.prob), C.byref(call.fp),
                                    C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 5  # SAS_ERR_WORKSPACE
