"""Ring rows (pure sliding window of 65..128 keys, kRowRing): the two K
stages keep the window from one query of a sequence to the next and take in
one key row per query.  Checked against the CPU oracle across the cases that
change the ring's path: warm queries (long runs of consecutive tokens), cold
starts (sequence changes, worker boundaries), split rows (small worker counts
cut rows into pieces, which load in the plain layout), prefixes (act_kv >
act_q), short sequences (positions below 0 in the ring), page sizes 16 / 64 /
128, windows 65 / 101 / 128, d_qk 512, fp16, BSND padding, H = 16 / 128, -inf
sinks, and the cp.async gather mode (ring rows in the plain layout)."""

import os

import numpy as np
import pytest
import torch

os.environ.setdefault("SAS_CHECK_DEVICE_ERRORS", "1")

from tests import workloads as W  # noqa: E402
from tests.checks import check_lse_tight, check_north_star  # noqa: E402
from tests.test_gpu_parity import oracle, run  # noqa: E402

pytestmark = pytest.mark.gpu

BASE = dict(layout_q="TND", scenario=1, H=64, q_lens=(300, 70, 129), kv_lens=(300, 500, 129))

CASES = [
    dict(seed=801, **BASE),
    dict(seed=802, **dict(BASE, win_left=64)),
    dict(seed=803, **dict(BASE, win_left=100, block_size=16)),
    dict(seed=804, **dict(BASE, block_size=128, sinks="-inf")),
    dict(seed=805, **dict(BASE, D=512, d_v=None)),
    dict(seed=806, **dict(BASE, dtype=torch.float16, H=16)),
    dict(seed=807, layout_q="BSND", B=2, scenario=1, H=128, q_lens=(70, 30),
         kv_lens=(200, 30)),
    dict(seed=808, layout_q="TND", scenario=1, H=64, B=4, q_lens=(1, 2, 63, 65),
         kv_lens=(1, 2, 63, 65), sinks="-inf"),
]


@pytest.mark.parametrize("num_sms", [148, 7, 1])
@pytest.mark.parametrize("kw", CASES)
def test_ring_rows_vs_oracle(kw, num_sms):
    case = W.random_case(**kw)
    out, lse = run(case, num_sms=num_sms)
    ex, gold, o_lse = oracle(case)
    check_north_star(out, ex, gold)
    check_lse_tight(lse, o_lse)


def test_ring_rows_in_cp_async_mode(monkeypatch):
    case = W.random_case(seed=811, **BASE)
    ring = run(case)
    monkeypatch.setenv("SAS_GATHER", "lsu")
    plain = run(case)
    ex, gold, o_lse = oracle(case)
    for out, lse in (ring, plain):
        check_north_star(out, ex, gold)
        check_lse_tight(lse, o_lse)


def test_ring_rows_deterministic():
    case = W.random_case(seed=812, **BASE)
    a = run(case, num_sms=20)
    b = run(case, num_sms=20)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
