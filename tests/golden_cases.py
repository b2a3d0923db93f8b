"""Shared helpers: load the committed golden vectors and rebuild their inputs.

The fixtures (``tests/golden/attn_golden.*``) hold the reference golden's
outputs; the inputs are regenerated from the recorded parameters by
``tests.workloads`` (same seeds, same RNG call order).
"""

from __future__ import annotations

import json
import os
from typing import Dict, Tuple

import numpy as np
import torch

from tests import workloads as W

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN_DIR = os.path.join(HERE, "golden")

_ATTN_META = None
_ATTN_ARR = None


def attn_fixtures() -> Dict:
    global _ATTN_META, _ATTN_ARR
    if _ATTN_META is None:
        with open(os.path.join(GOLDEN_DIR, "attn_golden.json")) as f:
            _ATTN_META = json.load(f)
        _ATTN_ARR = np.load(os.path.join(GOLDEN_DIR, "attn_golden.npz"))
    return _ATTN_META


def fixture_expected(key: str) -> Tuple[np.ndarray, np.ndarray]:
    """(out float32, lse float32) stored for fixture ``key``."""
    attn_fixtures()
    bits = _ATTN_ARR[f"{key}.out"]
    dtype = _ATTN_META[key]["dtype"]
    if dtype == "bf16":
        out = (bits.astype(np.uint32) << 16).view(np.float32)
    else:
        out = bits.view(np.float16).astype(np.float32)
    return out, _ATTN_ARR[f"{key}.lse"]


def fixture_case(key: str) -> W.Case:
    meta = attn_fixtures()[key]
    if meta["kind"] == "reference_scenario":
        dt = torch.bfloat16 if meta["dtype"] == "bf16" else torch.float16
        return W.reference_scenario_case(meta["scenario"], dt)
    kw = dict(meta["params"])
    for k in ("q_lens", "kv_lens"):
        if k in kw:
            kw[k] = tuple(kw[k])
    kw["dtype"] = torch.float16 if kw.get("dtype") == "fp16" else torch.bfloat16
    return W.random_case(**kw)


def case_to_numpy(case: W.Case) -> Dict:
    """Keyword arguments of ``oracle.sas_oracle.forward`` for a ``Case``."""
    def f(t):
        return None if t is None else t.detach().cpu().to(torch.float32).numpy()

    def i(t):
        return None if t is None else t.detach().cpu().to(torch.int64).numpy()

    dt = {torch.bfloat16: "bf16", torch.float16: "fp16"}[case.q.dtype]
    return dict(q=f(case.q), ori_kv=f(case.ori_kv), ori_block_table=i(case.ori_block_table),
                seqused_kv=[int(x) for x in case.seqused_kv.tolist()],
                sinks=f(case.sinks), softmax_scale=case.softmax_scale, layout_q=case.layout_q,
                cu_seqlens_q=(None if case.cu_seqlens_q is None
                              else [int(x) for x in case.cu_seqlens_q.tolist()]),
                cmp_kv=f(case.cmp_kv), cmp_block_table=i(case.cmp_block_table),
                cmp_sparse_indices=i(case.cmp_sparse_indices),
                cmp_ratio=case.cmp_ratio if case.cmp_ratio is not None else 4,
                ori_win_left=case.ori_win_left, head_dim_v=case.head_dim_v, dtype=dt)
