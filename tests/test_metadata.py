"""The C++ scheduler (``sas_metadata``) against the reference metadata.py.

Fixtures: ``tests/golden/metadata_golden.json``, produced by running the
reference's ``metadata.sparse_attn_sharedkv_metadata`` (metadata.py:1018-1086)
on the reference suite's scenarios, the 8K prefill shapes and a seeded random
sweep (``tests/golden/make_golden.py``).  The gate is bit equality of the
int32[1024] table.  The invariants of the reference's own CPU tests
(test_sparse_attn_sharedkv.py:721-924) are re-checked on our output.
"""

import json
import os

import pytest
import torch

from tests import workloads as W
from sparse_attn_sharedkv_b200.metadata import (AIC_CORE_NUM, FA_METADATA_SIZE, SAS_META_SIZE,
                                                sparse_attn_sharedkv_metadata)

HERE = os.path.dirname(os.path.abspath(__file__))
with open(os.path.join(HERE, "golden", "metadata_golden.json")) as f:
    FIX = json.load(f)


def _call(kw):
    call = {k: (torch.tensor(v, dtype=torch.int32) if isinstance(v, list) else v)
            for k, v in kw.items()}
    return sparse_attn_sharedkv_metadata(**call)


@pytest.mark.parametrize("name", sorted(FIX))
def test_metadata_bit_exact(name):
    out = _call(FIX[name]["kwargs"])
    assert out.dtype == torch.int32 and out.shape == (SAS_META_SIZE,)
    assert out.tolist() == FIX[name]["out"]


def _kwargs_for(name, aic=24):
    cfg = W.REFERENCE_SCENARIOS[name]
    scen = cfg["scenario"]
    kw = dict(num_heads_q=cfg["N1"], num_heads_kv=cfg["N2"], head_dim=cfg["D"],
              cu_seqlens_q=torch.tensor(cfg["cu_seqlens_q"], dtype=torch.int32),
              seqused_kv=torch.tensor(cfg["seqused_kv"], dtype=torch.int32),
              batch_size=cfg["B"], max_seqlen_q=cfg["T1"], max_seqlen_kv=max(cfg["seqused_kv"]),
              ori_mask_mode=4, ori_win_left=cfg["ori_win_left"], ori_win_right=0,
              layout_q="TND", layout_kv="PA_ND", has_ori_kv=True, has_cmp_kv=scen >= 2,
              aic_core_num=aic)
    if scen >= 2:
        kw.update(cmp_ratio=cfg["cmp_ratio"], cmp_mask_mode=3)
    if scen == 3:
        kw["cmp_topk"] = cfg["K"]
    return kw, cfg


@pytest.mark.parametrize("name", sorted(W.REFERENCE_SCENARIOS))
def test_metadata_shape_and_continuity(name):
    """Enabled cores chain (bn2, m, s2)_start == previous end
    (test_sparse_attn_sharedkv.py:721-792)."""
    kw, cfg = _kwargs_for(name)
    md = sparse_attn_sharedkv_metadata(**kw)
    fa = md[: AIC_CORE_NUM * FA_METADATA_SIZE].view(AIC_CORE_NUM, FA_METADATA_SIZE)
    assert int(fa[:, 0].sum()) >= 1
    prev = (0, 0, 0)
    for row in fa[fa[:, 0] == 1].tolist():
        assert tuple(row[1:4]) == prev
        prev = tuple(row[4:7])
    assert prev[0] in (cfg["B"] * cfg["N2"], 0)


@pytest.mark.parametrize("name", sorted(W.REFERENCE_SCENARIOS))
def test_metadata_drives_complete_coverage(name):
    """Every valid (b, s) is visited exactly once by the linearised core
    windows (test_sparse_attn_sharedkv.py:795-893)."""
    kw, cfg = _kwargs_for(name)
    md = sparse_attn_sharedkv_metadata(**kw).numpy()
    fa = md[: AIC_CORE_NUM * FA_METADATA_SIZE].reshape(AIC_CORE_NUM, FA_METADATA_SIZE)
    cu = cfg["cu_seqlens_q"]
    B = cfg["B"]
    act = [cu[i + 1] - cu[i] for i in range(B)]
    max_seq = max(act)
    seen, dup = set(), []
    for cid in range(24):
        en, b0, m0, _, b1, m1, _, _ = fa[cid].tolist()
        if not en:
            continue
        for pid in range(b0 * max_seq + m0, b1 * max_seq + m1):
            b, s = divmod(pid, max_seq)
            if b < B and s < act[b]:
                if (b, s) in seen:
                    dup.append((cid, b, s))
                seen.add((b, s))
    assert not dup
    assert seen == {(b, s) for b in range(B) for s in range(act[b])}


def test_metadata_prefill_uses_all_cores():
    """8K prefill spreads over all 24 AICs (test_sparse_attn_sharedkv.py:896-924)."""
    md = torch.tensor(FIX["prefill8k_s3"]["out"], dtype=torch.int32)
    fa = md[: AIC_CORE_NUM * FA_METADATA_SIZE].view(AIC_CORE_NUM, FA_METADATA_SIZE)
    assert int(fa[:, 0].sum()) == 24
    assert _call(FIX["prefill8k_s3"]["kwargs"]).tolist() == FIX["prefill8k_s3"]["out"]


def test_metadata_errors():
    with pytest.raises(ValueError):
        sparse_attn_sharedkv_metadata(num_heads_q=64, num_heads_kv=0, head_dim=512,
                                      seqused_kv=torch.tensor([10]), batch_size=1,
                                      max_seqlen_q=1, max_seqlen_kv=10)
    with pytest.raises(ValueError):  # two batches, one kv length
        sparse_attn_sharedkv_metadata(num_heads_q=64, num_heads_kv=1, head_dim=512,
                                      seqused_kv=torch.tensor([10]), batch_size=2,
                                      max_seqlen_q=1, max_seqlen_kv=10, layout_q="BSND")


def test_metadata_device_argument():
    out = sparse_attn_sharedkv_metadata(num_heads_q=64, num_heads_kv=1, head_dim=512,
                                        seqused_kv=torch.tensor([100]), batch_size=1,
                                        max_seqlen_q=1, max_seqlen_kv=100, device="cpu")
    assert out.device.type == "cpu" and out.numel() == SAS_META_SIZE
