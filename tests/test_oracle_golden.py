"""Pin the CPU oracle against the reference golden's committed outputs.

The fixtures were produced by ``tests/golden/make_golden.py`` from the
reference's ``golden.sparse_attn_sharedkv_golden_bnsd`` (golden.py:69-204) on
inputs that are tensor-identical to the reference suite's ``_build_case``
(test_sparse_attn_sharedkv.py:238-391) plus extension cases.  Both sides are
fp32 with different reduction orders, so ``out`` may differ by one
bf16/fp16 rounding step on rare elements; LSE agrees to ~1e-5.
"""

import math

import numpy as np
import pytest

from oracle import sas_oracle as O
from tests.golden_cases import attn_fixtures, case_to_numpy, fixture_case, fixture_expected

KEYS = sorted(attn_fixtures().keys())


def _ulp_close(got, exp, dtype):
    """Difference in units of the output dtype's spacing at ``|exp|``.  Small
    values come from cancellation, where the fp32 reduction order dominates, so
    they are measured against the spacing at a floor (2^-8 for bf16, 2^-5 for
    fp16, i.e. an absolute 2^-15 either way)."""
    mant = 8 if dtype == "bf16" else 11
    mag = np.maximum(np.abs(exp), 2.0 ** (-8 if dtype == "bf16" else -5))
    spacing = 2.0 ** (np.floor(np.log2(mag)) - (mant - 1))
    return np.abs(got - exp) / spacing


@pytest.mark.parametrize("key", KEYS)
def test_oracle_matches_reference_golden(key):
    meta = attn_fixtures()[key]
    case = fixture_case(key)
    kw = case_to_numpy(case)
    toks = meta["tokens"]
    out, lse = O.forward(**kw, tokens=toks)
    exp_out, exp_lse = fixture_expected(key)
    if toks is not None:
        out, lse = out[toks], lse[toks]
    if meta.get("heads") is not None:
        out = out[:, meta["heads"]]
    assert out.shape == exp_out.shape and lse.shape == exp_lse.shape
    ulps = _ulp_close(out, exp_out, meta["dtype"])
    # 2: one rounding step on each side of a binade boundary.
    assert float(ulps.max()) <= 2.0, f"{key}: max {ulps.max()} ulp"
    assert float((ulps > 0).mean()) < 1e-2, f"{key}: {(ulps > 0).mean()} differ"
    fin = np.isfinite(exp_lse)
    assert np.array_equal(fin, np.isfinite(lse))
    np.testing.assert_allclose(lse[fin], exp_lse[fin], rtol=2e-6, atol=2e-5)
    assert np.array_equal(lse[~fin], exp_lse[~fin])


def test_oracle_tiled_walk_matches_one_shot():
    """The reference's ``test_golden_math_matches_single_shot_softmax``
    (test_sparse_attn_sharedkv.py:930-1002): chunked online softmax with sinks
    vs a one-shot softmax over the same key set, on our oracle."""
    rng = np.random.default_rng(0)
    H, D, L, ratio, K, S1 = 64, 512, 128, 4, 8, 4
    q = rng.uniform(-1, 1, (S1, H, D)).astype(np.float32)
    dense = rng.uniform(-1, 1, (L, D)).astype(np.float32)
    cdense = rng.uniform(-1, 1, (L // ratio, D)).astype(np.float32)
    ori = dense.reshape(L // 64, 64, 1, D)
    cmp = np.zeros((1, 64, 1, D), np.float32)
    cmp[0, : L // ratio, 0] = cdense
    sinks = rng.uniform(0, 0.1, H).astype(np.float32)
    idx = np.full((S1, 1, K), -1, np.int64)
    for s in range(S1):
        thr = (L - S1 + s + 1) // ratio
        take = min(K, max(thr, 0))
        idx[s, 0, :take] = np.arange(take)
    out, lse = O.forward(q=q, ori_kv=ori, ori_block_table=np.array([[0, 1]]), seqused_kv=[L],
                         sinks=sinks, softmax_scale=1 / math.sqrt(D), cu_seqlens_q=[0, S1],
                         cmp_kv=cmp, cmp_block_table=np.array([[0]]), cmp_sparse_indices=idx,
                         cmp_ratio=ratio, dtype="fp32", s2_tile=16)
    for s in range(S1):
        s_g = L - S1 + s
        keys = np.concatenate([dense[max(s_g - 127, 0): s_g + 1],
                               cdense[idx[s, 0][(idx[s, 0] >= 0)]]])
        o1, l1 = O.one_shot(q[s], keys, sinks, 1 / math.sqrt(D), "fp32", D)
        np.testing.assert_allclose(out[s], o1, rtol=2e-4, atol=2e-4)
        np.testing.assert_allclose(lse[s], l1, rtol=1e-4, atol=1e-4)


def test_scfa_index_semantics():
    """-1 stops the scan, ids >= threshold are skipped, only the first
    min(K, threshold) entries are scanned (golden.py:48-62)."""
    row = np.array([3, 9, 2, -1, 1, 0], dtype=np.int64)
    # act_kv=40, act_q=1, s=0, ratio=4 -> threshold 10, cmp_act_kv 10
    assert O.scfa_positions(row, 40, 1, 0, 4) == [3, 9, 2]
    # threshold 3: scan the first 3 entries only; 3 and 9 are >= 3.
    assert O.scfa_positions(row, 12, 1, 0, 4) == [2]
    # threshold <= 0: nothing.
    assert O.scfa_positions(row, 3, 1, 0, 4) == []
    # duplicates are attended twice.
    assert O.scfa_positions(np.array([1, 1, -1]), 40, 1, 0, 4) == [1, 1]
    # an id past the compressed length is dropped even under the threshold
    # (act_kv=41, act_q=2, s=1 -> threshold 10, cmp_act_kv 10).
    assert O.scfa_positions(np.array([10, 4]), 41, 2, 1, 4) == [4]


def test_empty_rows_give_sink_lse_and_zero_out():
    """No attended key: out = 0, lse = sink (or -inf when the sink is -inf)."""
    D = 64
    q = np.ones((2, 4, D), np.float32)
    ori = np.ones((1, 64, 1, D), np.float32)
    sinks = np.array([0.5, -1.0, -np.inf, 2.0], np.float32)
    out, lse = O.forward(q=q, ori_kv=ori, ori_block_table=np.array([[0]]), seqused_kv=[2],
                         sinks=sinks, softmax_scale=0.1, cu_seqlens_q=[0, 2], ori_win_left=-1)
    assert np.all(out == 0)
    assert np.array_equal(lse[0], sinks) and np.array_equal(lse[1], sinks)
