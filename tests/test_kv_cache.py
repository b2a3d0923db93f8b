"""Paged-cache writer: the oracle against the reference's paged layout (CPU)
and the CUDA writer against the oracle, bit for bit (GPU)."""

import numpy as np
import pytest
import torch

from oracle import sas_oracle as O


def _layout_case(seed=0, B=3, bs=64, D=32, lens=(130, 1, 64), blocks=12):
    rng = np.random.default_rng(seed)
    per = [-(-n // bs) for n in lens]
    perm = rng.permutation(blocks).astype(np.int32)
    table = np.full((B, max(per)), -1, np.int32)
    c = 0
    for b, nb in enumerate(per):
        table[b, :nb] = perm[c:c + nb]
        c += nb
    dense = [rng.integers(0, 2 ** 16, size=(n, D), dtype=np.uint16) for n in lens]
    return table, dense


def test_oracle_append_matches_reference_placement():
    # The reference generator (golden.py:315-360) places row p of batch b at
    # pa[table[b, p // bs], p % bs]; appending each sequence in uneven chunks
    # must build the same pool.
    bs, D = 64, 32
    table, dense = _layout_case(bs=bs, D=D)
    want = np.zeros((12, bs, D), np.uint16)
    for b, rows in enumerate(dense):
        for p in range(len(rows)):
            want[table[b, p // bs], p % bs] = rows[p]
    got = np.zeros_like(want)
    done = [0] * len(dense)
    for chunk in (1, 7, 64, 1000):
        new = [rows[done[b]:done[b] + chunk] for b, rows in enumerate(dense)]
        cu = np.concatenate([[0], np.cumsum([len(x) for x in new])])
        bad = O.append_paged(got, table, np.concatenate(new, axis=0), cu, done)
        assert bad == []
        done = [d + len(x) for d, x in zip(done, new)]
    assert np.array_equal(got, want)


def test_oracle_append_skips_unmapped_pages():
    pool = np.zeros((2, 4, 8), np.uint16)
    table = np.array([[1, -1]], np.int32)
    rows = np.arange(6 * 8, dtype=np.uint16).reshape(6, 8) + 1
    bad = O.append_paged(pool, table, rows, [0, 6], [2])
    # positions 2, 3 -> block 1; 4..7 -> unmapped
    assert bad == [2, 3, 4, 5]
    assert np.array_equal(pool[1, 2], rows[0]) and np.array_equal(pool[1, 3], rows[1])
    assert not pool[0].any()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gpu_append_bit_exact(dtype):
    from sparse_attn_sharedkv_b200.kv_cache import append_paged_kv
    rng = np.random.default_rng(3)
    B, bs, D, blocks = 5, 64, 576, 64
    table = rng.permutation(blocks)[:B * 8].reshape(B, 8).astype(np.int32)
    before = np.array([0, 63, 64, 200, 511], np.int32)
    add = np.array([3, 1, 0, 129, 1], np.int32)  # ragged, one empty batch
    cu = np.concatenate([[0], np.cumsum(add)]).astype(np.int32)
    pool0 = rng.integers(0, 2 ** 16, size=(blocks, bs, D), dtype=np.uint16)
    rows = rng.integers(0, 2 ** 16, size=(int(cu[-1]), D), dtype=np.uint16)
    want = pool0.copy()
    assert O.append_paged(want, table, rows, cu, before) == []
    t = lambda a: torch.from_numpy(a.view(np.int16)).view(dtype).cuda()
    pool = t(pool0).view(blocks, bs, 1, D).contiguous()
    err = append_paged_kv(pool, torch.from_numpy(table).cuda(), t(rows).view(-1, 1, D),
                          torch.from_numpy(cu), torch.from_numpy(before), check_errors=True)
    assert err is None
    got = pool.view(torch.int16).cpu().numpy().view(np.uint16).reshape(blocks, bs, D)
    assert np.array_equal(got, want)


@pytest.mark.gpu
def test_gpu_append_reports_unmapped_page():
    from sparse_attn_sharedkv_b200.kv_cache import append_paged_kv
    D, bs = 576, 64
    pool = torch.zeros(4, bs, 1, D, dtype=torch.bfloat16, device="cuda")
    table = torch.tensor([[2, -1]], dtype=torch.int32, device="cuda")
    rows = torch.ones(3, D, dtype=torch.bfloat16, device="cuda")
    err = append_paged_kv(pool, table, rows, torch.tensor([0, 3]), torch.tensor([63]),
                          check_errors=True)
    # position 63 -> block 2, row 63; positions 64, 65 -> unmapped page
    assert err is not None and err[0] == 6 and err[1] == 50 and err[2] in (1, 2)
    assert torch.all(pool[2, 63] == 1) and int(pool.float().abs().sum()) == D


@pytest.mark.gpu
def test_appended_cache_feeds_attention():
    # Build a cache by appending, then run the forward: equal to the forward on
    # the directly generated cache (the writer produces the path's input layout).
    from tests import workloads as W
    from sparse_attn_sharedkv_b200.api import sparse_attn_sharedkv
    from sparse_attn_sharedkv_b200.kv_cache import append_paged_kv
    case = W.random_case(seed=91, layout_q="TND", H=64, q_lens=(3, 2), kv_lens=(700, 300),
                         K=256, scenario=3).to("cuda")
    kw = case.kwargs()
    ref_out, ref_lse = sparse_attn_sharedkv(case.q, return_softmax_lse=True, **kw)
    pool = case.ori_kv
    bs = pool.shape[1]
    table = case.ori_block_table
    lens = case.seqused_kv.cpu().tolist()
    rebuilt = torch.zeros_like(pool)
    rows = []
    for b, n in enumerate(lens):
        for p in range(n):
            rows.append(pool[int(table[b, p // bs]), p % bs, 0])
    rows = torch.stack(rows)
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32)
    assert append_paged_kv(rebuilt, table, rows, cu, torch.zeros(len(lens), dtype=torch.int32),
                           check_errors=True) is None
    kw["ori_kv"] = rebuilt
    if kw.get("cmp_kv") is case.ori_kv:
        kw["cmp_kv"] = rebuilt
    out, lse = sparse_attn_sharedkv(case.q, return_softmax_lse=True, **kw)
    assert torch.equal(out, ref_out) and torch.equal(lse, ref_lse)
