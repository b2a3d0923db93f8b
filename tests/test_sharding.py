"""Multi-GPU sharding of a call: shard plans, shard inputs (cut sequences,
compacted pages) and the output all-gather.  The host logic is checked on
CPU with the oracle standing in for the per-rank compute, including a real
two-rank gloo all-gather; one GPU test runs the shards through the CUDA
kernel."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import sas_oracle as O
from sparse_attn_sharedkv_b200 import sharding as SH
from tests import workloads as W
from tests.golden_cases import case_to_numpy

CASES = [
    dict(seed=201, layout_q="TND", B=3, H=16, q_lens=(40, 7, 90), kv_lens=(300, 7, 200), K=64,
         scenario=3, ratio=2, idx_mode="dirty"),
    dict(seed=202, layout_q="TND", H=16, q_lens=(70, 33), kv_lens=(150, 400), scenario=2,
         ratio=4),
    dict(seed=203, layout_q="TND", H=16, q_lens=(130,), kv_lens=(260,), scenario=1),
    dict(seed=204, layout_q="BSND", B=5, H=16, q_lens=(1, 1, 1, 1, 1),
         kv_lens=(900, 40, 300, 64, 1000), K=128, scenario=3, sinks="random"),
    dict(seed=205, layout_q="TND", H=16, q_lens=(20, 30), kv_lens=(400, 500), K=96,
         ratio=1, win_left=-1, scenario=3),
    dict(seed=206, layout_q="TND", B=3, H=128, q_lens=(3, 64, 5), kv_lens=(3000, 64, 900),
         K=512, scenario=3, idx_mode="sorted"),
]


def _case(i):
    return W.random_case(D=576, **CASES[i])


def _to_case(q, kw, name="shard"):
    return W.Case(name=name, layout_q=kw.get("layout_q", "TND"), q=q, ori_kv=kw["ori_kv"],
                  ori_block_table=kw["ori_block_table"], seqused_kv=torch.as_tensor(kw["seqused_kv"]),
                  sinks=kw["sinks"], softmax_scale=kw["softmax_scale"],
                  cu_seqlens_q=kw.get("cu_seqlens_q"), cmp_kv=kw.get("cmp_kv"),
                  cmp_block_table=kw.get("cmp_block_table"),
                  cmp_sparse_indices=kw.get("cmp_sparse_indices"), cmp_ratio=kw.get("cmp_ratio"),
                  ori_win_left=kw.get("ori_win_left", 127), head_dim_v=kw.get("head_dim_v"))


def _oracle(q, kw):
    return O.forward(**case_to_numpy(_to_case(q, kw)))


@pytest.mark.parametrize("i", range(len(CASES)))
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_plan_covers_contiguously_and_balances(i, world):
    c = _case(i)
    kw = c.kwargs()
    plan = SH.plan_shards(c.q, kw, world)
    assert plan[0][0] == 0 and len(plan) == world
    for (b0, e0), (b1, e1) in zip(plan, plan[1:]):
        assert e0 == b1 and b0 <= e0
    cost = SH.row_costs(c.q, kw)
    if c.layout_q != "TND":
        cost = cost.reshape(-1, c.q.shape[1]).sum(axis=1)
    assert plan[-1][1] == len(cost)
    per = [int(cost[b:e].sum()) for b, e in plan]
    assert max(per) <= cost.sum() / world + cost.max()


@pytest.mark.parametrize("i", range(len(CASES)))
@pytest.mark.parametrize("compact", [True, False])
def test_shards_reassemble_the_full_call_exactly(i, compact):
    c = _case(i)
    kw = c.kwargs()
    full_out, full_lse = _oracle(c.q, kw)
    world = 3
    outs, lses = [], []
    for r, bounds in enumerate(SH.plan_shards(c.q, kw, world)):
        sh = SH.make_shard(c.q, kw, bounds, rank=r, compact_pages=compact)
        if sh.empty:
            continue
        if compact:
            # compaction keeps only reachable pages
            assert sh.kwargs["ori_kv"].shape[0] <= c.ori_kv.shape[0]
        o, l = _oracle(sh.q, sh.kwargs)
        outs.append(o)
        lses.append(l)
    assert np.array_equal(np.concatenate(outs), full_out)
    assert np.array_equal(np.concatenate(lses), full_lse)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_worker(rank, world, port, i, result_dir, mode="all"):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        c = _case(i)
        kw = c.kwargs()
        plan = SH.plan_shards(c.q, kw, world)
        sh = SH.make_shard(c.q, kw, plan[rank], rank=rank)
        H, dv = c.q.shape[-2], 512
        if c.layout_q == "TND":
            unit, lunit = (H, dv), (H,)
        else:
            unit, lunit = (c.q.shape[1], H, dv), (c.q.shape[1], H)
        o = l = None
        if not sh.empty:
            o, l = _oracle(sh.q, sh.kwargs)
            o, l = torch.from_numpy(o), torch.from_numpy(l)
        if mode == "all":
            go, gl = SH.gather_outputs(o, l, plan, rank, unit, lunit, torch.float32, "cpu")
        else:
            res = SH.gather_to_rank0(o, l, plan, rank, unit, lunit, torch.float32, "cpu")
            assert (res is None) == (rank != 0)
            go, gl = res if res is not None else (None, None)
        if rank == 0:
            np.save(os.path.join(result_dir, "out.npy"), go.numpy())
            np.save(os.path.join(result_dir, "lse.npy"), gl.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("i", [0, 3, 5])
def test_two_rank_gloo_allgather(i, tmp_path):
    world = 2
    mp.start_processes(_gloo_worker, args=(world, _free_port(), i, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    c = _case(i)
    full_out, full_lse = _oracle(c.q, c.kwargs())
    assert np.array_equal(np.load(tmp_path / "out.npy").reshape(full_out.shape), full_out)
    assert np.array_equal(np.load(tmp_path / "lse.npy").reshape(full_lse.shape), full_lse)


@pytest.mark.parametrize("i", [0, 4])
def test_two_rank_gloo_gather_to_rank0(i, tmp_path):
    world = 2
    mp.start_processes(_gloo_worker, args=(world, _free_port(), i, str(tmp_path), "rank0"),
                       nprocs=world, join=True, start_method="spawn")
    c = _case(i)
    full_out, full_lse = _oracle(c.q, c.kwargs())
    assert np.array_equal(np.load(tmp_path / "out.npy").reshape(full_out.shape), full_out)
    assert np.array_equal(np.load(tmp_path / "lse.npy").reshape(full_lse.shape), full_lse)


@pytest.mark.gpu
@pytest.mark.parametrize("i", range(len(CASES)))
def test_gpu_shards_match_oracle(i):
    from sparse_attn_sharedkv_b200.api import sparse_attn_sharedkv
    from tests.checks import check_lse_tight, check_north_star
    c = _case(i).to("cuda")
    kw = c.kwargs()
    outs, lses = [], []
    for r, bounds in enumerate(SH.plan_shards(c.q, kw, 4)):
        sh = SH.make_shard(c.q, kw, bounds, rank=r)
        if sh.empty:
            continue
        o, l = sparse_attn_sharedkv(sh.q, return_softmax_lse=True, **sh.kwargs)
        outs.append(o.float().cpu().numpy())
        lses.append(l.cpu().numpy())
    cc = c.to("cpu")
    exact, _ = O.forward(**dict(case_to_numpy(cc), dtype="fp32"))
    gold, glse = O.forward(**case_to_numpy(cc))
    out, lse = np.concatenate(outs), np.concatenate(lses)
    flat = (lambda a: a) if c.layout_q == "TND" else (lambda a: a.reshape((-1,) + a.shape[2:]))
    check_north_star(flat(out), flat(exact), flat(gold))
    check_lse_tight(flat(lse), flat(glse))
