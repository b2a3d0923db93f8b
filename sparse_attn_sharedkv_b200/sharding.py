"""Multi-GPU sharding of one sparse shared-KV attention call.

Every query row's output depends only on its own key set, so a call splits
into independent shards, one per rank (one process per GPU), with a single
exchange at the end: an all-gather of the output and LSE shards.

* ``plan_shards``: contiguous ranges of the call's rows, balanced on the
  kernel's work (1 + 64-key tiles per row, the cost the single-GPU planner
  also uses).  BSND (decode) splits by batch; TND (prefill) by flat token,
  cutting a sequence where needed: a piece ``[t0, t1)`` of a sequence with
  ``(act_q, act_kv)`` becomes a sequence of ``t1 - t0`` queries over
  ``act_kv - (act_q - t1)`` keys, which keeps every query's global position
  ``s_g = act_kv - act_q + s`` (golden.py:125-150) and hence its window,
  threshold and top-k filter.
* ``make_shard``: the shard's operator inputs.  With ``compact_pages`` the
  shard gets only the KV pages its rows can reach, in a compacted pool with
  remapped block tables (pages outside the reachable range map to -1).
* ``gather_outputs``: all-gather of the output / LSE shards (NCCL over
  NVLink on GPUs, gloo on CPU) back into the full call's layout.

Host-side logic only; the compute of a shard is an ordinary
``sparse_attn_sharedkv`` call on the rank's GPU.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

TILE = 64


def _row_keys(act_q: int, act_kv: int, s: int, win_left: int, scenario: int, ratio: int,
              topk: int) -> int:
    """Key slots of query s (window + compressed), golden.py:125-150."""
    s_g = act_kv - act_q + s
    lo = max(s_g - win_left, 0)
    window = max(s_g + 1 - lo, 0)
    cmp = 0
    if scenario >= 2 and ratio:
        thr = (s_g + 1) // ratio
        cmp = max(thr, 0)
        if scenario == 3:
            cmp = min(cmp, topk)
    return window + cmp


def _scenario(kw: Dict) -> int:
    if kw.get("cmp_kv") is None:
        return 1
    return 3 if kw.get("cmp_sparse_indices") is not None else 2


def _topk(kw: Dict) -> int:
    idx = kw.get("cmp_sparse_indices")
    return int(idx.shape[-1]) if idx is not None else 0


def row_costs(q: torch.Tensor, kw: Dict) -> np.ndarray:
    """Per output row: 1 + number of 64-key tiles (padded BSND rows: 1)."""
    layout = kw.get("layout_q", "TND")
    lens_kv = [int(x) for x in torch.as_tensor(kw["seqused_kv"]).cpu().tolist()]
    scen, ratio, topk = _scenario(kw), int(kw.get("cmp_ratio") or 0), _topk(kw)
    win = int(kw.get("ori_win_left", 127))
    costs = []
    if layout == "TND":
        cu = [int(x) for x in torch.as_tensor(kw["cu_seqlens_q"]).cpu().tolist()]
        for b in range(len(cu) - 1):
            aq = cu[b + 1] - cu[b]
            for s in range(aq):
                k = _row_keys(aq, lens_kv[b], s, win, scen, ratio, topk)
                costs.append(1 + (k + TILE - 1) // TILE)
    else:
        B, S = q.shape[0], q.shape[1]
        seqused_q = kw.get("seqused_q")
        act = ([int(x) for x in torch.as_tensor(seqused_q).cpu().tolist()]
               if seqused_q is not None else [S] * B)
        for b in range(B):
            for s in range(S):
                if s >= act[b]:
                    costs.append(1)
                else:
                    k = _row_keys(act[b], lens_kv[b], s, win, scen, ratio, topk)
                    costs.append(1 + (k + TILE - 1) // TILE)
    return np.asarray(costs, dtype=np.int64)


def plan_shards(q: torch.Tensor, kw: Dict, world: int) -> List[Tuple[int, int]]:
    """Contiguous [begin, end) ranges per rank, balanced on work.

    TND: ranges of flat tokens.  BSND: ranges of batches (a decode batch
    entry is never split).  Ranks may receive an empty range when there are
    fewer units than ranks."""
    layout = kw.get("layout_q", "TND")
    cost = row_costs(q, kw)
    if layout != "TND":
        S = q.shape[1]
        cost = cost.reshape(-1, S).sum(axis=1)  # per batch
    n = len(cost)
    csum = np.concatenate([[0], np.cumsum(cost)])
    total = csum[-1]
    bounds = [0]
    for r in range(1, world):
        target = total * r / world
        # first unit whose prefix reaches the target
        i = int(np.searchsorted(csum, target, side="left"))
        bounds.append(min(max(i, bounds[-1]), n))
    bounds.append(n)
    return [(bounds[r], bounds[r + 1]) for r in range(world)]


@dataclass
class Shard:
    """One rank's part of a call: its operator inputs and its output rows."""

    rank: int
    begin: int            # first unit (TND token / BSND batch) of the call
    end: int
    q: Optional[torch.Tensor]
    kwargs: Optional[Dict]

    @property
    def empty(self) -> bool:
        return self.end <= self.begin


def _compact(pool: torch.Tensor, tables: torch.Tensor, reach: List[int], bs: int):
    """Pages of `tables` rows below `reach[i]` positions -> compacted pool."""
    t = tables.cpu().numpy().copy()
    ids = []
    for i, n in enumerate(reach):
        nb = (n + bs - 1) // bs
        row = t[i]
        row[nb:] = -1
        ids.extend(int(x) for x in row[:nb] if x >= 0)
    uniq = sorted(set(ids))
    remap = {old: new for new, old in enumerate(uniq)}
    for i in range(t.shape[0]):
        for j in range(t.shape[1]):
            if t[i, j] >= 0:
                t[i, j] = remap[int(t[i, j])]
    idx = torch.tensor(uniq if uniq else [0], dtype=torch.long, device=pool.device)
    return pool.index_select(0, idx).contiguous(), torch.from_numpy(t).to(tables.device)


def make_shard(q: torch.Tensor, kw: Dict, bounds: Tuple[int, int], rank: int = 0,
               compact_pages: bool = True) -> Shard:
    """Operator inputs of the shard covering units [begin, end) of the call."""
    begin, end = bounds
    if end <= begin:
        return Shard(rank, begin, end, None, None)
    layout = kw.get("layout_q", "TND")
    lens_kv = [int(x) for x in torch.as_tensor(kw["seqused_kv"]).cpu().tolist()]
    out = dict(kw)
    ori_bs = kw["ori_kv"].shape[1]
    ratio = int(kw.get("cmp_ratio") or 0)
    if layout == "TND":
        cu = [int(x) for x in torch.as_tensor(kw["cu_seqlens_q"]).cpu().tolist()]
        batches, new_q, new_kv = [], [], []
        for b in range(len(cu) - 1):
            t0, t1 = max(cu[b], begin), min(cu[b + 1], end)
            if t0 >= t1:
                continue
            aq = cu[b + 1] - cu[b]
            lt1 = t1 - cu[b]
            kv = lens_kv[b] - (aq - lt1)
            if kv < 0:
                raise ValueError("cannot cut a sequence with seqused_kv < act_q mid-way")
            batches.append(b)
            new_q.append(t1 - t0)
            new_kv.append(kv)
        sel = torch.tensor(batches, dtype=torch.long)
        qs = q[begin:end]
        dev = q.device
        out["cu_seqlens_q"] = torch.tensor(np.concatenate([[0], np.cumsum(new_q)]),
                                           dtype=torch.int32, device=dev)
        out["seqused_kv"] = torch.tensor(new_kv, dtype=torch.int32, device=dev)
        if kw.get("cmp_sparse_indices") is not None:
            out["cmp_sparse_indices"] = kw["cmp_sparse_indices"][begin:end]
    else:
        sel = torch.arange(begin, end, dtype=torch.long)
        qs = q[begin:end]
        new_kv = lens_kv[begin:end]
        out["seqused_kv"] = torch.as_tensor(kw["seqused_kv"])[begin:end]
        if kw.get("seqused_q") is not None:
            out["seqused_q"] = torch.as_tensor(kw["seqused_q"])[begin:end]
        if kw.get("cmp_sparse_indices") is not None:
            out["cmp_sparse_indices"] = kw["cmp_sparse_indices"][begin:end]
    sel = sel.to(kw["ori_block_table"].device)
    ori_bt = kw["ori_block_table"].index_select(0, sel)
    cmp_bt = (kw["cmp_block_table"].index_select(0, sel.to(kw["cmp_block_table"].device))
              if kw.get("cmp_block_table") is not None else None)
    shared = kw.get("cmp_kv") is not None and kw["cmp_kv"] is kw["ori_kv"]
    if compact_pages:
        reach = [(n // ratio) if ratio else 0 for n in new_kv]
        if shared and cmp_bt is not None:
            # One pool serves both branches (pure top-k): compact over both tables.
            pool, tabs = _compact(kw["ori_kv"], torch.cat([ori_bt, cmp_bt]),
                                  list(new_kv) + reach, ori_bs)
            out["ori_kv"] = out["cmp_kv"] = pool
            ori_bt, cmp_bt = tabs[:len(sel)], tabs[len(sel):]
        else:
            out["ori_kv"], ori_bt = _compact(kw["ori_kv"], ori_bt, new_kv, ori_bs)
            if cmp_bt is not None:
                out["cmp_kv"], cmp_bt = _compact(kw["cmp_kv"], cmp_bt, reach,
                                                 kw["cmp_kv"].shape[1])
    out["ori_block_table"] = ori_bt.contiguous()
    if cmp_bt is not None:
        out["cmp_block_table"] = cmp_bt.contiguous()
    return Shard(rank, begin, end, qs, out)


def gather_outputs(out: Optional[torch.Tensor], lse: Optional[torch.Tensor],
                   plan: List[Tuple[int, int]], rank: int, unit_shape: Tuple[int, ...],
                   lse_unit_shape: Tuple[int, ...], dtype: torch.dtype, device,
                   group=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """All-gather the output / LSE shards into the full call's tensors.

    unit_shape: output shape of one unit ([H, d_v] per TND token, [S, H, d_v]
    per BSND batch); lse_unit_shape likewise.  Shards are padded to the
    largest one for the collective (every rank takes the same steps)."""
    import torch.distributed as dist

    world = len(plan)
    sizes = [e - b for b, e in plan]
    mx = max(max(sizes), 1)
    pad_o = torch.zeros((mx, *unit_shape), dtype=dtype, device=device)
    pad_l = torch.zeros((mx, *lse_unit_shape), dtype=torch.float32, device=device)
    n = sizes[rank]
    if n:
        pad_o[:n].copy_(out.reshape(n, *unit_shape))
        pad_l[:n].copy_(lse.reshape(n, *lse_unit_shape))
    go = [torch.empty_like(pad_o) for _ in range(world)]
    gl = [torch.empty_like(pad_l) for _ in range(world)]
    dist.all_gather(go, pad_o, group=group)
    dist.all_gather(gl, pad_l, group=group)
    return (torch.cat([go[r][:sizes[r]] for r in range(world)], 0),
            torch.cat([gl[r][:sizes[r]] for r in range(world)], 0))


def gather_to_rank0(out: Optional[torch.Tensor], lse: Optional[torch.Tensor],
                    plan: List[Tuple[int, int]], rank: int, unit_shape: Tuple[int, ...],
                    lse_unit_shape: Tuple[int, ...], dtype: torch.dtype, device,
                    group=None) -> Optional[Tuple[torch.Tensor, torch.Tensor]]:
    """Gather the output / LSE shards into the full call's tensors on rank 0
    only (the rank that needs the whole output); other ranks send and get
    None.  Moves one copy of the output across the links instead of the N
    copies an all-gather makes.  Shards are padded to the largest one (every
    rank takes the same collective steps)."""
    import torch.distributed as dist

    world = len(plan)
    sizes = [e - b for b, e in plan]
    mx = max(max(sizes), 1)
    pad_o = torch.zeros((mx, *unit_shape), dtype=dtype, device=device)
    pad_l = torch.zeros((mx, *lse_unit_shape), dtype=torch.float32, device=device)
    n = sizes[rank]
    if n:
        pad_o[:n].copy_(out.reshape(n, *unit_shape))
        pad_l[:n].copy_(lse.reshape(n, *lse_unit_shape))
    go = [torch.empty_like(pad_o) for _ in range(world)] if rank == 0 else None
    gl = [torch.empty_like(pad_l) for _ in range(world)] if rank == 0 else None
    dist.gather(pad_o, go, dst=0, group=group)
    dist.gather(pad_l, gl, dst=0, group=group)
    if rank != 0:
        return None
    return (torch.cat([go[r][:sizes[r]] for r in range(world)], 0),
            torch.cat([gl[r][:sizes[r]] for r in range(world)], 0))
