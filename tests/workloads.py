"""Seeded synthetic inputs for the sparse shared-KV attention forward.

Two families:

* ``baseline_case(i)`` builds the five workloads the benchmark is quoted on
  (decode / SWA prefill / DeepSeek-V3.2-shape sparse decode / sparse prefill /
  SWA + top-k decode).  Shapes, value distributions and seeds follow the
  benchmark definition: Q and KV ``N(0,1) * 0.5`` in bf16, ``d_qk = 576``,
  ``d_v = 512``, one KV head, paged with ``block_size = 64`` through a random
  permutation of physical blocks.
* ``reference_scenario_case(name)`` regenerates, tensor for tensor, the inputs
  of the reference test suite's ``_build_case``
  (test_sparse_attn_sharedkv.py:238-391, generators golden.py:315-473): the
  same torch / numpy RNG calls in the same order, so the reference golden's
  outputs for those inputs can be committed as fixtures and re-checked on a
  machine without the reference.

Everything is generated with torch (CPU generators are deterministic across
machines with the same torch build; CUDA generators are used for the large
benchmark inputs).  All tensors are returned on ``device``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np
import torch


@dataclass
class Case:
    """One call's worth of operator inputs (reference argument names)."""

    name: str
    layout_q: str
    q: torch.Tensor                      # [T,H,D] (TND) or [B,S,H,D] (BSND)
    ori_kv: torch.Tensor                 # [nblk, bs, 1, D]
    ori_block_table: torch.Tensor        # [B, tl] int32
    seqused_kv: torch.Tensor             # [B] int32
    sinks: torch.Tensor                  # [H] fp32
    softmax_scale: float
    cu_seqlens_q: Optional[torch.Tensor] = None   # [B+1] int32
    cmp_kv: Optional[torch.Tensor] = None
    cmp_block_table: Optional[torch.Tensor] = None
    cmp_sparse_indices: Optional[torch.Tensor] = None  # [T,1,K] / [B,S,1,K]
    cmp_ratio: Optional[int] = None
    ori_win_left: int = 127
    head_dim_v: Optional[int] = None
    meta: Dict = field(default_factory=dict)

    @property
    def batch(self) -> int:
        return int(self.seqused_kv.numel())

    def kwargs(self) -> Dict:
        """Keyword arguments of ``sparse_attn_sharedkv`` (without ``q``)."""
        kw = dict(ori_kv=self.ori_kv, ori_block_table=self.ori_block_table,
                  cu_seqlens_q=self.cu_seqlens_q, seqused_kv=self.seqused_kv,
                  sinks=self.sinks, softmax_scale=self.softmax_scale,
                  ori_win_left=self.ori_win_left, layout_q=self.layout_q)
        if self.cmp_kv is not None:
            kw.update(cmp_kv=self.cmp_kv, cmp_block_table=self.cmp_block_table,
                      cmp_ratio=self.cmp_ratio)
        if self.cmp_sparse_indices is not None:
            kw["cmp_sparse_indices"] = self.cmp_sparse_indices
        if self.head_dim_v is not None:
            kw["head_dim_v"] = self.head_dim_v
        return kw

    def to(self, device) -> "Case":
        def mv(t):
            return t.to(device) if isinstance(t, torch.Tensor) else t
        c = Case(**{k: mv(v) for k, v in self.__dict__.items()})
        return c


# --------------------------------------------------------------------------
# Paged-pool helpers.
# --------------------------------------------------------------------------

def paged_pool_from_dense(dense: torch.Tensor, lengths: List[int], block_size: int,
                          num_blocks: int, perm: torch.Tensor) -> tuple:
    """Scatter ``dense [B, L, D]`` rows into a paged pool through ``perm``.

    Logical block ``i`` of batch ``b`` goes to physical block
    ``perm[cursor]`` with the cursor advancing batch by batch (the placement
    rule of golden.py:342-358).  Unused table entries are ``-1``.
    """
    B, L, D = dense.shape
    per = [math.ceil(n / block_size) for n in lengths]
    max_blk = max(max(per) if per else 0, 1)
    if sum(per) > num_blocks:
        raise ValueError(f"pool too small: {num_blocks} < {sum(per)}")
    table = torch.full((B, max_blk), -1, dtype=torch.int32)
    pool = torch.zeros((num_blocks, block_size, 1, D), dtype=dense.dtype, device=dense.device)
    cursor = 0
    perm = perm.to(torch.int64).cpu()
    for b, nb in enumerate(per):
        ids = perm[cursor:cursor + nb]
        table[b, :nb] = ids.to(torch.int32)
        cursor += nb
        n = lengths[b]
        if nb == 0:
            continue
        src = torch.zeros((nb * block_size, D), dtype=dense.dtype, device=dense.device)
        src[:n] = dense[b, :n]
        pool[ids.to(dense.device), :, 0, :] = src.view(nb, block_size, D)
    return pool, table.to(dense.device)


def _normal(shape, gen, device, std=0.5, dtype=torch.bfloat16):
    return (torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std).to(dtype)


def _sorted_unique_topk(lengths: torch.Tensor, L_max: int, K: int, gen, device) -> torch.Tensor:
    """Per row: ``min(K, len)`` distinct uniform positions in ``[0, len)``,
    sorted ascending, ``-1`` padded.  ``lengths [R]`` on ``device``."""
    R = lengths.numel()
    keys = torch.rand((R, L_max), generator=gen, device=device)
    pos = torch.arange(L_max, device=device)
    keys = keys.masked_fill(pos[None, :] >= lengths[:, None], 2.0)
    k_eff = min(K, L_max)
    sel = torch.topk(keys, k_eff, dim=1, largest=False).indices
    valid = torch.gather(keys, 1, sel) < 2.0
    sel = torch.where(valid, sel, torch.full_like(sel, L_max + 1))
    sel = torch.sort(sel, dim=1).values
    sel = torch.where(sel > L_max, torch.full_like(sel, -1), sel)
    if k_eff < K:
        pad = torch.full((R, K - k_eff), -1, dtype=sel.dtype, device=device)
        sel = torch.cat([sel, pad], dim=1)
    return sel.to(torch.int32)


# --------------------------------------------------------------------------
# The five benchmark workloads.
# --------------------------------------------------------------------------

BASELINE_NAMES = [
    "cfg1_decode_b2_h16_topk512",
    "cfg2_swa_prefill_tnd_t7680_h64",
    "cfg3_sparse_mla_decode_b64_h128_topk2048",
    "cfg4_sparse_prefill_tnd_t32768_h128_topk2048",
    "cfg5_swa_topk_decode_b256_h64",
]

D_QK, D_V, BLOCK = 576, 512, 64


def baseline_case(i: int, device="cpu", *, scale_down: int = 1,
                  minus_one_variant: bool = False, sequences: Optional[int] = None) -> Case:
    """Benchmark workload ``i`` (0-based index into the five configs).

    ``scale_down > 1`` shrinks the token / batch counts (keeping head count,
    head dims, block size and index density) for CPU-checkable parity runs.
    ``minus_one_variant`` shortens some sequences of the decode configs so the
    ``-1`` index padding path is exercised.  ``sequences`` (config 4 only)
    keeps that many of its 4096-token sequences, everything else unchanged
    (profiling captures of a few GB).
    """
    device = torch.device(device)
    seed = i
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    scale = 1.0 / math.sqrt(D_QK)

    if i == 0:  # decode B=2 H=16, L=4096, top-k 512, 128 blocks
        B, H, L, K = 2, 16, 4096, 512
        nblk = 128
        lengths = [L] * B
        q = _normal((B, 1, H, D_QK), gen, device)
        dense = _normal((B, L, D_QK), gen, device)
        perm = torch.randperm(nblk, generator=gen, device=device)
        pool, table = paged_pool_from_dense(dense, lengths, BLOCK, nblk, perm)
        idx = _sorted_unique_topk(torch.tensor(lengths, device=device), L, K, gen, device)
        return Case(BASELINE_NAMES[0], "BSND", q, pool, table,
                    torch.tensor(lengths, dtype=torch.int32, device=device),
                    torch.full((H,), float("-inf"), device=device), scale,
                    cmp_kv=pool, cmp_block_table=table,
                    cmp_sparse_indices=idx.view(B, 1, 1, K), cmp_ratio=1,
                    ori_win_left=-1, head_dim_v=D_V, meta=dict(K=K))

    if i == 1:  # SWA prefill TND lens {512,1024,2048,4096}, H=64, window 128
        lens = [512, 1024, 2048, 4096]
        if scale_down > 1:
            lens = [max(64, n // scale_down) for n in lens]
        H = 64
        B = len(lens)
        T = sum(lens)
        cu = [0]
        for n in lens:
            cu.append(cu[-1] + n)
        q = _normal((T, H, D_QK), gen, device)
        Lm = max(lens)
        dense = _normal((B, Lm, D_QK), gen, device)
        nblk = sum(math.ceil(n / BLOCK) for n in lens)
        perm = torch.randperm(nblk, generator=gen, device=device)
        pool, table = paged_pool_from_dense(dense, lens, BLOCK, nblk, perm)
        return Case(BASELINE_NAMES[1], "TND", q, pool, table,
                    torch.tensor(lens, dtype=torch.int32, device=device),
                    torch.full((H,), float("-inf"), device=device), scale,
                    cu_seqlens_q=torch.tensor(cu, dtype=torch.int32, device=device),
                    ori_win_left=127, head_dim_v=D_V)

    if i == 2:  # sparse MLA decode B=64 H=128 top-k 2048, L ~ U[8192, 32768]
        B, H, K = 64, 128, 2048
        lo, hi = 8192, 32768
        if scale_down > 1:
            B = max(2, B // scale_down)
            lo, hi = max(256, lo // scale_down), max(512, hi // scale_down)
        lengths = torch.randint(lo, hi + 1, (B,), generator=gen, device=device)
        if minus_one_variant:
            lengths[: B // 2] = torch.randint(K // 4, K, (B // 2,), generator=gen, device=device)
        lens = [int(x) for x in lengths.tolist()]
        q = _normal((B, 1, H, D_QK), gen, device)
        nblk = sum(math.ceil(n / BLOCK) for n in lens)
        perm = torch.randperm(nblk, generator=gen, device=device)
        pool, table = _pool_random_fill(lens, BLOCK, nblk, perm, gen, device)
        idx = _sorted_unique_topk(lengths, max(lens), K, gen, device)
        return Case(BASELINE_NAMES[2], "BSND", q, pool, table,
                    torch.tensor(lens, dtype=torch.int32, device=device),
                    torch.full((H,), float("-inf"), device=device), scale,
                    cmp_kv=pool, cmp_block_table=table,
                    cmp_sparse_indices=idx.view(B, 1, 1, K), cmp_ratio=1,
                    ori_win_left=-1, head_dim_v=D_V, meta=dict(K=K))

    if i == 3:  # sparse prefill TND 8 x 4096, H=128, top-k 2048 from [0, pos]
        nseq, L, H, K = 8, 4096, 128, 2048
        if sequences is not None:
            nseq = int(sequences)
        if scale_down > 1:
            nseq = max(1, nseq // scale_down)
            L = max(256, L // scale_down)
            K = max(64, K // scale_down)
        lens = [L] * nseq
        T = nseq * L
        cu = [k * L for k in range(nseq + 1)]
        q = _normal((T, H, D_QK), gen, device)
        nblk = sum(math.ceil(n / BLOCK) for n in lens)
        perm = torch.randperm(nblk, generator=gen, device=device)
        pool, table = _pool_random_fill(lens, BLOCK, nblk, perm, gen, device)
        pos = torch.arange(L, device=device).repeat(nseq)
        idx = _sorted_unique_topk(pos + 1, L, K, gen, device)
        return Case(BASELINE_NAMES[3], "TND", q, pool, table,
                    torch.tensor(lens, dtype=torch.int32, device=device),
                    torch.full((H,), float("-inf"), device=device), scale,
                    cu_seqlens_q=torch.tensor(cu, dtype=torch.int32, device=device),
                    cmp_kv=pool, cmp_block_table=table,
                    cmp_sparse_indices=idx.view(T, 1, K), cmp_ratio=1,
                    ori_win_left=-1, head_dim_v=D_V, meta=dict(K=K))

    if i == 4:  # SWA 128 over L=131072 + top-k 2048 over the 4x cache (32768)
        B, H, K, L, ratio = 256, 64, 2048, 131072, 4
        if scale_down > 1:
            B = max(2, B // scale_down)
            L = max(4096, L // scale_down)
        Lc = L // ratio
        lens = [L] * B
        q = _normal((B, 1, H, D_QK), gen, device)
        # Only the pages the window can reach are materialised: the last
        # ceil(128/64)+1 logical blocks of every sequence; the rest of the
        # table is -1 (never read: the window is the last 128 positions).
        nb_log = math.ceil(L / BLOCK)
        win_blocks = 3
        nblk = B * win_blocks
        perm = torch.randperm(nblk, generator=gen, device=device)
        table = torch.full((B, nb_log), -1, dtype=torch.int32, device=device)
        table[:, nb_log - win_blocks:] = perm.view(B, win_blocks).to(torch.int32)
        pool = _normal((nblk, BLOCK, 1, D_QK), gen, device)
        nblk_c = B * math.ceil(Lc / BLOCK)
        perm_c = torch.randperm(nblk_c, generator=gen, device=device)
        cpool, ctable = _pool_random_fill([Lc] * B, BLOCK, nblk_c, perm_c, gen, device)
        idx = _sorted_unique_topk(torch.full((B,), Lc, device=device), Lc, K, gen, device)
        return Case(BASELINE_NAMES[4], "BSND", q, pool, table,
                    torch.tensor(lens, dtype=torch.int32, device=device),
                    torch.full((H,), float("-inf"), device=device), scale,
                    cmp_kv=cpool, cmp_block_table=ctable,
                    cmp_sparse_indices=idx.view(B, 1, 1, K), cmp_ratio=ratio,
                    ori_win_left=127, head_dim_v=D_V, meta=dict(K=K))

    raise ValueError(f"no baseline config {i}")


def _pool_random_fill(lengths: List[int], block_size: int, num_blocks: int, perm: torch.Tensor,
                      gen, device) -> tuple:
    """Random ``N(0,1)*0.5`` pool whose table maps each sequence's logical
    blocks to ``perm`` in order (values need no dense staging copy)."""
    per = [math.ceil(n / block_size) for n in lengths]
    B = len(lengths)
    table = torch.full((B, max(max(per), 1)), -1, dtype=torch.int32, device=device)
    cursor = 0
    for b, nb in enumerate(per):
        table[b, :nb] = perm[cursor:cursor + nb].to(torch.int32)
        cursor += nb
    pool = _normal((num_blocks, block_size, 1, D_QK), gen, device)
    return pool, table


# --------------------------------------------------------------------------
# Reference test-suite scenarios (D = 512, N1 = 64, K == V).
# --------------------------------------------------------------------------

_REF_COMMON = dict(layout_q="TND", B=1, N1=64, N2=1, D=512, softmax_scale=0.04419417,
                   ori_win_left=127, ori_win_right=0, ori_mask_mode=4, cmp_mask_mode=3)

# Shapes of test_sparse_attn_sharedkv.py:81-220 (decode: S1=1, seqused 8193).
REFERENCE_SCENARIOS = {
    "scfa_decode": dict(_REF_COMMON, scenario=3, S1=1, T1=1, K=512, block_num1=65,
                        block_num2=17, block_size1=128, block_size2=128,
                        cu_seqlens_q=[0, 1], seqused_kv=[8193], cmp_ratio=4),
    "swa_decode": dict(_REF_COMMON, scenario=1, S1=1, T1=1, K=0, block_num1=65,
                       block_num2=1, block_size1=128, block_size2=1,
                       cu_seqlens_q=[0, 1], seqused_kv=[8193], cmp_ratio=4),
    "cfa_decode": dict(_REF_COMMON, scenario=2, S1=1, T1=1, K=512, block_num1=65,
                       block_num2=17, block_size1=128, block_size2=128,
                       cu_seqlens_q=[0, 1], seqused_kv=[8193], cmp_ratio=128),
    # Full-length prefills (S1 = 8192), test_sparse_attn_sharedkv.py:105-128,
    # 151-174, 197-220.
    "scfa_prefill": dict(_REF_COMMON, scenario=3, S1=8192, T1=8192, K=512, block_num1=65,
                         block_num2=17, block_size1=128, block_size2=128,
                         cu_seqlens_q=[0, 8192], seqused_kv=[8192], cmp_ratio=4),
    "swa_prefill": dict(_REF_COMMON, scenario=1, S1=8192, T1=8192, K=0, block_num1=65,
                        block_num2=1, block_size1=128, block_size2=1,
                        cu_seqlens_q=[0, 8192], seqused_kv=[8192], cmp_ratio=4),
    "cfa_prefill": dict(_REF_COMMON, scenario=2, S1=8192, T1=8192, K=512, block_num1=65,
                        block_num2=17, block_size1=128, block_size2=128,
                        cu_seqlens_q=[0, 8192], seqused_kv=[8192], cmp_ratio=128),
}


def _shrink(name: str, s1: int) -> dict:
    """Small-S1 prefill shape derivation of test_sparse_attn_sharedkv_fast.py:84-104."""
    base = {"swa": "swa_decode", "cfa": "cfa_decode", "scfa": "scfa_decode"}[name]
    cfg = dict(REFERENCE_SCENARIOS[base])
    cfg.update(S1=s1, T1=s1, cu_seqlens_q=[0, s1], seqused_kv=[s1])
    cfg["block_num1"] = math.ceil(s1 / cfg["block_size1"]) + 2
    if cfg["scenario"] >= 2:
        cfg["block_num2"] = max(1, math.ceil((s1 // cfg["cmp_ratio"]) / cfg["block_size2"])) + 1
    return cfg


def _shrink_multibatch(name: str, seqs=(768, 512)) -> dict:
    """Ragged B=2 shape derivation of test_sparse_attn_sharedkv_fast.py:107-144."""
    base = {"swa": "swa_decode", "cfa": "cfa_decode", "scfa": "scfa_decode"}[name]
    cfg = dict(REFERENCE_SCENARIOS[base])
    cu = [0]
    for s in seqs:
        cu.append(cu[-1] + s)
    cfg.update(B=len(seqs), S1=max(seqs), T1=sum(seqs), cu_seqlens_q=cu, seqused_kv=list(seqs))
    cfg["block_num1"] = sum(math.ceil(s / cfg["block_size1"]) for s in seqs) + 2
    if cfg["scenario"] >= 2:
        cfg["block_num2"] = sum(max(1, math.ceil((s // cfg["cmp_ratio"]) / cfg["block_size2"]))
                                for s in seqs) + 1
    return cfg


for _n in ("swa", "cfa", "scfa"):
    REFERENCE_SCENARIOS[f"{_n}_prefill_fast"] = _shrink(_n, 1024)
    REFERENCE_SCENARIOS[f"{_n}_prefill_b2"] = _shrink_multibatch(_n)


def _ref_paged(B, N2, D, block_num, block_size, lengths, dtype, lo, hi, rng, fill_len=None):
    """Paged pool + table with the RNG call order of golden.py:315-408.

    ``lengths`` fix the table; ``fill_len`` the rows copied into the pool
    (the compressed generator copies ``cmp_seqs[b]`` rows, the window
    generator copies up to ``max_s``)."""
    max_s = max(lengths) if lengths else 0
    dense = (torch.rand((B, N2, max(max_s, 1), D)) * (hi - lo) + lo).to(dtype)
    per = [math.ceil(s / block_size) if s > 0 else 0 for s in lengths]
    if block_num < max(sum(per), 1):
        raise ValueError("block_num too small")
    phys = rng.permutation(block_num).astype(np.int32)
    max_blk = max(math.ceil(max_s / block_size) if max_s > 0 else 1, 1)
    table = np.full((B, max_blk), -1, dtype=np.int32)
    cursor = 0
    for b, nb in enumerate(per):
        for i in range(nb):
            table[b, i] = phys[cursor]
            cursor += 1
    pool = torch.zeros((block_num, block_size, N2, D), dtype=dtype)
    for b in range(B):
        cap = fill_len[b] if fill_len is not None else max_s
        for i in range(per[b]):
            s0 = i * block_size
            s1 = min(s0 + block_size, cap)
            if s1 > s0:
                pool[int(table[b, i]), : s1 - s0] = dense[b, :, s0:s1, :].permute(1, 0, 2)
    return pool, torch.tensor(table, dtype=torch.int32)


def reference_scenario_case(name: str, dtype=torch.bfloat16, seed: int = 42) -> Case:
    """Inputs of the reference suite's ``_build_case(cfg, dtype, seed)``.

    Reproduces the RNG sequence of test_sparse_attn_sharedkv.py:243-326:
    Q, window pool (numpy rng ``seed``), compressed pool (rng ``seed+1``),
    indices (torch generator ``seed+7``, a fresh ``randperm`` per query), sinks.
    """
    cfg = REFERENCE_SCENARIOS[name]
    torch.manual_seed(seed)
    np.random.seed(seed)
    B, T1, N1, N2, D = cfg["B"], cfg["T1"], cfg["N1"], cfg["N2"], cfg["D"]
    K, ratio, scen = cfg["K"], cfg["cmp_ratio"], cfg["scenario"]
    seqused = cfg["seqused_kv"]
    cu = cfg["cu_seqlens_q"]
    q = (torch.rand((T1, N1, D)) * 20 - 10).to(dtype)
    ori, ori_bt = _ref_paged(B, N2, D, cfg["block_num1"], cfg["block_size1"], seqused, dtype,
                             -10, 10, np.random.default_rng(seed))
    cmp_kv = cmp_bt = idx = None
    if scen >= 2:
        cmp_seqs = [s // ratio for s in seqused]
        cmp_kv, cmp_bt = _ref_paged(B, N2, D, cfg["block_num2"], cfg["block_size2"], cmp_seqs,
                                    dtype, -5, 10, np.random.default_rng(seed + 1),
                                    fill_len=cmp_seqs)
    if scen == 3:
        g = torch.Generator()
        g.manual_seed(seed + 7)
        idx = torch.full((T1, N2, K), -1, dtype=torch.int32)
        for b in range(B):
            s_start, s_end = cu[b], cu[b + 1]
            act_q = s_end - s_start
            for s in range(act_q):
                cur = max(0, (seqused[b] - act_q + s + 1) // ratio)
                perm = (torch.randperm(cur, generator=g).to(torch.int32) if cur > 0
                        else torch.empty((0,), dtype=torch.int32))
                take = min(cur, K)
                idx[s_start + s, 0, :take] = perm[:take]
    sinks = (torch.rand(N1) * 2 - 1).to(torch.float32)
    return Case(name, "TND", q, ori, ori_bt, torch.tensor(seqused, dtype=torch.int32), sinks,
                cfg["softmax_scale"], cu_seqlens_q=torch.tensor(cu, dtype=torch.int32),
                cmp_kv=cmp_kv, cmp_block_table=cmp_bt, cmp_sparse_indices=idx,
                cmp_ratio=ratio if scen >= 2 else None, ori_win_left=cfg["ori_win_left"],
                meta=dict(scenario=scen, K=K, cfg=cfg))


# --------------------------------------------------------------------------
# Small random cases for parity sweeps.
# --------------------------------------------------------------------------

def random_case(*, seed: int, layout_q: str = "TND", B: int = 2, H: int = 64, D: int = 576,
                d_v: Optional[int] = 512, block_size: int = 64, scenario: int = 3,
                q_lens=(5, 3), kv_lens=(300, 700), K: int = 96, ratio: int = 4,
                win_left: int = 127, sinks: str = "random", dtype=torch.bfloat16,
                idx_mode: str = "perm", device="cpu") -> Case:
    """A small case of any scenario / layout (CPU-oracle sized).

    ``idx_mode``: ``perm`` (shuffled valid positions, -1 padded, like the
    reference generator), ``sorted`` (sorted unique), ``dirty`` (adds -1 in the
    middle, out-of-range and duplicate ids).
    """
    g = torch.Generator()
    g.manual_seed(seed)
    rng = np.random.default_rng(seed)
    q_lens = list(q_lens)[:B]
    kv_lens = list(kv_lens)[:B]
    if layout_q == "TND":
        cu = [0]
        for n in q_lens:
            cu.append(cu[-1] + n)
        T = cu[-1]
        q = (torch.randn((T, H, D), generator=g) * 0.5).to(dtype)
        cu_t = torch.tensor(cu, dtype=torch.int32)
        S = max(q_lens)
    else:
        S = max(q_lens)
        q = (torch.randn((B, S, H, D), generator=g) * 0.5).to(dtype)
        T = B * S
        cu_t = (torch.tensor(np.concatenate([[0], np.cumsum(q_lens)]), dtype=torch.int32)
                if any(n != S for n in q_lens) else None)
        cu = [b * S for b in range(B + 1)]
    Lm = max(kv_lens)
    dense = (torch.randn((B, Lm, D), generator=g) * 0.5).to(dtype)
    nblk = sum(math.ceil(n / block_size) for n in kv_lens) + 3
    perm = torch.from_numpy(rng.permutation(nblk).astype(np.int64))
    ori, ori_bt = paged_pool_from_dense(dense, kv_lens, block_size, nblk, perm)
    cmp_kv = cmp_bt = idx = None
    if scenario >= 2:
        cl = [n // ratio for n in kv_lens]
        cd = (torch.randn((B, max(max(cl), 1), D), generator=g) * 0.5).to(dtype)
        nb2 = sum(max(1, math.ceil(n / block_size)) for n in cl) + 2
        perm2 = torch.from_numpy(rng.permutation(nb2).astype(np.int64))
        cmp_kv, cmp_bt = paged_pool_from_dense(cd, cl, block_size, nb2, perm2)
    if scenario == 3:
        rows = []
        for b in range(B):
            aq, akv = q_lens[b], kv_lens[b]
            for s in range(S if layout_q == "BSND" else aq):
                cur = max(0, (akv - aq + s + 1) // ratio)
                r = np.full(K, -1, dtype=np.int32)
                if idx_mode == "sorted":
                    take = min(cur, K)
                    r[:take] = np.sort(rng.choice(cur, take, replace=False)) if take else []
                else:
                    p = rng.permutation(cur).astype(np.int32)
                    take = min(cur, K)
                    r[:take] = p[:take]
                if idx_mode.startswith("dirty") and K >= 8:
                    r[rng.integers(0, K)] = cur + 5          # beyond threshold
                    r[rng.integers(0, K)] = max(cur - 1, 0)  # duplicate-ish
                    if rng.random() < 0.5:
                        r[rng.integers(K // 2, K)] = -1      # early stop
                    if idx_mode == "dirty":
                        r[rng.integers(0, K)] = -7           # malformed negative
                rows.append(r)
        idx_np = np.stack(rows)
        if layout_q == "TND":
            idx = torch.from_numpy(idx_np).view(T, 1, K)
        else:
            idx = torch.from_numpy(idx_np).view(B, S, 1, K)
    if sinks == "random":
        snk = torch.rand(H, generator=g) * 2 - 1
    elif sinks == "-inf":
        snk = torch.full((H,), float("-inf"))
    else:
        snk = torch.full((H,), float(sinks))
    c = Case(f"random_s{seed}", layout_q, q, ori, ori_bt,
             torch.tensor(kv_lens, dtype=torch.int32), snk.to(torch.float32),
             1.0 / math.sqrt(D), cu_seqlens_q=cu_t if layout_q == "TND" else cu_t,
             cmp_kv=cmp_kv, cmp_block_table=cmp_bt, cmp_sparse_indices=idx,
             cmp_ratio=ratio if scenario >= 2 else None, ori_win_left=win_left,
             head_dim_v=d_v, meta=dict(scenario=scenario, K=K))
    return c.to(device)


# --------------------------------------------------------------------------
# Algorithmic work of one call.
# --------------------------------------------------------------------------

def accounting(case: Case) -> Dict:
    """Valid keys, FLOPs and compulsory HBM bytes of one forward call.

    * keys: attended (query, key) pairs after the window, threshold, ``-1``
      stop and range masks (golden.py:28-66, 125-150);
    * FLOPs: ``2 * H * keys * (d_qk + d_v)`` (QK^T and PV);
    * bytes: Q + O + LSE + indices + every distinct KV row touched (a row
      shared by several queries of a window is read once: compulsory traffic).
    Vectorised in torch on the case's device.
    """
    dev = case.q.device
    H = case.q.shape[-2]
    D = case.q.shape[-1]
    dv = case.head_dim_v or D
    B = case.batch
    if case.layout_q == "TND":
        cu = case.cu_seqlens_q.to(torch.int64).cpu()
        starts = cu[:-1]
        lens = cu[1:] - cu[:-1]
        T = int(case.q.shape[0])
    else:
        S = case.q.shape[1]
        T = B * S
        starts = torch.arange(B) * S
        lens = ((case.cu_seqlens_q[1:] - case.cu_seqlens_q[:-1]).cpu().to(torch.int64)
                if case.cu_seqlens_q is not None else torch.full((B,), S, dtype=torch.int64))
    kv = case.seqused_kv.to(torch.int64).cpu()
    # per valid token: batch, position
    tb = torch.repeat_interleave(torch.arange(B), lens)
    ts = torch.cat([torch.arange(int(n)) for n in lens]) if T else torch.zeros(0, dtype=torch.int64)
    tok = starts[tb] + ts
    aq, akv = lens[tb], kv[tb]
    s_g = akv - aq + ts
    wl = case.ori_win_left
    lo = torch.clamp(s_g - wl, min=0)
    hi = s_g + 1
    win = torch.clamp(hi - lo, min=0)
    keys = int(win.sum())
    uniq = 0
    # distinct window rows: windows of consecutive queries of a batch overlap
    for b in range(B):
        m = tb == b
        if m.any() and int(win[m].sum()) > 0:
            nz = win[m] > 0
            uniq += int(hi[m][nz].max() - lo[m][nz].min())
    cmp_keys = 0
    idx_bytes = 0
    if case.cmp_kv is not None:
        ratio = case.cmp_ratio
        thr = torch.div(akv - aq + ts + 1, ratio, rounding_mode="floor")
        if case.cmp_sparse_indices is not None:
            idx = case.cmp_sparse_indices.reshape(T, -1).to(dev)
            K = idx.shape[1]
            idx_bytes = T * K * 4
            idx = idx[tok.to(dev)]
            thr_d = thr.to(dev)
            ar = torch.arange(K, device=dev)
            in_rng = ar[None, :] < torch.clamp(thr_d, max=K)[:, None]
            m1 = (idx == -1) & in_rng
            before = (torch.cumsum(m1.to(torch.int32), dim=1) - m1.to(torch.int32)) > 0
            valid = in_rng & (idx >= 0) & (idx < thr_d[:, None]) & ~before
            cmp_keys = int(valid.sum())
            ids = (tb.to(dev)[:, None] * (1 << 32) + idx.to(torch.int64))[valid]
            uniq += int(torch.unique(ids).numel()) if ids.numel() else 0
        else:
            c = torch.clamp(thr, min=0)
            cmp_keys = int(c.sum())
            for b in range(B):
                m = tb == b
                if m.any():
                    uniq += int(c[m].max())
    keys += cmp_keys
    flops = 2.0 * H * keys * (D + dv)
    esz = case.q.element_size()
    nbytes = T * H * D * esz + T * H * dv * esz + T * H * 4 + idx_bytes + uniq * D * esz
    return dict(tokens=int(lens.sum()), keys=keys, window_keys=keys - cmp_keys,
                cmp_keys=cmp_keys, unique_kv_rows=uniq, flops=flops, bytes=nbytes)
