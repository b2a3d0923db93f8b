"""CPU oracle for the sparse shared-KV attention forward (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs
of ``bench.py`` may import it.  The product path (``sparse_attn_sharedkv_b200``)
runs hand-written sm_100a CUDA and fails loudly when that library is missing.

It restates, in numpy fp32, the math of the reference oracle
``golden.py::sparse_attn_sharedkv_golden_bnsd`` (golden.py:69-204) directly on
the paged inputs the operator receives (no dense BNSD unpack):

* sliding window over ``ori_kv``: logical rows
  ``[max(s_g - ori_win_left, 0), s_g]`` with ``s_g = act_kv - act_q + s``
  (golden.py:125-131); ``ori_win_left = -1`` gives an empty window;
* compressed branch over ``cmp_kv``:
  - SCFA (top-k indices): ``_gather_cmp_kv_tokens`` semantics
    (golden.py:28-66): threshold ``floor((act_kv - act_q + s + 1) / ratio)``,
    scan the first ``min(K, threshold)`` entries, stop at ``-1``, skip
    ``id >= threshold``, drop ``id >= floor(act_kv / ratio)``;
  - CFA (dense): rows ``[0, max(threshold, 0))`` (golden.py:146-150);
* online softmax seeded by the per-head sink (``m = sink``, ``l = 1``,
  golden.py:156-164), walked in tiles of 512 keys, ori tiles first, then cmp
  tiles (golden.py:166-196); P is rounded to the input dtype before P.V while
  the row sum uses the unrounded fp32 P (golden.py:192-195);
* ``out = acc / l`` cast to the input dtype, ``lse = m + ln(l)``
  (golden.py:198-200).  Padded BSND slots (``s >= act_q``) stay zero.

Extensions the reference golden also supports unchanged (verified against it):
``head_dim_v < head_dim`` (output = first ``d_v`` columns of ``P.K``), any
number of query heads, ``block_size`` 64, ``sinks = -inf``.

Negative indices other than ``-1`` are treated as masked entries (the golden
would wrap them around the dense tensor, which has no paged meaning), and a
block-table entry of ``-1`` under an attended position reads as a zero row.
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

GOLDEN_S2_TILE = 512  # golden.py:25


# --------------------------------------------------------------------------
# bf16 / fp16 helpers (round-to-nearest-even, like torch's .to(dtype)).
# --------------------------------------------------------------------------

def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 (exact)."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> uint16 bf16 bit patterns, round to nearest even."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    r = r.astype(np.uint16)
    if nan.any():
        r[nan] = 0x7FC0
    return r


def round_to_dtype(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` ('bf16' or 'fp16') and back to float32."""
    if dtype == "bf16":
        return bf16_bits_to_f32(f32_to_bf16_bits(x))
    if dtype == "fp16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "fp32":
        return x.astype(np.float32)
    raise ValueError(f"unsupported dtype {dtype}")


# --------------------------------------------------------------------------
# Index semantics.
# --------------------------------------------------------------------------

def floor_div(a: int, b: int) -> int:
    """math.floor(a / b) for integers (golden.py:44 uses float floor)."""
    return a // b


def cmp_threshold(act_kv: int, act_q: int, s: int, ratio: int) -> int:
    """Causal limit of the compressed branch for query ``s`` (golden.py:44, 147)."""
    return floor_div(act_kv - act_q + s + 1, ratio)


def scfa_positions(idx_row: np.ndarray, act_kv: int, act_q: int, s: int,
                   ratio: int) -> List[int]:
    """Compressed-cache positions attended by one query (golden.py:28-66).

    ``idx_row`` is the ``K`` top-k entries of this query (int32).
    """
    K = int(idx_row.shape[0])
    cmp_act_kv = floor_div(act_kv, ratio)
    thr = cmp_threshold(act_kv, act_q, s, ratio)
    valid = min(K, thr)  # ceil(thr / sparse_block_size) with block size 1
    out: List[int] = []
    for i in range(max(valid, 0)):
        tid = int(idx_row[i])
        if tid == -1:
            break
        if tid < 0:
            continue  # malformed entry: masked (see module docstring)
        end = min(tid + 1, cmp_act_kv, thr)
        if tid >= thr or end <= tid:
            continue
        out.append(tid)
    return out


def window_positions(act_kv: int, act_q: int, s: int, win_left: int) -> Tuple[int, int]:
    """Half-open logical range of the sliding window (golden.py:128-131)."""
    s_g = act_kv - act_q + s
    lo = max(s_g - win_left, 0)
    hi = s_g + 1
    return lo, max(hi, lo)


def paged_rows(pool: np.ndarray, table_row: np.ndarray, positions: Sequence[int]) -> np.ndarray:
    """Fetch logical rows ``positions`` through one block-table row.

    ``pool``: [num_blocks, block_size, D] float32 (the single KV head squeezed).
    """
    bs = pool.shape[1]
    pos = np.asarray(positions, dtype=np.int64)
    if pos.size == 0:
        return np.zeros((0, pool.shape[2]), dtype=np.float32)
    phys = table_row[pos // bs].astype(np.int64)
    rows = pool[np.maximum(phys, 0), pos % bs]
    # An unmapped page (table entry -1) reads as zeros, like the zero-filled
    # dense unpack of golden.py:247-268.
    rows[phys < 0] = 0.0
    return rows


# --------------------------------------------------------------------------
# The forward pass.
# --------------------------------------------------------------------------

def _online_softmax(q: np.ndarray, tiles: List[np.ndarray], sink: np.ndarray,
                    scale: float, dtype: str, d_v: int) -> Tuple[np.ndarray, np.ndarray]:
    """Tile walk of golden.py:162-200 for one query token (all heads)."""
    G = q.shape[0]
    m = sink.astype(np.float32).copy()
    l = np.ones(G, dtype=np.float32)
    acc = np.zeros((G, d_v), dtype=np.float32)
    with np.errstate(over="ignore", invalid="ignore"):
        for k in tiles:
            if k.shape[0] == 0:
                continue
            sc = (q @ k.T) * np.float32(scale)
            m_old = m
            m = np.maximum(m_old, sc.max(axis=1))
            alpha = np.exp(m_old - m)
            p = np.exp(sc - m[:, None])
            l = alpha * l + p.sum(axis=1, dtype=np.float32)
            p_low = round_to_dtype(p, dtype)
            acc = acc * alpha[:, None] + p_low @ k[:, :d_v]
        out = acc / l[:, None]
        lse = m + np.log(l)
    return out.astype(np.float32), lse.astype(np.float32)


def token_key_rows(*, b: int, s: int, act_q: int, act_kv: int,
                   ori_pool: np.ndarray, ori_table: np.ndarray,
                   cmp_pool: Optional[np.ndarray], cmp_table: Optional[np.ndarray],
                   idx_row: Optional[np.ndarray], ratio: int,
                   win_left: int) -> Tuple[np.ndarray, np.ndarray]:
    """(window rows, compressed rows) attended by query ``(b, s)``."""
    lo, hi = window_positions(act_kv, act_q, s, win_left)
    ori_k = paged_rows(ori_pool, ori_table[b], range(lo, hi))
    if cmp_pool is None:
        cmp_k = np.zeros((0, ori_pool.shape[2]), dtype=np.float32)
    elif idx_row is not None:
        cmp_k = paged_rows(cmp_pool, cmp_table[b],
                           scfa_positions(idx_row, act_kv, act_q, s, ratio))
    else:
        thr = max(cmp_threshold(act_kv, act_q, s, ratio), 0)
        cmp_k = paged_rows(cmp_pool, cmp_table[b], range(thr))
    return ori_k, cmp_k


def forward(*, q: np.ndarray, ori_kv: np.ndarray, ori_block_table: np.ndarray,
            seqused_kv: Sequence[int], sinks: np.ndarray, softmax_scale: float,
            layout_q: str = "TND", cu_seqlens_q: Optional[Sequence[int]] = None,
            cmp_kv: Optional[np.ndarray] = None, cmp_block_table: Optional[np.ndarray] = None,
            cmp_sparse_indices: Optional[np.ndarray] = None, cmp_ratio: int = 4,
            ori_win_left: int = 127, head_dim_v: Optional[int] = None, dtype: str = "bf16",
            tokens: Optional[Sequence[int]] = None, s2_tile: int = GOLDEN_S2_TILE,
            out_dtype: Optional[str] = None) -> Tuple[np.ndarray, np.ndarray]:
    """Oracle forward on paged inputs.

    Arguments mirror ``api.sparse_attn_sharedkv`` (api.py:129-153) with numpy
    float32 values (already rounded to the input dtype):

    * ``q``: ``[T, N1, D]`` (TND) or ``[B, S, N1, D]`` (BSND);
    * ``ori_kv`` / ``cmp_kv``: ``[blocks, block_size, 1, D]``;
    * block tables ``[B, table_len]`` int32 (``-1`` unused);
    * ``cmp_sparse_indices``: ``[T, 1, K]`` (TND) or ``[B, S, 1, K]`` (BSND);
    * ``tokens``: optional subset of flat token ids to compute (others zero);
    * ``out_dtype``: rounding of the output (default ``dtype``, as golden.py:198;
      ``"fp32"`` keeps the unrounded fp32 result, the reference an accuracy
      gate measures against).

    Returns ``(out, lse)`` as float32 arrays in q's layout (out rounded to
    ``dtype``), ``out[..., :head_dim_v]`` and ``lse [T, N1]`` / ``[B, S, N1]``.
    """
    D = q.shape[-1]
    d_v = D if head_dim_v is None else int(head_dim_v)
    N1 = q.shape[-2]
    if ori_kv.shape[2] != 1:
        raise ValueError("only one KV head (N2=1) is supported")
    ori_pool = ori_kv[:, :, 0, :]
    cmp_pool = cmp_kv[:, :, 0, :] if cmp_kv is not None else None

    if layout_q == "TND":
        if cu_seqlens_q is None:
            raise ValueError("cu_seqlens_q is required for TND")
        cu = [int(x) for x in cu_seqlens_q]
        B = len(cu) - 1
        q_flat = q
        starts = cu[:-1]
        act_q_lens = [cu[i + 1] - cu[i] for i in range(B)]
        idx_flat = cmp_sparse_indices[:, 0, :] if cmp_sparse_indices is not None else None
        T = q.shape[0]
        S_stride = None
    else:
        B, S_max = q.shape[0], q.shape[1]
        T = B * S_max
        q_flat = q.reshape(T, N1, D)
        starts = [b * S_max for b in range(B)]
        if cu_seqlens_q is not None:
            cu = [int(x) for x in cu_seqlens_q]
            act_q_lens = [cu[i + 1] - cu[i] for i in range(B)]
        else:
            act_q_lens = [S_max] * B
        idx_flat = (cmp_sparse_indices.reshape(T, cmp_sparse_indices.shape[-1])
                    if cmp_sparse_indices is not None else None)
        S_stride = S_max

    out = np.zeros((T, N1, d_v), dtype=np.float32)
    lse = np.zeros((T, N1), dtype=np.float32)
    want = None if tokens is None else set(int(t) for t in tokens)
    sinks = np.asarray(sinks, dtype=np.float32)

    for b in range(B):
        act_q, act_kv = act_q_lens[b], int(seqused_kv[b])
        for s in range(act_q):
            t = starts[b] + s
            if want is not None and t not in want:
                continue
            ori_k, cmp_k = token_key_rows(
                b=b, s=s, act_q=act_q, act_kv=act_kv, ori_pool=ori_pool,
                ori_table=ori_block_table, cmp_pool=cmp_pool, cmp_table=cmp_block_table,
                idx_row=idx_flat[t] if idx_flat is not None else None,
                ratio=cmp_ratio, win_left=ori_win_left)
            tiles = [ori_k[i:i + s2_tile] for i in range(0, ori_k.shape[0], s2_tile)]
            tiles += [cmp_k[i:i + s2_tile] for i in range(0, cmp_k.shape[0], s2_tile)]
            o, ls = _online_softmax(q_flat[t].astype(np.float32), tiles, sinks,
                                    softmax_scale, dtype, d_v)
            out[t] = round_to_dtype(o, out_dtype or dtype)
            lse[t] = ls

    if layout_q == "BSND":
        out = out.reshape(B, S_stride, N1, d_v)
        lse = lse.reshape(B, S_stride, N1)
    return out, lse


def one_shot(q_tok: np.ndarray, k_rows: np.ndarray, sinks: np.ndarray, scale: float,
             dtype: str, d_v: int) -> Tuple[np.ndarray, np.ndarray]:
    """Single-shot ``softmax(scores U sinks) @ V`` for one token (golden.py:207-244).

    Used to pin the tiled walk (the reference's own
    ``test_golden_math_matches_single_shot_softmax``).
    """
    q = q_tok.astype(np.float32)
    sc = (q @ k_rows.T) * np.float32(scale)
    snk = np.asarray(sinks, dtype=np.float32)[:, None]
    xmax = np.maximum(sc.max(axis=1, keepdims=True) if sc.shape[1] else snk, snk)
    y = np.exp(sc - xmax)
    den = y.sum(axis=1, keepdims=True) + np.exp(snk - xmax)
    p = round_to_dtype(y / den, dtype)
    out = round_to_dtype(p @ k_rows[:, :d_v], dtype)
    return out, (xmax + np.log(den))[:, 0]


# --------------------------------------------------------------------------
# Algorithmic work accounting (FLOPs / bytes per call).
# --------------------------------------------------------------------------

def count_keys(*, layout_q: str, cu_seqlens_q: Optional[Sequence[int]], B: int, S: int,
               seqused_kv: Sequence[int], cmp_sparse_indices: Optional[np.ndarray],
               has_cmp: bool, cmp_ratio: int, ori_win_left: int) -> Dict[str, int]:
    """Valid keys per call (window + compressed, after masks and -1 handling)."""
    if layout_q == "TND":
        cu = [int(x) for x in cu_seqlens_q]
        starts, lens = cu[:-1], [cu[i + 1] - cu[i] for i in range(len(cu) - 1)]
    else:
        starts = [b * S for b in range(B)]
        lens = ([int(cu_seqlens_q[i + 1]) - int(cu_seqlens_q[i]) for i in range(B)]
                if cu_seqlens_q is not None else [S] * B)
    idx = None
    if cmp_sparse_indices is not None:
        idx = cmp_sparse_indices.reshape(-1, cmp_sparse_indices.shape[-1])
    win = cmpk = tokens = 0
    for b, (st, aq) in enumerate(zip(starts, lens)):
        akv = int(seqused_kv[b])
        for s in range(aq):
            tokens += 1
            lo, hi = window_positions(akv, aq, s, ori_win_left)
            win += hi - lo
            if has_cmp:
                if idx is not None:
                    cmpk += len(scfa_positions(idx[st + s], akv, aq, s, cmp_ratio))
                else:
                    cmpk += max(cmp_threshold(akv, aq, s, cmp_ratio), 0)
    return {"tokens": tokens, "window_keys": win, "cmp_keys": cmpk, "keys": win + cmpk}


# ---------------------------------------------------------------------------
# Paged-cache writer (the step before the attention path).
# ---------------------------------------------------------------------------

def append_paged(pool: np.ndarray, block_table: np.ndarray, rows: np.ndarray,
                 cu_new: Sequence[int], start_pos: Sequence[int]) -> List[int]:
    """Write new key rows into a paged cache, in place.

    The paged layout is the reference's (golden.py:315-360, inverse of
    ``unpack_paged_kv``, golden.py:247-268): logical position ``p`` of batch
    ``b`` lives at ``pool[block_table[b, p // bs], p % bs]``.  Batch ``b``
    appends ``rows[cu_new[b]:cu_new[b+1]]`` at positions ``start_pos[b] + i``.
    ``pool`` is ``[blocks, bs, D]`` (the N2 = 1 axis dropped), ``rows``
    ``[T_new, D]``; any dtype (the writer copies bits).

    Returns the indices of the new rows that could not be written (position
    past the block table, or an unmapped / out-of-pool page); those rows are
    skipped, as the CUDA writer does.
    """
    blocks, bs = pool.shape[0], pool.shape[1]
    table_len = block_table.shape[1]
    bad = []
    for b in range(len(cu_new) - 1):
        for i in range(int(cu_new[b]), int(cu_new[b + 1])):
            pos = int(start_pos[b]) + (i - int(cu_new[b]))
            lb = pos // bs
            blk = int(block_table[b, lb]) if 0 <= lb < table_len else -1
            if blk < 0 or blk >= blocks or pos < 0:
                bad.append(i)
                continue
            pool[blk, pos % bs] = rows[i]
    return bad
