"""``sparse_attn_sharedkv_metadata``: the companion scheduler op.

Same signature and output as the reference's
``metadata.sparse_attn_sharedkv_metadata`` (metadata.py:1018-1086): an int32
tensor of ``SAS_META_SIZE = 1024`` entries holding
``faMetadata[36][8]`` (per AIC core: enable, bn2/m/s2 start, bn2/m/s2 end,
first FD workspace index) followed by ``fdMetadata[72][8]``.  The schedule is
computed by the C++ port in ``libsas.so`` (``sas_metadata``), bit-exact with
the reference's Python port of the aicpu kernel.

The B200 forward does not execute this table (148 SMs do not fit its 36
rows); it plans its own split-KV work (``sas_plan``).  The table is accepted
by ``sparse_attn_sharedkv(metadata=...)`` for API parity, as in the reference
whose kernels also leave it unused (kernel.py:367, 1851, 3416).
"""

from __future__ import annotations

import ctypes as C
from typing import Optional

import torch

from . import _lib

SAS_META_SIZE = _lib.SAS_META_SIZE
AIC_CORE_NUM = _lib.SAS_AIC_CORE_NUM
AIV_CORE_NUM = _lib.SAS_AIV_CORE_NUM
FA_METADATA_SIZE = _lib.SAS_FA_METADATA_SIZE
FD_METADATA_SIZE = _lib.SAS_FD_METADATA_SIZE

FA_CORE_ENABLE_INDEX = 0
FA_BN2_START_INDEX = 1
FA_M_START_INDEX = 2
FA_S2_START_INDEX = 3
FA_BN2_END_INDEX = 4
FA_M_END_INDEX = 5
FA_S2_END_INDEX = 6
FA_FIRST_FD_DATA_WORKSPACE_IDX_INDEX = 7
FD_CORE_ENABLE_INDEX = 0
FD_BN2_IDX_INDEX = 1
FD_M_IDX_INDEX = 2
FD_WORKSPACE_IDX_INDEX = 3
FD_WORKSPACE_NUM_INDEX = 4
FD_M_START_INDEX = 5
FD_M_NUM_INDEX = 6


class SparseMode:
    """Mask modes of the reference operator (metadata.py:71-77)."""

    DEFAULT_MASK = 0
    ALL_MASK = 1
    LEFT_UP_CAUSAL = 2
    RIGHT_DOWN_CAUSAL = 3
    BAND = 4
    SPARSE_BUTT = 5


def _as_i64(t):
    """Tensor / list / None -> (ctypes int64 array or None, length)."""
    if t is None:
        return None, 0
    if isinstance(t, torch.Tensor):
        if t.numel() == 0:
            return None, 0
        vals = t.detach().to("cpu", torch.int64).reshape(-1).tolist()
    elif isinstance(t, (list, tuple)):
        vals = [int(x) for x in t]
        if not vals:
            return None, 0
    else:
        return None, 0
    arr = (C.c_int64 * len(vals))(*vals)
    return arr, len(vals)


def sparse_attn_sharedkv_metadata(
    *,
    num_heads_q: int,
    num_heads_kv: int,
    head_dim: int,
    cu_seqlens_q: Optional[torch.Tensor] = None,
    cu_seqlens_ori_kv: Optional[torch.Tensor] = None,
    cu_seqlens_cmp_kv: Optional[torch.Tensor] = None,
    seqused_q: Optional[torch.Tensor] = None,
    seqused_kv: Optional[torch.Tensor] = None,
    batch_size: int = 0,
    max_seqlen_q: int = 0,
    max_seqlen_kv: int = 0,
    ori_topk: int = 0,
    cmp_topk: int = 0,
    cmp_ratio: int = -1,
    ori_mask_mode: int = 4,
    cmp_mask_mode: int = 3,
    ori_win_left: int = 127,
    ori_win_right: int = 0,
    layout_q: str = "BSND",
    layout_kv: str = "PA_ND",
    has_ori_kv: bool = True,
    has_cmp_kv: bool = True,
    aic_core_num: int = 24,
    aiv_core_num: int = 48,
    device: Optional[str] = None,
) -> torch.Tensor:
    """int32[1024] load-balancing table of the SparseAttnSharedkvMetadata op.

    Raises ``ValueError`` where the reference would fail (inconsistent
    lengths, zero KV heads) and ``RuntimeError`` where the reference's
    scheduler would not terminate.
    """
    keep = []
    p = _lib.SasMetaParams()
    p.num_heads_q, p.num_heads_kv, p.head_dim = num_heads_q, num_heads_kv, head_dim
    for name, t in (("cu_seqlens_q", cu_seqlens_q), ("cu_seqlens_ori_kv", cu_seqlens_ori_kv),
                    ("cu_seqlens_cmp_kv", cu_seqlens_cmp_kv), ("seqused_q", seqused_q),
                    ("seqused_kv", seqused_kv)):
        arr, n = _as_i64(t)
        keep.append(arr)
        setattr(p, name, C.cast(arr, C.POINTER(C.c_int64)) if arr is not None else None)
        setattr(p, "n_" + name, n)
    p.batch_size, p.max_seqlen_q, p.max_seqlen_kv = batch_size, max_seqlen_q, max_seqlen_kv
    p.ori_topk, p.cmp_topk, p.cmp_ratio = ori_topk, cmp_topk, cmp_ratio
    p.ori_mask_mode, p.cmp_mask_mode = ori_mask_mode, cmp_mask_mode
    p.ori_win_left, p.ori_win_right = ori_win_left, ori_win_right
    p.layout_q = _lib.LAYOUTS.get(layout_q, -1)
    p.layout_kv = _lib.LAYOUTS.get(layout_kv, -1)
    p.has_ori_kv, p.has_cmp_kv = int(bool(has_ori_kv)), int(bool(has_cmp_kv))
    p.aic_core_num, p.aiv_core_num = aic_core_num, aiv_core_num
    out = torch.zeros(SAS_META_SIZE, dtype=torch.int32)
    rc = _lib.lib().sas_metadata(C.byref(p),
                                 C.cast(out.data_ptr(), C.POINTER(C.c_int32)), SAS_META_SIZE)
    if rc == 1:
        raise ValueError("sparse_attn_sharedkv_metadata: invalid arguments "
                         "(lengths / head counts inconsistent with batch_size and layout)")
    if rc == 4:
        raise RuntimeError("sparse_attn_sharedkv_metadata: scheduler found no further key "
                           "block (the reference port would not terminate)")
    _lib.check("sas_metadata", rc)
    if device is not None:
        out = out.to(device)
    return out
