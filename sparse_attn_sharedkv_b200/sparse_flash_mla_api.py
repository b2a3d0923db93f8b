"""``sparse_flash_mla``: drop-in for the reference's upstream entry point
``sparse_flash_mla/sparse_flash_mla_api.py::sparse_flash_mla``
(sparse_flash_mla_api.py:94-253).

Same operator as :func:`sparse_attn_sharedkv_b200.api.sparse_attn_sharedkv`
without the ``metadata`` argument; the upstream names the compressed
scenarios HCA (dense, scenario 2) and CSA (top-k, scenario 3)
(sparse_flash_mla_kernel.py:41-42).  Same extensions (``head_dim_v``,
1..128 heads, d_qk 576, empty window, ``num_sms``).
"""

from __future__ import annotations

from typing import Optional, Tuple, Union

import torch

from .api import DEFAULT_CORE_NUM, _check_modes, _checked_forward, _restore_layout


def sparse_flash_mla(
    q: torch.Tensor,
    *,
    ori_kv: torch.Tensor,
    cmp_kv: Optional[torch.Tensor] = None,
    cmp_sparse_indices: Optional[torch.Tensor] = None,
    ori_block_table: torch.Tensor,
    cmp_block_table: Optional[torch.Tensor] = None,
    cu_seqlens_q: Optional[torch.Tensor] = None,
    seqused_q: Optional[torch.Tensor] = None,
    seqused_kv: torch.Tensor,
    sinks: torch.Tensor,
    softmax_scale: float,
    cmp_ratio: Optional[int] = None,
    ori_mask_mode: int = 4,
    cmp_mask_mode: int = 3,
    ori_win_left: int = 127,
    ori_win_right: int = 0,
    layout_q: str = "TND",
    layout_kv: str = "PA_ND",
    return_softmax_lse: bool = False,
    core_num: int = DEFAULT_CORE_NUM,
    topk_cmp: Optional[int] = None,
    head_dim_v: Optional[int] = None,
    num_sms: Optional[int] = None,
) -> Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]]:
    """Sparse flash MLA forward (SWA / HCA / CSA)."""
    del seqused_q, core_num
    _check_modes(cmp_kv, ori_mask_mode, cmp_mask_mode, ori_win_right, layout_q, layout_kv)
    out_flat, lse_flat = _checked_forward(
        q, ori_kv=ori_kv, cmp_kv=cmp_kv, cmp_sparse_indices=cmp_sparse_indices,
        ori_block_table=ori_block_table, cmp_block_table=cmp_block_table,
        cu_seqlens_q=cu_seqlens_q, seqused_kv=seqused_kv, sinks=sinks,
        softmax_scale=softmax_scale, cmp_ratio=cmp_ratio, ori_win_left=ori_win_left,
        layout_q=layout_q, topk_cmp=topk_cmp, head_dim_v=head_dim_v, num_sms=num_sms)
    return _restore_layout(q, out_flat, lse_flat, layout_q, return_softmax_lse)
