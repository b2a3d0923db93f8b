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

from .api import DEFAULT_CORE_NUM, _check_device_errors, _forward, _require, _restore_layout



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
    _require(ori_mask_mode == 4, "only ori_mask_mode=4 supported")
    _require(cmp_mask_mode == 3 or cmp_kv is None, "only cmp_mask_mode=3 supported")
    _require(ori_win_right == 0, "only ori_win_right=0 supported")
    _require(layout_kv == "PA_ND", "only layout_kv=PA_ND supported")
    _require(layout_q in ("TND", "BSND"), f"unsupported layout_q={layout_q!r}")
    err = torch.zeros(4, dtype=torch.int32, device=q.device) if _check_device_errors() else None
    out_flat, lse_flat = _forward(
        q, ori_kv=ori_kv, cmp_kv=cmp_kv, cmp_sparse_indices=cmp_sparse_indices,
        ori_block_table=ori_block_table, cmp_block_table=cmp_block_table,
        cu_seqlens_q=cu_seqlens_q, seqused_kv=seqused_kv, sinks=sinks,
        softmax_scale=softmax_scale, cmp_ratio=cmp_ratio, ori_win_left=ori_win_left,
        layout_q=layout_q, topk_cmp=topk_cmp, head_dim_v=head_dim_v, num_sms=num_sms, err=err)
    if err is not None:
        e = err.tolist()
        if e[0] != 0:
            raise RuntimeError(f"sas_fwd device check failed: code={e[0]} site={e[1]} "
                               f"detail={e[2]} block={e[3]}")
    return _restore_layout(q, out_flat, lse_flat, layout_q, return_softmax_lse)
