"""Paged-cache writer: append new key rows into a paged KV pool.

The attention path reads its keys from paged pools ``[blocks, block_size, 1,
D]`` through per-batch block tables; this is the step that fills them.  The
layout is the reference's (golden.py:315-360, the inverse of
``unpack_paged_kv``, golden.py:247-268): logical position ``p`` of batch ``b``
lives at ``pool[block_table[b, p // block_size], p % block_size]``.  The
reference has no device writer (its tests pack caches on the host), so this
op has no reference signature; it follows the operator's own conventions
(TND ``cu_seqlens`` for the new rows, int32 tables with -1 = unmapped).

Runs ``sas_kv_append`` from ``libsas.so`` on the caller's stream; there is no
CPU fallback.
"""

from __future__ import annotations

import ctypes as C
from typing import Optional

import torch

from . import _lib


def append_paged_kv(kv_pool: torch.Tensor, block_table: torch.Tensor, new_rows: torch.Tensor,
                    cu_seqlens_new: torch.Tensor, start_pos: torch.Tensor,
                    check_errors: bool = False) -> Optional[list]:
    """Write ``new_rows`` into ``kv_pool`` in place.

    kv_pool:        [blocks, block_size, 1, D] (or [blocks, block_size, D]), bf16/fp16, CUDA.
    block_table:    [B, table_len] int32 (-1 = unmapped page), CUDA.
    new_rows:       [T_new, 1, D] or [T_new, D], same dtype as the pool, CUDA.
    cu_seqlens_new: [B + 1] int32: batch b appends rows cu[b] .. cu[b+1].
    start_pos:      [B] int32: logical position of batch b's first new row
                    (normally its length before the append).

    Rows whose position falls past the table or on an unmapped page are
    skipped.  With ``check_errors`` the call synchronises and returns the
    device error record ``[code, site, row, batch]`` if any row was skipped
    (else None).
    """
    assert kv_pool.is_cuda and new_rows.is_cuda, "kv_pool and new_rows must be CUDA tensors"
    assert kv_pool.dtype == new_rows.dtype, "new_rows must have the pool's dtype"
    assert kv_pool.dim() in (3, 4) and (kv_pool.dim() == 3 or kv_pool.shape[2] == 1), \
        "kv_pool must be [blocks, block_size, 1, D]"
    D = kv_pool.shape[-1]
    assert new_rows.shape[-1] == D, "new_rows last dim must match the pool"
    assert kv_pool.is_contiguous() and new_rows.is_contiguous(), "tensors must be contiguous"
    dev = kv_pool.device
    bt = block_table.to(device=dev, dtype=torch.int32).contiguous()
    cu = cu_seqlens_new.to(device=dev, dtype=torch.int32).contiguous()
    sp = start_pos.to(device=dev, dtype=torch.int32).contiguous()
    B = bt.shape[0]
    assert cu.numel() == B + 1 and sp.numel() == B, "cu_seqlens_new [B+1], start_pos [B]"
    total = new_rows.numel() // D
    err = torch.zeros(4, dtype=torch.int32, device=dev) if check_errors else None
    stream = torch.cuda.current_stream(dev).cuda_stream
    _lib.check("sas_kv_append", _lib.lib().sas_kv_append(
        C.c_void_p(kv_pool.data_ptr()), kv_pool.shape[0], kv_pool.shape[1],
        D * kv_pool.element_size(), C.c_void_p(bt.data_ptr()), bt.shape[1],
        C.c_void_p(new_rows.data_ptr()), C.c_void_p(cu.data_ptr()), C.c_void_p(sp.data_ptr()),
        B, total, C.c_void_p(err.data_ptr() if err is not None else 0), C.c_void_p(stream)))
    if err is not None:
        e = err.tolist()
        return e if e[0] != 0 else None
    return None
