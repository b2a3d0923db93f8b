"""``sparse_attn_sharedkv``: drop-in for the reference ``api.sparse_attn_sharedkv``.

Same keyword signature, scenario resolution and return contract as the
reference (api.py:129-397):

* ``cmp_kv=None, cmp_sparse_indices=None``  -> SWA  (scenario 1)
* ``cmp_kv=<t>,  cmp_sparse_indices=None``  -> CFA  (scenario 2)
* ``cmp_kv=<t>,  cmp_sparse_indices=<t>``   -> SCFA (scenario 3)

``q`` is ``[T, N1, D]`` (TND, with ``cu_seqlens_q``) or ``[B, S, N1, D]``
(BSND); KV caches are paged ``[blocks, block_size, 1, D]`` with int32 block
tables.  Returns ``out`` in q's layout (last dim ``d_v``) and, with
``return_softmax_lse=True``, ``(out, lse)`` with ``lse`` fp32 ``[T, N1]`` /
``[B, S, N1]``.

Computation: one call into ``libsas.so`` (``sas_fwd``), which plans the work
for all SMs, runs the sm_100a tcgen05 kernel and the split-KV combine.  There
is no CPU or PyTorch fallback.

Extensions over the reference (additive keyword arguments; defaults keep the
reference behaviour where the reference supports the shape):

* ``head_dim_v``: output width; V is the first ``d_v`` columns of the shared
  K/V rows.  Defaults to ``D`` for ``D = 512`` and to 512 for ``D = 576``
  (the MLA latent/rope split).  Only ``d_v = 512`` is built.
* ``N1`` in 1..128 query heads (the reference requires 64); ``D`` in
  {512, 576} (the reference requires 512); any block size.
* ``ori_win_left = -1``: empty window (pure top-k attention when combined
  with SCFA, ``cmp_ratio = 1`` and ``cmp_kv`` the same cache).
* ``num_sms``: number of persistent workers (default: all SMs).
* ``device_plan``: keep ``cu_seqlens_q`` / ``seqused_kv`` on the device and
  build the work plan on the GPU (``sas_fwd_prepare_device``): the call reads
  no length on the host (the reference syncs on them, api.py:210, 260, 336),
  so it can be recorded in a CUDA graph and replayed with new lengths of the
  same shapes.

``metadata`` (the SparseAttnSharedkvMetadata table) and ``core_num`` are
accepted and validated for API parity; like the reference kernels
(kernel.py:367, 1851, 3416) the B200 kernel plans its own work split.
``seqused_q`` is accepted and unused, as in the reference (api.py:186).
"""

from __future__ import annotations

import ctypes as C
import os
from collections import OrderedDict
from typing import Optional, Tuple, Union

import torch

from . import _lib

DEFAULT_CORE_NUM = 24  # the reference's AIC count default (kernel.py:70)
SAS_META_SIZE = _lib.SAS_META_SIZE

def _check_device_errors() -> bool:
    """SAS_CHECK_DEVICE_ERRORS=1: give each call a device error word and raise
    if the kernel recorded an error (costs a sync).  Read per call; off while
    a CUDA graph is being captured (the read-back cannot be recorded)."""
    return (os.environ.get("SAS_CHECK_DEVICE_ERRORS", "0") == "1"
            and not torch.cuda.is_current_stream_capturing())

# Plans (host schedule uploaded into a device workspace) are reused across
# calls with the same lengths and shapes, as a serving step reuses one
# metadata table for every layer.  Keyed by everything the plan depends on,
# including the stream (the workspace also holds the split-KV partials).
_PLAN_CACHE: "OrderedDict" = OrderedDict()
_PLAN_CACHE_SIZE = 8
last_plan_info = None  # SasPlanInfo of the most recent call (diagnostics / bench)


def _require(cond: bool, msg: str) -> None:
    # The reference uses bare asserts (api.py:187-191); keep AssertionError but
    # make the check independent of ``python -O``.
    if not cond:
        raise AssertionError(msg)


def _dtype_code(t: torch.dtype) -> int:
    if t == torch.bfloat16:
        return _lib.DTYPE_BF16
    if t == torch.float16:
        return _lib.DTYPE_FP16
    raise ValueError(f"unsupported torch dtype {t}")


def _i32_array(vals):
    # Slice assignment fills the ctypes array in C (several times faster than
    # unpacking the list into its constructor; it runs on every call).
    arr = (C.c_int32 * len(vals))()
    arr[:] = vals
    return arr


def _dev_i32(t: torch.Tensor, device) -> torch.Tensor:
    return t.to(device=device, dtype=torch.int32).contiguous()


class CallArgs:
    """C-ABI argument blocks of one forward call (``SasProblem`` +
    ``SasFwdParams``), the flat outputs they point to, and every buffer the
    pointers reference (kept alive with the object)."""

    def __init__(self, **kw):
        self.__dict__.update(kw)


def build_call(q: torch.Tensor, *, ori_kv, cmp_kv=None, cmp_sparse_indices=None,
               ori_block_table, cmp_block_table=None, cu_seqlens_q=None, seqused_kv,
               sinks, softmax_scale, cmp_ratio=None, ori_win_left=127, layout_q="TND",
               topk_cmp=None, head_dim_v=None, num_sms=None, err=None,
               device_plan=False) -> CallArgs:
    """Validate the reference-style arguments and build the C-ABI structs.

    Mirrors api.py:196-366 (scenario resolution, TND/BSND flattening, K
    resolution, shape checks); allocates the flat ``out [T, N1, d_v]`` and
    ``lse [T, N1]`` that ``sas_fwd`` writes.  With ``device_plan`` the
    per-batch lengths stay on the device and ``SasProblem`` carries device
    pointers (for ``sas_fwd_prepare_device``): the call reads no length on the
    host.
    """
    dtype = q.dtype
    dcode = _dtype_code(dtype)
    dev = q.device
    if dev.type != "cuda":
        raise RuntimeError("sparse_attn_sharedkv runs on a CUDA (sm_100a) device only; "
                           f"got q on {dev}")

    if cmp_kv is None:
        scenario = _lib.SCENARIO_SWA
    elif cmp_sparse_indices is None:
        scenario = _lib.SCENARIO_CFA
    else:
        scenario = _lib.SCENARIO_SCFA

    # ---- flat [T, N1, D] view + per-batch offsets (api.py:204-240) ----
    if layout_q == "TND":
        _require(cu_seqlens_q is not None, "cu_seqlens_q is required for TND")
        T1, N1, D = q.shape
        total = T1
        q_flat = q
        if device_plan:
            B = cu_seqlens_q.numel() - 1
            cu_d = cu_seqlens_q.to(device=dev, dtype=torch.int32)
            q_start = cu_d[:-1].contiguous()
            q_len = (cu_d[1:] - cu_d[:-1]).contiguous()
            S_max = 0
        else:
            cu = cu_seqlens_q.to(torch.int64).cpu().tolist()
            B = len(cu) - 1
            q_start = cu[:-1]
            q_len = [cu[i + 1] - cu[i] for i in range(B)]
            S_max = max(q_len) if q_len else 0
        idx_flat = None
        if scenario == _lib.SCENARIO_SCFA:
            idx_flat = cmp_sparse_indices
            N2i = idx_flat.shape[1]
            idx_flat = idx_flat.reshape(total, N2i, idx_flat.shape[-1])
    elif layout_q == "BSND":
        B, S_max, N1, D = q.shape
        total = B * S_max
        q_flat = q.reshape(total, N1, D)
        if device_plan:
            q_start = torch.arange(0, max(total, 1), max(S_max, 1), dtype=torch.int32,
                                   device=dev)[:B].contiguous()
            if cu_seqlens_q is not None:
                cu_d = cu_seqlens_q.to(device=dev, dtype=torch.int32)
                q_len = (cu_d[1:] - cu_d[:-1]).contiguous()
            else:
                q_len = torch.full((B,), S_max, dtype=torch.int32, device=dev)
        else:
            q_start = [b * S_max for b in range(B)]
            q_len = [S_max] * B
            if cu_seqlens_q is not None:
                cu = cu_seqlens_q.to(torch.int64).cpu().tolist()
                q_len = [cu[i + 1] - cu[i] for i in range(B)]
        idx_flat = None
        if scenario == _lib.SCENARIO_SCFA:
            ci = cmp_sparse_indices
            idx_flat = ci.reshape(total, ci.shape[2], ci.shape[3])
    else:
        raise AssertionError(f"unsupported layout_q={layout_q!r}")

    _require(seqused_kv.numel() >= B, "seqused_kv must have one entry per batch")
    if device_plan:
        kv_len = seqused_kv.reshape(-1)[:B].to(device=dev, dtype=torch.int32).contiguous()
    else:
        kv_len = seqused_kv.to(torch.int64).cpu().tolist()[:B]

    if scenario == _lib.SCENARIO_SCFA:
        N2 = idx_flat.shape[1]
        K = topk_cmp if topk_cmp is not None else idx_flat.shape[2]
        _require(K == idx_flat.shape[2], "topk_cmp does not match cmp_sparse_indices last dim")
    elif scenario == _lib.SCENARIO_CFA:
        N2 = cmp_kv.shape[2]
        K = 0
    else:
        N2 = ori_kv.shape[2]
        K = 0
    if N2 != 1 or ori_kv.shape[2] != 1:
        raise ValueError(f"only one KV head is supported (got N2={N2})")
    if D not in (512, 576):
        raise ValueError(f"head dim D must be 512 or 576 (got {D})")
    if head_dim_v is None:
        head_dim_v = 512
    if head_dim_v != 512:
        raise ValueError(f"only head_dim_v=512 is built (got {head_dim_v})")
    if not 1 <= N1 <= 128:
        raise ValueError(f"query heads N1 must be in [1, 128] (got {N1})")
    if ori_kv.shape[-1] != D or (cmp_kv is not None and cmp_kv.shape[-1] != D):
        raise ValueError("q, ori_kv and cmp_kv must share the head dim")
    if ori_kv.dtype != dtype or (cmp_kv is not None and cmp_kv.dtype != dtype):
        raise ValueError("q, ori_kv and cmp_kv must share the dtype")
    ratio = int(cmp_ratio) if cmp_ratio is not None else 4  # api.py:287
    if scenario >= _lib.SCENARIO_CFA and ratio < 1:
        raise ValueError(f"cmp_ratio must be >= 1 (got {ratio})")

    q_flat = q_flat.contiguous()
    ori = ori_kv.contiguous()
    ori_bt = _dev_i32(ori_block_table, dev)
    cmp = cmp_kv.contiguous() if cmp_kv is not None else None
    cmp_bt = _dev_i32(cmp_block_table, dev) if cmp_kv is not None else None
    idx = (_dev_i32(idx_flat.reshape(total, -1), dev) if idx_flat is not None else None)
    snk = sinks.to(device=dev, dtype=torch.float32).contiguous()
    _require(snk.numel() >= N1, "sinks must hold one value per query head")

    out = torch.empty((total, N1, head_dim_v), dtype=dtype, device=dev)
    lse = torch.empty((total, N1), dtype=torch.float32, device=dev)

    prob = _lib.SasProblem()
    prob.batch = B
    prob.layout_q = _lib.LAYOUTS[layout_q]
    prob.max_q_len = S_max
    prob.total_tokens = total
    if device_plan:
        a_start, a_len, a_kv = q_start, q_len, kv_len  # device int32 tensors
        prob.q_start = C.cast(C.c_void_p(q_start.data_ptr()), C.POINTER(C.c_int32))
        prob.q_len = C.cast(C.c_void_p(q_len.data_ptr()), C.POINTER(C.c_int32))
        prob.kv_len = C.cast(C.c_void_p(kv_len.data_ptr()), C.POINTER(C.c_int32))
    else:
        a_start, a_len, a_kv = _i32_array(q_start), _i32_array(q_len), _i32_array(kv_len)
        prob.q_start = C.cast(a_start, C.POINTER(C.c_int32))
        prob.q_len = C.cast(a_len, C.POINTER(C.c_int32))
        prob.kv_len = C.cast(a_kv, C.POINTER(C.c_int32))
    prob.num_heads = N1
    prob.scenario = scenario
    prob.ori_win_left = int(ori_win_left)
    prob.cmp_ratio = ratio
    prob.topk = int(K)

    fp = _lib.SasFwdParams()
    fp.q = q_flat.data_ptr()
    fp.ori_kv = ori.data_ptr()
    fp.ori_block_table = ori_bt.data_ptr()
    fp.cmp_kv = cmp.data_ptr() if cmp is not None else None
    fp.cmp_block_table = cmp_bt.data_ptr() if cmp_bt is not None else None
    fp.cmp_indices = idx.data_ptr() if idx is not None else None
    fp.sinks = snk.data_ptr()
    fp.out = out.data_ptr()
    fp.lse = lse.data_ptr()
    fp.err = err.data_ptr() if err is not None else None
    fp.head_dim = D
    fp.head_dim_v = head_dim_v
    fp.dtype = dcode
    fp.softmax_scale = float(softmax_scale)
    fp.ori_block_size, fp.ori_num_blocks = ori.shape[1], ori.shape[0]
    fp.ori_table_len = ori_bt.shape[1]
    if cmp is not None:
        fp.cmp_block_size, fp.cmp_num_blocks = cmp.shape[1], cmp.shape[0]
        fp.cmp_table_len = cmp_bt.shape[1]
    fp.num_sms = int(num_sms or 0)
    lengths_key = (("device", B) if device_plan
                   else (tuple(q_start), tuple(q_len), tuple(kv_len)))
    return CallArgs(prob=prob, fp=fp, out=out, lse=lse, total=total, device=dev,
                    device_plan=bool(device_plan),
                    plan_key=(layout_q, lengths_key, N1, scenario, int(ori_win_left), ratio,
                              int(K), fp.num_sms, total, S_max),
                    keep=(q_flat, ori, ori_bt, cmp, cmp_bt, idx, snk, err, a_start, a_len,
                          a_kv))


def _forward(q: torch.Tensor, **kw):
    """Shared implementation of both entry points; returns flat (out, lse)."""
    global last_plan_info
    call = build_call(q, **kw)
    prob, fp, out, lse, dev = call.prob, call.fp, call.out, call.lse, call.device
    L = _lib.lib()
    if call.total == 0:
        return out, lse
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        key = (dev.index, stream) + call.plan_key
        if call.device_plan:
            # The plan depends on device-resident lengths: rebuilt on the GPU
            # every call (one small kernel); the workspace is cached per shape.
            hit = _PLAN_CACHE.get(key)
            if hit is None:
                ws_bytes = C.c_size_t(0)
                _lib.check("sas_fwd_workspace_size_device",
                           L.sas_fwd_workspace_size_device(C.byref(prob), fp.num_sms,
                                                           C.byref(ws_bytes)))
                ws = torch.empty(max(ws_bytes.value, 256), dtype=torch.uint8, device=dev)
                hit = (ws, ws_bytes.value, None)
                _PLAN_CACHE[key] = hit
                while len(_PLAN_CACHE) > _PLAN_CACHE_SIZE:
                    _PLAN_CACHE.popitem(last=False)
            ws, nbytes, _ = hit
            info = _lib.SasPlanInfo()
            _lib.check("sas_fwd_prepare_device",
                       L.sas_fwd_prepare_device(C.byref(prob), C.byref(fp), ws.data_ptr(), nbytes,
                                                C.c_void_p(stream), C.byref(info)))
            last_plan_info = info
            _lib.check("sas_fwd_execute",
                       L.sas_fwd_execute(C.byref(prob), C.byref(fp), C.byref(info),
                                         ws.data_ptr(), nbytes, C.c_void_p(stream),
                                         _lib.PHASE_ALL))
            return out, lse
        hit = _PLAN_CACHE.get(key)
        if hit is None:
            ws_bytes = C.c_size_t(0)
            _lib.check("sas_fwd_workspace_size",
                       L.sas_fwd_workspace_size(C.byref(prob), fp.num_sms, C.byref(ws_bytes)))
            ws = torch.empty(max(ws_bytes.value, 256), dtype=torch.uint8, device=dev)
            info = _lib.SasPlanInfo()
            _lib.check("sas_fwd_prepare",
                       L.sas_fwd_prepare(C.byref(prob), C.byref(fp), ws.data_ptr(),
                                         ws_bytes.value, C.c_void_p(stream), C.byref(info)))
            hit = (ws, ws_bytes.value, info)
            _PLAN_CACHE[key] = hit
            while len(_PLAN_CACHE) > _PLAN_CACHE_SIZE:
                _PLAN_CACHE.popitem(last=False)
        else:
            _PLAN_CACHE.move_to_end(key)
        ws, nbytes, info = hit
        last_plan_info = info
        _lib.check("sas_fwd_execute",
                   L.sas_fwd_execute(C.byref(prob), C.byref(fp), C.byref(info), ws.data_ptr(),
                                     nbytes, C.c_void_p(stream), _lib.PHASE_ALL))
    return out, lse


def sparse_attn_sharedkv(
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
    metadata: Optional[torch.Tensor] = None,
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
    device_plan: bool = False,
) -> Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]]:
    """Sparse shared-KV attention forward; see the module docstring."""
    del seqused_q, core_num  # API parity (api.py:186); the B200 plan uses all SMs
    _check_modes(cmp_kv, ori_mask_mode, cmp_mask_mode, ori_win_right, layout_q, layout_kv)
    if metadata is not None:
        _require(metadata.numel() == SAS_META_SIZE,
                 f"metadata must have {SAS_META_SIZE} int32 entries (got {metadata.numel()})")
    out_flat, lse_flat = _checked_forward(
        q, ori_kv=ori_kv, cmp_kv=cmp_kv, cmp_sparse_indices=cmp_sparse_indices,
        ori_block_table=ori_block_table, cmp_block_table=cmp_block_table,
        cu_seqlens_q=cu_seqlens_q, seqused_kv=seqused_kv, sinks=sinks,
        softmax_scale=softmax_scale, cmp_ratio=cmp_ratio, ori_win_left=ori_win_left,
        layout_q=layout_q, topk_cmp=topk_cmp, head_dim_v=head_dim_v, num_sms=num_sms,
        device_plan=device_plan)
    return _restore_layout(q, out_flat, lse_flat, layout_q, return_softmax_lse)


def _check_modes(cmp_kv, ori_mask_mode, cmp_mask_mode, ori_win_right, layout_q, layout_kv):
    """The mode / layout checks of both entry points (api.py:187-191)."""
    _require(ori_mask_mode == 4, "only ori_mask_mode=4 supported")
    _require(cmp_mask_mode == 3 or cmp_kv is None, "only cmp_mask_mode=3 supported")
    _require(ori_win_right == 0, "only ori_win_right=0 supported")
    _require(layout_kv == "PA_ND", "only layout_kv=PA_ND supported")
    _require(layout_q in ("TND", "BSND"), f"unsupported layout_q={layout_q!r}")


def _checked_forward(q: torch.Tensor, **kw):
    """_forward with the device error word when SAS_CHECK_DEVICE_ERRORS=1: a
    device-side check that fired (an out-of-pool page id, a timed-out wait)
    raises RuntimeError after the call."""
    err = None
    if _check_device_errors():
        err = torch.zeros(4, dtype=torch.int32, device=q.device)
    out_flat, lse_flat = _forward(q, err=err, **kw)
    if err is not None:
        e = err.tolist()
        if e[0] != 0:
            raise RuntimeError(f"sas_fwd device check failed: code={e[0]} site={e[1]} "
                               f"detail={e[2]} block={e[3]}")
    return out_flat, lse_flat


def _restore_layout(q, out_flat, lse_flat, layout_q, return_lse):
    """api.py:386-397."""
    if layout_q == "TND":
        out, lse = out_flat, lse_flat
    else:
        B, S = q.shape[0], q.shape[1]
        out = out_flat.reshape(B, S, q.shape[2], out_flat.shape[-1])
        lse = lse_flat.reshape(B, S, q.shape[2])
    if return_lse:
        return out, lse
    return out
