#!/usr/bin/env python3
"""Benchmark of the sparse shared-KV attention forward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl reference]
                    [--comparator flashmla]

One step = one call of the hot path (``sparse_attn_sharedkv``: plan reuse,
tcgen05 attention kernel, split-KV combine) over one batch of the workload.
The default workload is the benchmark's second configuration (SWA prefill,
TND, 4 sequences of 512..4096 tokens, 64 heads, d_qk 576 / d_v 512, window
128, paged block 64); ``--config 1..5`` selects any of the five.

Printed JSON line (rank 0):
* ``value``: whole-job algorithmic TFLOP/s with inputs resident in HBM
  (N ranks x FLOPs per step x K / max over ranks of the device time);
* ``e2e``: the same metric through the public API with host buffers: every
  step copies its inputs (q, indices, block tables) from pinned host memory
  and reads the LSE back; the KV caches stay resident, as in serving;
* ``roofline``: the attention kernel alone (CUDA events on its stream),
  algorithmic bytes (or FLOPs) per launch / duration vs the measured peak;
* ``cpu_baseline``: the CPU oracle (a port of the reference's golden
  attention) timed on this host on a bounded sample of the same workload.

``--comparator flashmla`` (configs 3 and 4) adds ``comparator``: vLLM's
FlashMLA sparse kernel, a library kernel, timed on the same inputs through its
Python wrapper, with the largest output difference — a yardstick, not part
of ``value``.

``--impl reference`` times that CPU implementation alone (the reference's
own implementation cannot run here: it needs an Ascend NPU / TileLang-Ascend;
its CPU golden cannot travel to the GPU box, so the oracle port stands in).

Multi-GPU (torchrun, one rank per GPU): the global workload is N copies of
the configuration's sequences, sharded one copy per rank (weak scaling; the
step itself needs no collective).  The sharded call's one exchange, the
all-gather of the output / LSE shards (sharding.gather_outputs, NCCL), is
timed separately under ``allgather``.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

METRIC = "sparse shared-KV attn μs/call, TFLOP/s & HBM GB/s vs roofline at 1/2/4/8 B200"
L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAKS = dict(hbm_gbs=6650.0, bf16_tflops=1590.0, bf16_tflops_sustained=1400.0)


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return dict(hbm_gbs=float(p["hbm_gbs"]), bf16_tflops=float(p["bf16_tflops"]),
                    bf16_tflops_sustained=float(p.get("bf16_tflops_sustained",
                                                      p["bf16_tflops"]))), "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


def load_traffic(workload: str):
    """DRAM bytes per launch of the attention kernel from the committed ncu
    summary (profiles/traffic.txt: ``<workload> <bytes>`` lines), or None."""
    path = os.path.join(REPO, "profiles", "traffic.txt")
    try:
        with open(path) as f:
            for line in f:
                parts = line.split()
                if len(parts) >= 2 and parts[0] == workload:
                    return float(parts[1])
    except OSError:
        pass
    return None


# ---------------------------------------------------------------------------
# Clock sampling (NVML) during the timed region.
# ---------------------------------------------------------------------------

class ClockSampler:
    """Samples SM clock and throttle reasons every ~2 ms on a thread."""

    REASONS = {
        "sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, device_index: int):
        self.ok = False
        self.samples = []
        self.reasons = 0
        try:
            import pynvml
            pynvml.nvmlInit()
            uuid = None
            try:
                import torch
                uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            except Exception:
                uuid = None
            h = None
            if uuid:
                for i in range(pynvml.nvmlDeviceGetCount()):
                    hh = pynvml.nvmlDeviceGetHandleByIndex(i)
                    u = pynvml.nvmlDeviceGetUUID(hh)
                    u = u.decode() if isinstance(u, bytes) else u
                    if u.replace("GPU-", "") == uuid.replace("GPU-", ""):
                        h = hh
                        break
            if h is None:
                h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.nv, self.h = pynvml, h
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None
        self._stop = threading.Event()

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                self.reasons |= int(self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h))
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [],
                    "samples": len(self.samples)}
        names = [n for n, bit in self.REASONS.items() if self.reasons & bit]
        return {"sm_mhz": float(statistics.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# CPU baseline: the oracle on a bounded sample.
# ---------------------------------------------------------------------------

def cpu_sample_run(case_cpu, acct_fn, budget_s: float, seed: int = 0):
    """Run the CPU oracle on growing token samples until ~budget_s seconds.

    Returns (flops_done, seconds, tokens_done, threads)."""
    import numpy as np
    import torch

    from oracle import sas_oracle as O
    from tests.golden_cases import case_to_numpy

    try:
        from threadpoolctl import threadpool_info
        threads = max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    except Exception:
        threads = os.cpu_count() or 1
    kw = case_to_numpy(case_cpu)
    T = (case_cpu.q.shape[0] if case_cpu.layout_q == "TND"
         else case_cpu.q.shape[0] * case_cpu.q.shape[1])
    rng = np.random.default_rng(seed)
    order = rng.permutation(T)
    per_tok = acct_fn(order)  # FLOPs of each token in `order`
    done_f, done_s, done_t, pos, chunk = 0.0, 0.0, 0, 0, 4
    while pos < T and done_s < budget_s:
        toks = order[pos:pos + chunk]
        t0 = time.perf_counter()
        O.forward(**kw, tokens=toks.tolist())
        dt = time.perf_counter() - t0
        done_s += dt
        done_f += float(per_tok[pos:pos + chunk].sum())
        done_t += len(toks)
        pos += chunk
        if dt < budget_s / 8:
            chunk *= 2
    return done_f, done_s, done_t, threads


def per_token_flops(case_cpu):
    """FLOPs of each flat token (for the CPU sample accounting)."""
    import numpy as np
    import torch

    from oracle import sas_oracle as O

    H, D = case_cpu.q.shape[-2], case_cpu.q.shape[-1]
    dv = case_cpu.head_dim_v or D
    B = case_cpu.batch
    if case_cpu.layout_q == "TND":
        cu = case_cpu.cu_seqlens_q.tolist()
        starts, lens = cu[:-1], [cu[i + 1] - cu[i] for i in range(B)]
        T = case_cpu.q.shape[0]
    else:
        S = case_cpu.q.shape[1]
        starts = [b * S for b in range(B)]
        lens = ([int(x) for x in (case_cpu.cu_seqlens_q[1:] - case_cpu.cu_seqlens_q[:-1])]
                if case_cpu.cu_seqlens_q is not None else [S] * B)
        T = B * S
    idx = (case_cpu.cmp_sparse_indices.reshape(T, -1).numpy()
           if case_cpu.cmp_sparse_indices is not None else None)
    f = np.zeros(T)
    for b in range(B):
        akv = int(case_cpu.seqused_kv[b])
        for s in range(lens[b]):
            t = starts[b] + s
            lo, hi = O.window_positions(akv, lens[b], s, case_cpu.ori_win_left)
            k = hi - lo
            if case_cpu.cmp_kv is not None:
                if idx is not None:
                    k += len(O.scfa_positions(idx[t], akv, lens[b], s, case_cpu.cmp_ratio))
                else:
                    k += max(O.cmp_threshold(akv, lens[b], s, case_cpu.cmp_ratio), 0)
            f[t] = 2.0 * H * k * (D + dv)
    return f


# ---------------------------------------------------------------------------
# Arms.
# ---------------------------------------------------------------------------

def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def run_reference(args):
    """The CPU implementation of the path (oracle port of golden.py) alone."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    import torch

    from sparse_attn_sharedkv_b200 import workloads as W

    case = W.baseline_case(args.config - 1, device="cpu")
    flops_tok = per_token_flops(case)
    budget = max(2.0, min(10.0, 150.0 / max(1, args.steps + args.warmup)))
    vals, samples = [], []
    threads = 1
    for i in range(args.warmup + args.steps):
        f, s, t, threads = cpu_sample_run(case, lambda o: flops_tok[o], budget, seed=i)
        if i >= args.warmup:
            vals.append(f / s / 1e12)
            samples.append(t)
    value = statistics.median(vals) if vals else 0.0
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": None, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 (bf16 inputs)", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": W.BASELINE_NAMES[args.config - 1], "device": "cpu"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": f"{int(statistics.median(samples))} query tokens per step "
                                   f"(~{budget:.0f} s of CPU work each), random tokens"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_gpu(args):
    import torch

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    from sparse_attn_sharedkv_b200 import api as A
    from sparse_attn_sharedkv_b200 import workloads as W

    cfg = args.config - 1
    case = W.baseline_case(cfg, device=dev)
    acct = W.accounting(case)
    kw = case.kwargs()
    # Lengths live on the host (the reference reads them with .cpu() anyway).
    kw["seqused_kv"] = case.seqused_kv.cpu()
    if case.cu_seqlens_q is not None:
        kw["cu_seqlens_q"] = case.cu_seqlens_q.cpu()
    q = case.q
    in_l2 = acct["bytes"] < 2 * L2_BYTES
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev) if in_l2 else None

    def step():
        return A.sparse_attn_sharedkv(q, return_softmax_lse=True, **kw)

    def barrier():
        if ws > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    barrier()
    info = A.last_plan_info
    launches_per_step = 1 + (1 if info.num_split_rows > 0 else 0)

    # ---- value: K steps, device time (per-step events when L2 is flushed) ----
    stream = torch.cuda.current_stream(dev)
    sampler = ClockSampler(local)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    barrier()
    with sampler:
        for i in range(args.steps):
            if flush is not None:
                flush.zero_()
            evs[i][0].record(stream)
            step()
            evs[i][1].record(stream)
        barrier()
    step_ms = [a.elapsed_time(b) for a, b in evs]
    total_ms = sum(step_ms)

    # ---- roofline: the attention kernel alone (same plan, same inputs) ----
    import ctypes as C

    from sparse_attn_sharedkv_b200 import _lib
    key_ws = None
    for k, v in A._PLAN_CACHE.items():
        key_ws = v
    ws_t, nbytes, pinfo = key_ws
    prob, fp, keep = _rebuild_call(A, case, kw)
    L = _lib.lib()
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    for i in range(args.steps):
        if flush is not None:
            flush.zero_()
        kev[i][0].record(stream)
        _lib.check("sas_fwd_execute",
                   L.sas_fwd_execute(C.byref(prob), C.byref(fp), C.byref(pinfo), ws_t.data_ptr(),
                                     nbytes, C.c_void_p(stream.cuda_stream), _lib.PHASE_ATTN))
        kev[i][1].record(stream)
    torch.cuda.synchronize()
    kern_ms = statistics.mean(a.elapsed_time(b) for a, b in kev)

    # ---- e2e: host buffers in, LSE out, through the public API ----
    host = {"q": q.cpu().pin_memory()}
    dev_bufs = {"q": torch.empty_like(q)}
    for name in ("cmp_sparse_indices", "ori_block_table", "cmp_block_table"):
        t = kw.get(name)
        if isinstance(t, torch.Tensor) and t.is_cuda:
            host[name] = t.cpu().pin_memory()
            dev_bufs[name] = torch.empty_like(t)
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    lse_host = None
    e2e_steps = max(1, min(args.steps, 20))
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        for name, t in host.items():
            dev_bufs[name].copy_(t, non_blocking=True)
        kw2 = dict(kw)
        for name in dev_bufs:
            if name != "q":
                kw2[name] = dev_bufs[name]
        out, lse = A.sparse_attn_sharedkv(dev_bufs["q"], return_softmax_lse=True, **kw2)
        if lse_host is None:
            lse_host = torch.empty(lse.shape, dtype=lse.dtype, pin_memory=True)
        lse_host.copy_(lse, non_blocking=True)
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    d2h = lse_host.numel() * lse_host.element_size()

    # ---- N > 1: the one exchange of a sharded call, an all-gather of the
    # output / LSE shards over NCCL (timed apart from `value`) ----
    gather_ms, gather_bytes, gather_note = 0.0, 0, None
    if ws > 1:
        from sparse_attn_sharedkv_b200 import sharding as SH
        out_t, lse_t = A.sparse_attn_sharedkv(q, return_softmax_lse=True, **kw)
        n_units = out_t.shape[0]
        gather_bytes = ws * (out_t.numel() * out_t.element_size() + lse_t.numel() * 4)
        if gather_bytes <= (16 << 30):
            plan = [(r * n_units, (r + 1) * n_units) for r in range(ws)]
            args_g = (plan, rank, tuple(out_t.shape[1:]), tuple(lse_t.shape[1:]), out_t.dtype, dev)
            SH.gather_outputs(out_t, lse_t, *args_g)  # warm-up
            barrier()
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            g0.record(stream)
            SH.gather_outputs(out_t, lse_t, *args_g)
            g1.record(stream)
            barrier()
            gather_ms = g0.elapsed_time(g1)
        else:
            gather_note = "skipped: gathered output above 16 GB per rank"
        del out_t, lse_t

    # ---- max over ranks ----
    vals = torch.tensor([total_ms, kern_ms, e2e_ms, gather_ms], dtype=torch.float64, device=dev)
    if ws > 1:
        import torch.distributed as dist
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    total_ms, kern_ms, e2e_ms, gather_ms = vals.tolist()

    if rank == 0:
        peaks, peak_src = load_peaks()
        flops, nbytes_alg = acct["flops"], acct["bytes"]
        ms_step = total_ms / args.steps
        value = ws * flops * args.steps / (total_ms * 1e-3) / 1e12
        ridge = peaks["bf16_tflops"] * 1e12 / (peaks["hbm_gbs"] * 1e9)
        bound = "hbm" if flops / nbytes_alg < ridge else "tensor"
        if bound == "hbm":
            ach = nbytes_alg / (kern_ms * 1e-3) / 1e9
            peak = peaks["hbm_gbs"]
            unit = "GB/s"
        else:
            ach = flops / (kern_ms * 1e-3) / 1e12
            peak = peaks["bf16_tflops"]
            unit = "TFLOP/s"
        # CPU baseline on this host (rank 0, N=1 only).
        cpu = None
        if ws == 1 and not args.no_cpu_baseline:
            c_cpu = case.to("cpu")
            ftok = per_token_flops(c_cpu)
            f, s, t, threads = cpu_sample_run(c_cpu, lambda o: ftok[o], args.cpu_seconds)
            cpu = {"value": f / s / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                   "sample": f"{t} of {acct['tokens']} query tokens (random), {s:.1f} s"}
        clocks = sampler.summary()
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded N(0,1)*0.5, random block tables)",
            "config": {
                "workload": W.BASELINE_NAMES[cfg], "tokens": acct["tokens"],
                "keys": acct["keys"], "flops_per_step": flops, "bytes_per_step": nbytes_alg,
                "us_per_call": ms_step * 1e3,
                "hbm_gbs_per_gpu": nbytes_alg / (ms_step * 1e-3) / 1e9,
                "l2": ("flushed between steps (256 MB write)" if in_l2
                       else "inputs larger than L2 (126 MB)"),
                "parallelism": (f"dp{ws}: one shard (a copy of the configuration's sequences) "
                                f"per rank, weak scaling"),
                "plan": {"workers": info.num_workers, "head_groups": info.head_groups,
                         "split_rows": info.num_split_rows, "tiles": int(info.total_tiles)},
            },
            "e2e": {"value": ws * flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms},
            "roofline": {"bound": bound, "achieved": ach, "peak": peak, "unit": unit,
                         "frac": ach / peak, "peak_source": f"{peak_src} (burst)",
                         "kernel": "sas_fwd_kernel", "kernel_ms": kern_ms,
                         "algorithmic_bytes": nbytes_alg, "algorithmic_flops": flops,
                         "traffic": load_traffic(W.BASELINE_NAMES[cfg]),
                         "tensor_tflops": flops / (kern_ms * 1e-3) / 1e12,
                         "hbm_gbs": nbytes_alg / (kern_ms * 1e-3) / 1e9},
            "cpu_baseline": cpu,
            "allgather": (None if ws == 1 else
                          {"ms": gather_ms, "bytes_gathered_per_rank": gather_bytes,
                           "what": "NCCL all-gather of every rank's output and LSE shard "
                                   "(the sharded call's one exchange); not part of value",
                           "note": gather_note}),
            "clocks": clocks,
            "gpu_launches": launches_per_step * args.steps,
        }
        if args.comparator == "flashmla":
            line["comparator"] = flashmla_comparator(A, case, kw)
        print(json.dumps(line), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


def flashmla_comparator(A, case, kw, reps: int = 20):
    """Optional yardstick (``--comparator flashmla``): vLLM's FlashMLA sparse
    prefill kernel (a library kernel, run through its Python wrapper) on the
    same inputs, for the pure top-k workloads it supports (configs 3 and 4:
    sinks -inf, no window).  The paged cache is viewed as one flat key array
    and each top-k position is translated to its pool row through the block
    table.  Returns its median kernel time and the largest output difference."""
    import torch
    try:
        from vllm.third_party.flashmla.flash_mla_interface import flash_mla_sparse_fwd
    except Exception as e:  # library absent or not built for this GPU
        return {"unavailable": f"vLLM FlashMLA not importable: {type(e).__name__}"}
    if case.cmp_sparse_indices is None or case.ori_win_left != -1 or case.q.shape[-2] % 64:
        return {"unavailable": "FlashMLA sparse covers pure top-k with 64k heads only"}
    q = case.q
    H = q.shape[-2]
    qf = q.reshape(-1, H, q.shape[-1]).contiguous()
    pool, table = case.cmp_kv, case.cmp_block_table
    bs = pool.shape[1]
    kvf = pool.reshape(-1, 1, pool.shape[-1])
    K = case.cmp_sparse_indices.shape[-1]
    idx = case.cmp_sparse_indices.reshape(-1, K).long()
    if case.layout_q == "TND":
        cu = case.cu_seqlens_q.long()
        bt = torch.repeat_interleave(torch.arange(len(cu) - 1, device=q.device), cu[1:] - cu[:-1])
    else:
        bt = torch.arange(q.shape[0], device=q.device).repeat_interleave(q.shape[1])
    pos = idx.clamp(min=0)
    rows = table.long()[bt[:, None], pos // bs] * bs + pos % bs
    rows = torch.where(idx >= 0, rows, torch.full_like(rows, -1))
    rows = rows.to(torch.int32).view(-1, 1, K).contiguous()
    run = lambda: flash_mla_sparse_fwd(qf, kvf, rows, case.softmax_scale, 512)
    out_fm = run()[0]
    ours = A.sparse_attn_sharedkv(q, **kw).reshape(-1, H, 512)
    diff = (ours.float() - out_fm.float()).abs().max().item()
    for _ in range(3):
        run()
    torch.cuda.synchronize()
    times = []
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(reps):
        s.record()
        run()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    times.sort()
    return {"impl": "vLLM FlashMLA flash_mla_sparse_fwd (library kernel, same inputs)",
            "kernel_ms": times[len(times) // 2], "max_abs_diff_out": diff}


def _rebuild_call(A, case, kw):
    """Argument structs of the last call (to launch the attention kernel
    alone through sas_fwd_execute on the cached plan)."""
    import ctypes as C

    import torch

    from sparse_attn_sharedkv_b200 import _lib
    captured = {}
    orig_exec = _lib.lib().sas_fwd_execute

    class Capture:
        def __call__(self, prob, fp, info, ws, n, stream, phases):
            captured["prob"] = _lib.SasProblem.from_buffer_copy(prob._obj)
            captured["fp"] = _lib.SasFwdParams.from_buffer_copy(fp._obj)
            return orig_exec(prob, fp, info, ws, n, stream, phases)

    L = _lib.lib()
    L.sas_fwd_execute = Capture()
    try:
        # The returned (out, lse) own the memory fp.out / fp.lse point to: keep them.
        keep = A.sparse_attn_sharedkv(case.q, return_softmax_lse=True, **kw)
    finally:
        L.sas_fwd_execute = orig_exec
    torch.cuda.synchronize()
    return captured["prob"], captured["fp"], keep


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=2, choices=[1, 2, 3, 4, 5],
                    help="benchmark configuration (1-based); default 2 (SWA prefill)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--comparator", default=None, choices=["flashmla"],
                    help="also time vLLM's FlashMLA sparse kernel on the same inputs "
                         "(configs 3 and 4; informational, not part of value)")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
