#!/usr/bin/env python3
"""Benchmark of the sparse shared-KV attention forward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl reference]
                    [--comparator flashmla]

One step = one call of the hot path (``sparse_attn_sharedkv``: plan reuse,
tcgen05 attention kernel, split-KV combine) over one batch of the workload.
The default workload is the benchmark's fourth configuration, the largest
that runs on one GPU (sparse prefill, TND, 8 sequences of 4096 tokens,
128 heads, top-k 2048 causal indices, d_qk 576 / d_v 512, paged block 64);
``--config 1..5`` selects any of the five.

Printed JSON line (rank 0):
* ``value``: whole-job algorithmic TFLOP/s with inputs resident in HBM
  (FLOPs of the call x K / max over ranks of the device time);
* ``e2e``: the same metric through the public API with host buffers: every
  step copies its inputs (q, indices, block tables) from pinned host memory
  and copies the output and the LSE back into pinned host memory; the KV
  caches stay resident, as in serving; steps are pipelined over three
  streams (copy-in, call, copy-out);
* ``roofline``: the attention kernel alone (CUDA events on its stream),
  algorithmic bytes (or FLOPs) per launch / duration vs the measured peak;
* ``per_config`` (N = 1): kernel and call times with their roofline
  fractions for the other four configurations, same process and GPU;
* ``cpu_baseline``: the CPU oracle (a port of the reference's golden
  attention) timed on this host on a bounded sample of the same workload,
  with the threads it used and the host's core count.

``--comparator flashmla`` (configs 3 and 4) adds ``comparator``: vLLM's
FlashMLA sparse kernel, a library kernel, timed on the same inputs through its
Python wrapper, with the largest output difference — a yardstick, not part
of ``value``.

``--impl reference`` times that CPU implementation alone (the reference's
own implementation cannot run here: it needs an Ascend NPU / TileLang-Ascend;
its CPU golden cannot travel to the GPU box, so the oracle port stands in).

Multi-GPU (torchrun, one rank per GPU): the configuration's call is split
over the N ranks (sharding.plan_shards: decode by batch, TND prefill by
token ranges, each rank holding only the KV pages its rows reach), so the
total work is fixed (strong scaling); ``value`` and ``e2e`` take the max over
ranks.  The sharded call's one exchange, a gather of the output / LSE shards
to rank 0 over NCCL, is timed separately under ``gather``; in ``e2e`` every
rank copies its own output shard to host memory.
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


def attention_kernel_name(info):
    """The attention kernel libsas launches for a plan: the CTA-pair kernel for
    two head groups (65..128 heads) unless SAS_FWD_KERNEL=single or the
    cp.async gather mode is chosen, else the one-CTA-per-head-group kernel."""
    pair = (info is not None and info.head_groups == 2
            and os.environ.get("SAS_FWD_KERNEL") != "single"
            and os.environ.get("SAS_GATHER") != "lsu")
    return "sas_pair_kernel" if pair else "sas_fwd_kernel"


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


def cpu_threads():
    """(threads the CPU oracle uses, host cores)."""
    host = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_info
        used = max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    except Exception:
        used = host
    return used, host


def run_reference(args):
    """The CPU implementation of the path (oracle port of golden.py) alone."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0

    from tests import workloads as W

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
    _, host = cpu_threads()
    # time of one whole step (every token of the workload) at the sampled rate
    step_flops = float(sum(flops_tok))
    ms_step = step_flops / (value * 1e12) * 1e3 if value > 0 else None
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong" if args.gpus > 1 else "weak",
        "vs_baseline": None, "dtype": "f32 (bf16 inputs)", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": W.BASELINE_NAMES[args.config - 1], "device": "cpu",
                   "ms_per_step": "one whole step of the workload at the sampled rate"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads,
                         "host_cores": host, "kind": "port",
                         "sample": f"{int(statistics.median(samples))} query tokens per step "
                                   f"(~{budget:.0f} s of CPU work each), random tokens"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# Workloads on the GPU.
# ---------------------------------------------------------------------------

def host_lengths(kw):
    """Lengths on the host (the reference reads them with .cpu() anyway)."""
    kw = dict(kw)
    kw["seqused_kv"] = kw["seqused_kv"].cpu()
    if kw.get("cu_seqlens_q") is not None:
        kw["cu_seqlens_q"] = kw["cu_seqlens_q"].cpu()
    return kw


def shard_case(W, full, q, kw):
    """A Case for a shard's (q, kwargs), for the work accounting."""
    return W.Case(full.name, full.layout_q, q, kw["ori_kv"], kw["ori_block_table"],
                  torch_tensor(kw["seqused_kv"]), full.sinks, full.softmax_scale,
                  cu_seqlens_q=(torch_tensor(kw["cu_seqlens_q"])
                                if kw.get("cu_seqlens_q") is not None else None),
                  cmp_kv=kw.get("cmp_kv"), cmp_block_table=kw.get("cmp_block_table"),
                  cmp_sparse_indices=kw.get("cmp_sparse_indices"),
                  cmp_ratio=full.cmp_ratio, ori_win_left=full.ori_win_left,
                  head_dim_v=full.head_dim_v)


def torch_tensor(x):
    import torch
    return torch.as_tensor(x)


def kernel_alone_ms(A, q, kw, steps, flush, stream):
    """Mean device time of the attention kernel alone (sas_fwd_execute with
    the attention phase only, on the call's cached plan), CUDA events on the
    launching stream."""
    import ctypes as C

    import torch

    from sparse_attn_sharedkv_b200 import _lib
    prob, fp, keep = _rebuild_call(A, q, kw)
    hit = None
    for v in A._PLAN_CACHE.values():
        hit = v
    ws_t, nbytes, pinfo = hit
    L = _lib.lib()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]
    for i in range(steps):
        if flush is not None:
            flush.zero_()
        evs[i][0].record(stream)
        _lib.check("sas_fwd_execute",
                   L.sas_fwd_execute(C.byref(prob), C.byref(fp), C.byref(pinfo), ws_t.data_ptr(),
                                     nbytes, C.c_void_p(stream.cuda_stream), _lib.PHASE_ATTN))
        evs[i][1].record(stream)
    torch.cuda.synchronize()
    del keep
    return statistics.mean(a.elapsed_time(b) for a, b in evs)


def step_times_ms(A, q, kw, steps, flush, stream, sampler=None):
    """Device time of each of `steps` full calls (plan reuse, attention,
    combine), CUDA events on the launching stream."""
    import contextlib

    import torch
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]
    with (sampler if sampler is not None else contextlib.nullcontext()):
        for i in range(steps):
            if flush is not None:
                flush.zero_()
            evs[i][0].record(stream)
            A.sparse_attn_sharedkv(q, return_softmax_lse=True, **kw)
            evs[i][1].record(stream)
        torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in evs]


def roofline(acct, kern_ms, peaks):
    flops, nbytes = acct["flops"], acct["bytes"]
    ridge = peaks["bf16_tflops"] * 1e12 / (peaks["hbm_gbs"] * 1e9)
    if flops / nbytes < ridge:
        ach = nbytes / (kern_ms * 1e-3) / 1e9
        return "hbm", ach, peaks["hbm_gbs"], "GB/s"
    ach = flops / (kern_ms * 1e-3) / 1e12
    return "tensor", ach, peaks["bf16_tflops"], "TFLOP/s"


def e2e_pipelined(A, q, kw, n_steps, dev):
    """End to end through the public API with host buffers: every step copies
    its inputs (q, indices, block tables) from pinned host memory, runs the
    call and copies the output and the LSE back into pinned host memory.
    Steps are pipelined over three streams (copy-in of step i + 1 and
    copy-out of step i - 1 overlap the call of step i; PCIe is full duplex).
    Returns (ms per step, h2d bytes per step, d2h bytes per step)."""
    import torch

    names = ["q"] + [n for n in ("cmp_sparse_indices", "ori_block_table", "cmp_block_table")
                     if isinstance(kw.get(n), torch.Tensor) and kw[n].is_cuda]
    src = {"q": q}
    src.update({n: kw[n] for n in names if n != "q"})
    host = {n: t.cpu().pin_memory() for n, t in src.items()}
    bufs = [{n: torch.empty_like(t) for n, t in src.items()} for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    s_in, s_run, s_out = (torch.cuda.Stream(dev) for _ in range(3))
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_run = [torch.cuda.Event() for _ in range(2)]
    out_host = lse_host = None

    def one(i):
        nonlocal out_host, lse_host
        s = i % 2
        with torch.cuda.stream(s_in):
            if i >= 2:
                s_in.wait_event(ev_run[s])  # the call two steps back read bufs[s]
            for n, t in host.items():
                bufs[s][n].copy_(t, non_blocking=True)
            ev_in[s].record(s_in)
        with torch.cuda.stream(s_run):
            s_run.wait_event(ev_in[s])
            kw2 = dict(kw)
            for n in names:
                if n != "q":
                    kw2[n] = bufs[s][n]
            out, lse = A.sparse_attn_sharedkv(bufs[s]["q"], return_softmax_lse=True, **kw2)
            ev_run[s].record(s_run)
        if out_host is None:
            out_host = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
            lse_host = torch.empty(lse.shape, dtype=lse.dtype, pin_memory=True)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_run[s])
            out_host.copy_(out, non_blocking=True)
            lse_host.copy_(lse, non_blocking=True)
            out.record_stream(s_out)
            lse.record_stream(s_out)

    one(0)  # warm-up: plans for the run stream, pinned output buffers
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    for i in range(n_steps):
        one(i)
    e1.record(s_out)
    torch.cuda.synchronize()
    d2h = out_host.numel() * out_host.element_size() + lse_host.numel() * 4
    ms = e0.elapsed_time(e1) / n_steps
    return ms, h2d, d2h


def other_configs(A, W, cfgs, dev, stream, peaks, steps):
    """Per-configuration kernel and step times of the workloads other than the
    headline one, on this GPU, in this process (same clock sampler context)."""
    import gc

    import torch
    res = {}
    for cfg in cfgs:
        case = W.baseline_case(cfg, device=dev)
        acct = W.accounting(case)
        kw = host_lengths(case.kwargs())
        in_l2 = acct["bytes"] < 2 * L2_BYTES
        flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev) if in_l2 else None
        for _ in range(3):
            A.sparse_attn_sharedkv(case.q, return_softmax_lse=True, **kw)
        torch.cuda.synchronize()
        n = max(5, steps)
        st = step_times_ms(A, case.q, kw, n, flush, stream)
        kms = kernel_alone_ms(A, case.q, kw, n, flush, stream)
        bound, ach, peak, unit = roofline(acct, kms, peaks)
        info = A.last_plan_info
        res[W.BASELINE_NAMES[cfg]] = {
            "us_per_call": statistics.mean(st) * 1e3, "kernel_us": kms * 1e3,
            "tflops": acct["flops"] / (kms * 1e-3) / 1e12,
            "hbm_gbs": acct["bytes"] / (kms * 1e-3) / 1e9,
            "roofline": {"bound": bound, "achieved": ach, "peak": peak, "unit": unit,
                         "frac": ach / peak},
            "flops": acct["flops"], "bytes": acct["bytes"],
            "plan": {"workers": info.num_workers, "head_groups": info.head_groups,
                     "split_rows": info.num_split_rows, "tiles": int(info.total_tiles)},
            "l2": "flushed between steps" if in_l2 else "inputs larger than L2",
        }
        del case, kw, flush
        A._PLAN_CACHE.clear()
        gc.collect()
        torch.cuda.empty_cache()
    return res


def run_gpu(args):
    import gc

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
    from sparse_attn_sharedkv_b200 import sharding as SH
    from tests import workloads as W

    cfg = args.config - 1
    full = W.baseline_case(cfg, device=dev,
                           sequences=args.sequences if cfg == 3 else None)
    acct_full = W.accounting(full)
    kw_full = host_lengths(full.kwargs())
    if ws > 1:
        # The north-star split: one call's rows partitioned over the ranks
        # (decode by batch, TND prefill by token ranges), each rank holding
        # only the KV pages its rows reach; total work fixed (strong scaling).
        bounds = SH.plan_shards(full.q, full.kwargs(), ws)
        sh = SH.make_shard(full.q, full.kwargs(), bounds[rank], rank, compact_pages=True)
        if sh.empty:
            q, kw, acct = None, None, dict(flops=0.0, bytes=1, tokens=0)
        else:
            q, kw = sh.q.contiguous(), host_lengths(sh.kwargs)
            acct = W.accounting(shard_case(W, full, q, sh.kwargs))
    else:
        bounds = [(0, 0)]
        q, kw, acct = full.q, kw_full, acct_full
    in_l2 = acct_full["bytes"] / ws < 2 * L2_BYTES
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev) if in_l2 else None
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if ws > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize()

    if q is not None:
        for _ in range(args.warmup):
            A.sparse_attn_sharedkv(q, return_softmax_lse=True, **kw)
    barrier()
    info = A.last_plan_info if q is not None else None
    launches_per_step = (0 if info is None else 1 + (1 if info.num_split_rows > 0 else 0))

    # ---- value: K full calls, device time per step (max over ranks) ----
    sampler = ClockSampler(local)
    barrier()
    if q is not None:
        step_ms = step_times_ms(A, q, kw, args.steps, flush, stream, sampler)
    else:
        with sampler:
            pass
        step_ms = [0.0] * args.steps
    barrier()
    total_ms = sum(step_ms)

    # ---- roofline: the attention kernel alone (same plan, same inputs) ----
    kern_ms = kernel_alone_ms(A, q, kw, args.steps, flush, stream) if q is not None else 0.0

    # ---- e2e: host buffers in and out, through the public API ----
    e2e_steps = max(1, min(args.steps, 20))
    barrier()
    if q is not None:
        e2e_ms, h2d, d2h = e2e_pipelined(A, q, kw, e2e_steps, dev)
    else:
        e2e_ms, h2d, d2h = 0.0, 0, 0
    barrier()

    # ---- N > 1: the sharded call's one exchange, a gather of the output /
    # LSE shards to rank 0 over NCCL (timed apart from value and e2e) ----
    gather_ms, gather_bytes = 0.0, 0
    if ws > 1:
        o_shape = (full.q.shape[-2], full.head_dim_v or full.q.shape[-1])
        unit_o = o_shape if full.layout_q == "TND" else (full.q.shape[1],) + o_shape
        unit_l = o_shape[:1] if full.layout_q == "TND" else (full.q.shape[1], o_shape[0])
        if q is not None:
            out_t, lse_t = A.sparse_attn_sharedkv(q, return_softmax_lse=True, **kw)
        else:
            out_t = lse_t = None
        gargs = (bounds, rank, unit_o, unit_l, full.q.dtype, dev)
        SH.gather_to_rank0(out_t, lse_t, *gargs)  # warm-up
        barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        SH.gather_to_rank0(out_t, lse_t, *gargs)
        g1.record(stream)
        barrier()
        gather_ms = g0.elapsed_time(g1)
        gather_bytes = (acct_full["tokens"] if full.layout_q == "TND" else full.q.shape[0]
                        * full.q.shape[1]) * o_shape[0] * (o_shape[1] * full.q.element_size() + 4)
        del out_t, lse_t

    # ---- max over ranks ----
    vals = torch.tensor([total_ms, kern_ms, e2e_ms, gather_ms], dtype=torch.float64, device=dev)
    if ws > 1:
        import torch.distributed as dist
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    total_ms, kern_ms, e2e_ms, gather_ms = vals.tolist()
    clocks = sampler.summary()
    peaks, peak_src = load_peaks()

    # ---- N = 1: the other configurations, and the CPU baseline ----
    per_config, cpu = None, None
    if ws == 1:
        c_cpu = None
        if not args.no_cpu_baseline:
            c_cpu = full.to("cpu")
        del q, kw, full, kw_full, flush
        A._PLAN_CACHE.clear()
        gc.collect()
        torch.cuda.empty_cache()
        if not args.no_per_config:
            per_config = other_configs(A, W, [c for c in range(5) if c != cfg], dev, stream,
                                       peaks, min(args.steps, 20))
        if c_cpu is not None:
            ftok = per_token_flops(c_cpu)
            f, s, t, threads = cpu_sample_run(c_cpu, lambda o: ftok[o], args.cpu_seconds)
            _, host = cpu_threads()
            cpu = {"value": f / s / 1e12, "unit": "TFLOP/s", "cores": threads,
                   "host_cores": host, "kind": "port",
                   "sample": f"{t} of {acct_full['tokens']} query tokens (random), {s:.1f} s, "
                             f"{threads} BLAS threads on a {host}-core host"}

    if rank == 0:
        flops = acct_full["flops"]
        ms_step = total_ms / args.steps
        value = flops * args.steps / (total_ms * 1e-3) / 1e12
        bound, ach, peak, unit = roofline(acct, kern_ms, peaks)
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong" if ws > 1 else "weak",
            "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded N(0,1)*0.5, random block tables)",
            "config": {
                "workload": W.BASELINE_NAMES[cfg] + ("" if args.sequences is None or cfg != 3
                                                     else f"_seqs{args.sequences}"),
                "tokens": acct_full["tokens"],
                "keys": acct_full["keys"], "flops_per_step": flops,
                "bytes_per_step": acct_full["bytes"],
                "us_per_call": ms_step * 1e3,
                "hbm_gbs_per_gpu": acct_full["bytes"] / ws / (ms_step * 1e-3) / 1e9,
                "l2": ("flushed between steps (256 MB write)" if in_l2
                       else "inputs larger than L2 (126 MB)"),
                "parallelism": ("single GPU" if ws == 1 else
                                f"{ws} ranks: the call's rows split "
                                f"{'by batch' if full.layout_q != 'TND' else 'by token ranges'}"
                                f" (sharding.plan_shards), strong scaling"),
                "plan": (None if info is None else
                         {"workers": info.num_workers, "head_groups": info.head_groups,
                          "split_rows": info.num_split_rows, "tiles": int(info.total_tiles)}),
            },
            "e2e": {"value": flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms,
                    "what": "public API per step: inputs (q, indices, block tables) copied "
                            "from pinned host memory, output and LSE copied back to pinned "
                            "host memory; steps pipelined over three streams"
                            + ("; each rank copies its own shard" if ws > 1 else "")},
            "roofline": {"bound": bound, "achieved": ach, "peak": peak, "unit": unit,
                         "frac": ach / peak, "peak_source": f"{peak_src} (burst)",
                         "kernel": attention_kernel_name(info), "kernel_ms": kern_ms,
                         "algorithmic_bytes": acct["bytes"], "algorithmic_flops": acct["flops"],
                         "traffic": (load_traffic(W.BASELINE_NAMES[cfg])
                                     if ws == 1 and (args.sequences is None or cfg != 3)
                                     else None),
                         "tensor_tflops": acct["flops"] / (kern_ms * 1e-3) / 1e12,
                         "hbm_gbs": acct["bytes"] / (kern_ms * 1e-3) / 1e9},
            "cpu_baseline": cpu,
            "per_config": per_config,
            "gather": (None if ws == 1 else
                       {"ms": gather_ms, "bytes": gather_bytes,
                        "what": "NCCL gather of every rank's output / LSE shard to rank 0 "
                                "(the sharded call's one exchange); not part of value or e2e"}),
            "clocks": clocks,
            "gpu_launches": launches_per_step * args.steps,
        }
        if args.comparator == "flashmla":
            c2 = W.baseline_case(cfg, device=dev)
            line["comparator"] = flashmla_comparator(A, c2, host_lengths(c2.kwargs()))
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


def _rebuild_call(A, q, kw):
    """Argument structs of one call of (q, kw) (to launch the attention kernel
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
        keep = A.sparse_attn_sharedkv(q, return_softmax_lse=True, **kw)
    finally:
        L.sas_fwd_execute = orig_exec
    torch.cuda.synchronize()
    return captured["prob"], captured["fp"], keep


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=4, choices=[1, 2, 3, 4, 5],
                    help="benchmark configuration (1-based); default 4 (sparse prefill, "
                         "T=32768, H=128, top-k 2048: the largest single-GPU configuration)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sequences", type=int, default=None,
                    help="config 4 only: keep this many of its 4096-token sequences "
                         "(profiling captures of a few GB); default all 8")
    ap.add_argument("--no-per-config", action="store_true",
                    help="skip the per-configuration times of the other four workloads")
    ap.add_argument("--comparator", default=None, choices=["flashmla"],
                    help="also time vLLM's FlashMLA sparse kernel on the same inputs "
                         "(configs 3 and 4; informational, not part of value)")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
