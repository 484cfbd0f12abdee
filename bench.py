"""Benchmark of the GDN-2 hot path on B200: prints ONE JSON line.

Headline workload (per GPU): chunked GDN-2 prefill, B=8, H=16, T=4096,
d_k = d_v = 128, chunk 64, bf16 q/k/v, f32 alpha/beta and state.  A step is one prefill pass over
one batch.  With N GPUs every rank runs its own B=8 batch (batch x head sharding with no
data-path collective: weak scaling); the time is the max over ranks.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

value  : tokens (B*T, all heads) per second over all ranks, inputs resident in HBM.
e2e    : the same through the public API (delta_block_lm_b200.gdn2_prefill) with the step's
         inputs copied from pinned host memory and its outputs copied back inside the timed region.
--impl reference: the reference's CPU algorithm (chunk::scan, crates/mixers/src/chunk.rs:129-250,
         restated in C under oracle/ because the Rust workspace cannot be built here), timed on
         the host cores on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "GDN-2 prefill Mtok/s/GPU, decode tok/s; % of HBM / tensor-core roofline"
B, T, H, D, CHUNK = 8, 4096, 16, 128, 64
# algorithmic minimum bytes per token-head: q,k,v,o bf16 (4 x 128 x 2) + alpha, beta f32
BYTES_PER_TOKEN_HEAD = 4 * D * 2 + 8
FLOPS_PER_TOKEN_HEAD = 2 * (CHUNK * (3 * D + 2 * D) + 3 * D * D)
L2_BYTES = 126 * 2 ** 20


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def ncu_traffic(kernel_key: str):
    """DRAM bytes per launch of `kernel_key` from the committed ncu summary, if one exists."""
    try:
        with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
            return json.load(f).get(kernel_key)
    except Exception:
        return None


class ClockSampler:
    """SM clock and clock-event-reason samples of one GPU during the timed region (read-only).

    NVML is polled from a thread about every millisecond, so a timed region of a few milliseconds
    still gets samples; the first sample is taken before start() returns.  Without NVML it falls
    back to an `nvidia-smi -lms 20` process.
    """

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits (nvml.h: nvmlClocksEventReason*)
    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device_index: int):
        self.proc = None
        self.thread = None
        self.ident = None
        self.samples = []
        try:
            import torch
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            self.ident = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
        except Exception:
            self.ident = str(device_index)

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(self.ident)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(int(os.environ.get("LOCAL_RANK", "0")))

    def start(self):
        import threading
        try:
            nv, h = self._nvml_handle()
            reasons_fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            self._stop = threading.Event()

            def poll():
                while True:
                    try:
                        self.samples.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                             int(reasons_fn(h))))
                    except Exception:
                        return
                    if self._stop.wait(0.001):
                        return

            self.samples.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)), int(reasons_fn(h))))
            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.thread = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.ident, f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.thread is not None:
            self._stop.set()
            self.thread.join(timeout=5)
            if not self.samples:
                return None
            reasons = sorted({n for _, bits in self.samples for n, b in self.REASON_BITS.items() if bits & b})
            return {"sm_mhz": statistics.median(s for s, _ in self.samples), "sm_max_mhz": self.max_mhz,
                    "reasons": reasons, "samples": len(self.samples), "source": "nvml"}
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, val in zip(names, parts[3:7]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvidia-smi"}


# ------------------------------------------------------------------------------ CPU baseline
def cpu_chunk_sample(target_s: float, nthreads: int, reps: int = 1):
    """Time the reference CPU algorithm (chunk.rs restated, f32, chunk 16) on B8/H16/d128 with a
    T chosen so one call takes about target_s seconds.  Returns (tok_per_s, T_sample, secs)."""
    import numpy as np

    from oracle import oracle as O

    def inputs(t):
        rng = np.random.default_rng(0)
        q = rng.standard_normal((B, t, H, D), dtype=np.float32)
        k = rng.standard_normal((B, t, H, D), dtype=np.float32)
        q /= np.linalg.norm(q, axis=-1, keepdims=True)
        k /= np.linalg.norm(k, axis=-1, keepdims=True)
        v = rng.standard_normal((B, t, H, D), dtype=np.float32)
        beta = (1 / (1 + np.exp(-rng.standard_normal((B, t, H))))).astype(np.float32)
        alpha = np.exp(-np.logaddexp(0, -rng.normal(3, 1, (B, t, H)))).astype(np.float32)
        a = np.ascontiguousarray(np.broadcast_to(alpha[..., None], (B, t, H, D)))
        e = np.ascontiguousarray(np.broadcast_to(beta[..., None], (B, t, H, D)))
        return q / math.sqrt(D), k, v, a, e, e

    def run(t):
        x = inputs(t)
        t0 = time.perf_counter()
        O.chunk_scan_f32(*x, chunk=16, nthreads=nthreads, want_scores=False)
        return time.perf_counter() - t0

    probe_t = 32
    dt = run(probe_t)
    t_s = int(max(16, min(T, probe_t * target_s / max(dt, 1e-6))) // 16 * 16)
    times = [run(t_s) for _ in range(reps)]
    secs = statistics.median(times)
    return B * t_s / secs, t_s, secs


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return 0
    cores = host_cores()
    from oracle import oracle as O
    O.build()
    # warm-up and timed samples of the same workload (B8/H16/d128, shorter T)
    vals = []
    t_s = None
    for i in range(args.warmup + args.steps):
        v, t_s, _ = cpu_chunk_sample(target_s=2.0 if t_s is None else 2.0, nthreads=cores)
        if i >= args.warmup:
            vals.append(v)
    value = statistics.median(vals) / 1e6
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "Mtok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": B * t_s / (value * 1e6) * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"c1 prefill sample B{B}/H{H}/T{t_s}/d{D} (chunk 16, the reference's maximum)",
                   "batch_per_gpu": B, "heads": H, "seq_len_sample": t_s, "d_k": D, "d_v": D},
        "cpu_baseline": {"value": value, "unit": "Mtok/s", "cores": cores, "kind": "port",
                         "sample": f"B{B}/H{H}/T{t_s}/d{D} per step, chunk::scan restated in C (OpenMP)",
                         "scope": "the whole host: every core of the node that holds the GPUs (rank 0 alone runs "
                                  "it at any N; the ours arm at N GPUs shares this one host)"},
        "e2e": {"value": value, "unit": "Mtok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------ GPU workloads
def make_prefill_inputs(torch, dev, seed, b=B, t=T, h=H, d=D):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    q = torch.randn((b, t, h, d), device=dev, generator=g)
    k = torch.randn((b, t, h, d), device=dev, generator=g)
    q = (q / q.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    k = (k / k.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    v = torch.randn((b, t, h, d), device=dev, generator=g).to(torch.bfloat16)
    beta = torch.sigmoid(torch.randn((b, t, h), device=dev, generator=g))
    alpha = torch.exp(torch.nn.functional.logsigmoid(3.0 + torch.randn((b, t, h), device=dev, generator=g)))
    return q, k, v, alpha.contiguous(), beta.contiguous()


def bench_prefill(torch, dist, args, dev, rank, world):
    import ctypes

    import delta_block_lm_b200 as dbl
    from delta_block_lm_b200 import _native as N
    from delta_block_lm_b200.kernels import _prefill_args

    q, k, v, alpha, beta = make_prefill_inputs(torch, dev, 1234 + rank)
    out = torch.empty((B, T, H, D), device=dev, dtype=torch.bfloat16)
    fin = torch.empty((B, H, D, D), device=dev, dtype=torch.float32)
    a = _prefill_args(q, k, v, alpha, beta, 1.0 / math.sqrt(D), None, None, None, out, fin, CHUNK)
    lib = N.lib()
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream

    def step():
        N.check(lib.dbl_gdn2_prefill(ctypes.byref(a), sh))

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    sampler = ClockSampler(dev.index)
    sampler.start()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        ev[i][0].record(stream)
        step()
        ev[i][1].record(stream)
    t_end.record(stream)
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    if world > 1:
        dist.barrier()
    elapsed_ms = t_start.elapsed_time(t_end)
    launch_ms = statistics.mean(s.elapsed_time(e) for s, e in ev)
    if world > 1:
        tt = torch.tensor([elapsed_ms, launch_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        elapsed_ms, launch_ms = tt.tolist()
    ms_per_step = elapsed_ms / args.steps
    tokens = B * T * world * args.steps
    value = tokens / (elapsed_ms / 1e3) / 1e6

    # e2e through the public API with host buffers
    e2e_steps = max(1, min(args.steps, 5))
    hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
    ha, hb = alpha.cpu().pin_memory(), beta.cpu().pin_memory()
    ho = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    hf = torch.empty(fin.shape, dtype=fin.dtype).pin_memory()

    def e2e_step():
        # host buffers in, host buffers out: the copies and the kernels of the batch slices are
        # pipelined on side streams that the current stream waits for, so the events below bracket
        # every copy of the step
        dbl.gdn2_prefill_host(hq, hk, hv, ha, hb, device=dev, out=ho, final_state=hf, pieces=8)

    e2e_step()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    s1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = s0.elapsed_time(s1)
    if world > 1:
        tt = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_ms = tt.item()
    h2d = sum(x.numel() * x.element_size() for x in (hq, hk, hv, ha, hb))
    d2h = ho.numel() * ho.element_size() + hf.numel() * hf.element_size()
    # the copy path alone on this rank: the same host buffers in and out, no kernel
    dq_, dk_, dv_ = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    c0, c1, c2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    c0.record(stream)
    for x, y in ((dq_, hq), (dk_, hk), (dv_, hv)):
        x.copy_(y, non_blocking=True)
    c1.record(stream)
    ho.copy_(out, non_blocking=True)
    hf.copy_(fin, non_blocking=True)
    c2.record(stream)
    torch.cuda.synchronize(dev)
    h2d_gbs = (h2d - sum(x.numel() * x.element_size() for x in (ha, hb))) / (c0.elapsed_time(c1) / 1e3) / 1e9
    d2h_gbs = d2h / (c1.elapsed_time(c2) / 1e3) / 1e9
    del dq_, dk_, dv_
    e2e = {"value": B * T * world * e2e_steps / (e2e_ms / 1e3) / 1e6, "unit": "Mtok/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": e2e_steps,
           "copy_rate_rank0_gbs": {"h2d": h2d_gbs, "d2h": d2h_gbs,
                                   "note": "pinned host <-> this rank's GPU, copies alone on one stream; every "
                                           "rank of a node shares the host's memory bandwidth"}}

    hbm, tflops, src = peaks()
    token_heads = B * T * H
    alg_bytes = token_heads * BYTES_PER_TOKEN_HEAD + B * H * D * D * 4
    alg_flops = token_heads * FLOPS_PER_TOKEN_HEAD
    achieved = alg_bytes / (launch_ms / 1e3) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "peak_source": src,
                "traffic": ncu_traffic("gdn2_prefill_c1"),
                "traffic_source": "profiles/ncu_traffic.json: dram bytes of one launch of this kernel at this "
                                  "workload from an ncu capture, not measured in this run",
                "algorithmic_bytes_per_launch": alg_bytes,
                "tensor_tflops": alg_flops / (launch_ms / 1e3) / 1e12,
                "tensor_frac": alg_flops / (launch_ms / 1e3) / 1e12 / tflops,
                "roofline_time_us": max(alg_bytes / hbm / 1e3, alg_flops / tflops / 1e6)}
    input_bytes = sum(x.numel() * x.element_size() for x in (q, k, v, alpha, beta))
    result = {
        "value": value, "ms_per_step": ms_per_step, "launch_ms": launch_ms, "clocks": clocks,
        "e2e": e2e, "gpu_launches": args.steps, "roofline": roofline,
        "config": {"workload": f"c1 prefill B{B}/H{H}/T{T}/d{D} bf16 chunk {CHUNK} per GPU",
                   "batch_per_gpu": B, "heads": H, "seq_len": T, "d_k": D, "d_v": D, "chunk": CHUNK,
                   "global_batch": B * world,
                   "parallelism": f"batch x head sharded over {world} GPU(s), no data-path collective",
                   "l2": f"no flush: inputs {input_bytes / 1e6:.0f} MB > {L2_BYTES / 1e6:.0f} MB L2"},
    }
    return result


def bench_long(torch, dist, args, dev, rank, world):
    """Config 4: one sequence B1/H16/T131072/d128 bf16, sharded along time over the ranks (strong
    scaling).  Phases, each max over ranks: pass 1 (the segment maps of this rank's span), the
    hand-off (the span map composed by the fold kernel, one all_gather of the span boundary objects
    -- the only collective -- and the fold of the earlier ranks' maps; on rank 0 the fold of its
    segment starts and end state), pass 2 (the fold of this rank's segment starts where the hand-off
    has not made them, and the rescan).  At one GPU there is no hand-off and the same work is also
    timed as the single C-ABI call dbl_gdn2_prefill_segmented."""
    from delta_block_lm_b200 import kernels, shard

    t_total = args.long_tokens
    lo, hi = shard.shard_bounds(t_total, world, rank, align=CHUNK)
    q, k, v, alpha, beta = make_prefill_inputs(torch, dev, 777 + rank, b=1, t=hi - lo)
    stream = torch.cuda.current_stream(dev)
    groups = shard.segment_groups(hi - lo, H, shard.sm_count(dev))
    segs = sum(c for _, c, _ in groups)
    K = V = D

    def step(ev=None):
        rec = (lambda i: ev[i].record(stream)) if ev else (lambda i: None)
        rec(0)
        maps = shard.segment_maps(q, k, v, alpha, beta, groups=groups)
        rec(1)
        starts = None
        s0 = torch.zeros((1, H, K, V), device=dev, dtype=torch.float32)
        start = s0
        if rank == 0 and world > 1:
            starts, e0 = shard.rank0_fold(maps, s0)
            shard.exchange_span_states(e0.unsqueeze(0), None, rank, world)
        elif rank > 0:
            At, Bt = shard.compose_maps(*maps)
            As, Bs = shard.exchange_span_states(At, Bt, rank, world)
            start = shard.fold_span_states(Bs[0], As, Bs, rank)
        rec(2)
        out = shard.segmented_prefill(q, k, v, alpha, beta, groups=groups, maps=maps, start=start,
                                      starts=starts)
        rec(3)
        return out

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        step(evs[i])
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    phases = [statistics.mean(ev[j].elapsed_time(ev[j + 1]) for ev in evs) for j in range(3)]
    if world > 1:
        tt = torch.tensor([ms] + phases, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms, *phases = tt.tolist()
    ms_step = ms / args.steps
    schedule = (f"{segs} segments per GPU ({' + '.join(f'{c} x {l // CHUNK}' for _, c, l in groups)} chunks): "
                "pass 1 maps, hand-off, pass 2 rescan")
    uniform = None
    eager = None
    if world > 1:
        # the same step (shard.time_sharded_prefill) captured as one CUDA graph per rank
        # (shard.TimeShardedPrefillGraph): the eager step above is many short launches from Python,
        # and a rank whose host falls behind holds every rank at the all_gather
        eager = {"ms_per_step": ms_step, "phases_ms": {"pass1_segment_maps": phases[0],
                                                       "handoff_compose_allgather_fold": phases[1],
                                                       "pass2_fold_and_rescan": phases[2]}}
        plan = shard.TimeShardedPrefillGraph(q, k, v, alpha, beta, warmup=args.warmup)
        for _ in range(args.warmup):
            plan.replay()
        torch.cuda.synchronize(dev)
        dist.barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        for _ in range(args.steps):
            plan.replay()
        g1.record(stream)
        torch.cuda.synchronize(dev)
        ms_step = _max_over_ranks(torch, dist, world, dev, g0.elapsed_time(g1) / args.steps)
        plan.release()
        del plan
        torch.cuda.synchronize(dev)
        dist.barrier()
        schedule += "; the step replayed as one CUDA graph per rank (shard.TimeShardedPrefillGraph)"
    if world == 1:
        # one GPU: the value is the single C-ABI call with the library's schedule (segments = 0: a
        # lead segment scanned from the initial state beside the maps of the other segments, which
        # needs no hand-off); the equal-segment steps timed above are kept for comparison
        uniform = {"schedule": schedule, "ms_per_step": ms_step,
                   "phases_ms": {"pass1_segment_maps": phases[0], "fold": phases[1],
                                 "pass2_fold_and_rescan": phases[2]}}
        for _ in range(args.warmup):
            kernels.gdn2_prefill_segmented(q, k, v, alpha, beta, segments=0)
        torch.cuda.synchronize(dev)
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(stream)
        for _ in range(args.steps):
            kernels.gdn2_prefill_segmented(q, k, v, alpha, beta, segments=0)
        c1.record(stream)
        torch.cuda.synchronize(dev)
        ms_step = c0.elapsed_time(c1) / args.steps
        m = shard.sm_count(dev) // H
        n = (hi - lo) // CHUNK
        lt = (5 * n + 5 * m + 8) // (5 * m + 9)
        schedule = (f"dbl_gdn2_prefill_segmented(segments=0): lead segment of {n - m * lt} chunks scanned "
                    f"from the initial state on a side stream beside the maps of {m - 1} segments of {lt} "
                    f"chunks, fold, one rescan of {m} segments of {lt} chunks")
    hbm, _, src = peaks()
    alg = t_total * H * BYTES_PER_TOKEN_HEAD + H * D * D * 4
    handoff_bytes = world * H * D * (D + D) * 4 if world > 1 else 0
    return {"workload": f"c4 B1/H{H}/T{t_total}/d{D} bf16 chunk {CHUNK}, time-sharded over {world} GPU(s)",
            "value": t_total / (ms_step / 1e3) / 1e6, "unit": "Mtok/s", "ms_per_step": ms_step,
            "scaling": "strong", "span_tokens": hi - lo, "schedule": schedule,
            "eager_steps": eager,
            "limited_by": "the per-chunk scan chain: three scans of a segment in sequence (maps A, maps B, "
                          "rescan)" + ("" if world == 1 else ", plus the hand-off"),
            "handoff": "one all_gather of (A_g | B_g) [H,K,K+V] f32 per rank" if world > 1 else None,
            "handoff_bytes_gathered_per_rank": handoff_bytes,
            "python_segments_one_gpu": uniform,
            "roofline": {"bound": "hbm", "algorithmic_bytes": alg,
                         "achieved_gbs_aggregate": alg / (ms_step / 1e3) / 1e9, "peak_per_gpu": hbm,
                         "frac_of_aggregate_peak": alg / (ms_step / 1e3) / 1e9 / (hbm * world),
                         "peak_source": src}}


def _max_over_ranks(torch, dist, world, dev, x):
    if world > 1:
        t = torch.tensor([x], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()
    return x


def bench_decode(torch, args, dev, dist=None, world=1):
    """Config 2: 256 sequences x 16 heads x 128^2 f32 state, 64 consecutive in-place steps.  With N
    ranks every rank decodes its own 256 sequences (sequence sharding, no communication): the time
    is the max over ranks and the rate counts every rank's sequences."""
    import ctypes

    from delta_block_lm_b200 import _native as N
    from delta_block_lm_b200.kernels import _strides

    n, steps = 256, 64
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    state = 0.02 * torch.randn((n, H, D, D), device=dev, generator=g)
    q = torch.randn((steps, n, H, D), device=dev, generator=g)
    k = torch.randn((steps, n, H, D), device=dev, generator=g)
    q = (q / q.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    k = (k / k.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    v = torch.randn((steps, n, H, D), device=dev, generator=g).to(torch.bfloat16)
    beta = torch.sigmoid(torch.randn((steps, n, H), device=dev, generator=g))
    alpha = torch.exp(torch.nn.functional.logsigmoid(3.0 + torch.randn((steps, n, H), device=dev, generator=g)))
    out = torch.empty((n, H, D), device=dev, dtype=torch.bfloat16)
    lib = N.lib()
    argv = []
    for s in range(steps):
        a = N.DecodeArgs()
        a.batch, a.heads, a.key_dim, a.value_dim, a.dtype, a.scale = n, H, D, D, N.DBL_BF16, 1 / math.sqrt(D)
        a.q, a.k, a.v = q[s].data_ptr(), k[s].data_ptr(), v[s].data_ptr()
        a.q_stride, a.k_stride, a.v_stride = _strides(q[s], 3), _strides(k[s], 3), _strides(v[s], 3)
        a.alpha, a.beta, a.state = alpha[s].data_ptr(), beta[s].data_ptr(), state.data_ptr()
        a.out, a.out_stride = out.data_ptr(), _strides(out, 3)
        argv.append(a)
    stream = torch.cuda.current_stream(dev)
    sh = stream.cuda_stream

    def run64():
        for a in argv:
            N.check(lib.dbl_gdn2_decode_step(ctypes.byref(a), sh))

    for _ in range(2):
        run64()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    e0.record(stream)
    for _ in range(reps):
        run64()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms_step = _max_over_ranks(torch, dist, world, dev, e0.elapsed_time(e1) / (reps * steps))
    hbm, _, src = peaks()
    alg = n * H * (2 * D * D * 4 + 3 * D * 2 + D * 2 + 8)
    gbs = alg / (ms_step / 1e3) / 1e9
    return {"workload": f"c2 decode {n} seq x H{H} x {D}x{D} f32 state per GPU, {steps} steps (x{reps}), "
                        f"{world} GPU(s) sharded by sequence",
            "tok_per_s": world * n / (ms_step / 1e3), "us_per_step": ms_step * 1e3, "scaling": "weak",
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                         "peak_source": src, "algorithmic_bytes_per_launch": alg,
                         "traffic": ncu_traffic("gdn2_decode_c2")},
            "gpu_launches": reps * steps}


def bench_relay(torch, args, dev, dist=None, world=1):
    """Config 3: shared 4096-token prefix + 64 x 1024 own tokens, H16, hd128, bf16, 1 query/seq.
    With N ranks every rank serves its own 64 sequences with a replica of the prefix (no
    communication): the time is the max over ranks and the rate counts every rank's queries."""
    import delta_block_lm_b200 as dbl

    n, lp, lo = 64, 4096, 1024
    g = torch.Generator(device=dev)
    g.manual_seed(9)
    mk = lambda *s: torch.randn(s, device=dev, generator=g).to(torch.bfloat16)  # noqa: E731
    q, kp, vp, ko, vo = mk(n, H, D), mk(H, lp, D), mk(H, lp, D), mk(n, H, lo, D), mk(n, H, lo, D)
    ws = torch.empty(dbl.relay_workspace_bytes(n, H, D, lp, lo), device=dev, dtype=torch.uint8)
    out = torch.empty((n, H, D), device=dev, dtype=torch.bfloat16)
    stream = torch.cuda.current_stream(dev)
    for _ in range(3):
        dbl.relay_merge_decode(q, kp, vp, ko, vo, out=out, workspace=ws, return_stats=False)
    torch.cuda.synchronize(dev)
    reps = 20
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        dbl.relay_merge_decode(q, kp, vp, ko, vo, out=out, workspace=ws, return_stats=False)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = _max_over_ranks(torch, dist, world, dev, e0.elapsed_time(e1) / reps)
    hbm, _, src = peaks()
    alg = (2 * H * lp * D + 2 * n * H * lo * D + 2 * n * H * D) * 2
    gbs = alg / (ms / 1e3) / 1e9
    return {"workload": f"c3 relay decode prefix {lp} + {n} x {lo} own per GPU, H{H}, hd{D}, bf16, "
                        f"{world} GPU(s) sharded by sequence",
            "queries_per_s": world * n * H / (ms / 1e3), "us_per_call": ms * 1e3, "scaling": "weak",
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                         "peak_source": src, "algorithmic_bytes_per_launch": alg,
                         "traffic": ncu_traffic("relay_merge_c3")},
            "gpu_launches": reps}


def _timed(torch, dev, fn, reps, warm=3):
    stream = torch.cuda.current_stream(dev)
    for _ in range(warm):
        fn()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1) / reps


def bench_config0(torch, dev):
    """Config 0 (the reference's CPU-runnable case): B2/H4/T512/d64 f32, chunked prefill on the GPU.
    Latency-bound (4.4 MB of traffic); reported as time and tokens/s, with no roofline claim."""
    import delta_block_lm_b200 as dbl
    b, t, h, d = 2, 512, 4, 64
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    q = torch.randn((b, t, h, d), device=dev, generator=g)
    k = torch.randn((b, t, h, d), device=dev, generator=g)
    q, k = q / q.norm(dim=-1, keepdim=True), k / k.norm(dim=-1, keepdim=True)
    v = torch.randn((b, t, h, d), device=dev, generator=g)
    beta = torch.sigmoid(torch.randn((b, t, h), device=dev, generator=g))
    alpha = torch.exp(torch.nn.functional.logsigmoid(3.0 + torch.randn((b, t, h), device=dev, generator=g)))
    ms = _timed(torch, dev, lambda: dbl.gdn2_prefill(q, k, v, alpha, beta), 50)
    return {"workload": f"c0 B{b}/H{h}/T{t}/d{d} f32", "ms": ms, "mtok_s": b * t / (ms / 1e3) / 1e6,
            "gpu_launches": 50}


def bench_dropin_c1(torch, dev):
    """The reference's own drop-in call, delta_kernels::gdn_training_scan (crates/kernels/src/
    gdn_training_ops.rs:288-333, what scan_selected(FusedGdn2) calls), at the config-1 shape
    B8/H16/T4096/K=V=128 bf16: channel-wise gate tensors (here the scalar gates broadcast over the
    channels), valid / reset, initial state, f32 outputs and scores."""
    import delta_block_lm_b200 as dbl
    q, k, v, alpha, beta = make_prefill_inputs(torch, dev, 1234)
    a = alpha[..., None].expand(B, T, H, D).contiguous()
    e = beta[..., None].expand(B, T, H, D).contiguous()
    valid, reset = torch.ones((B, T), device=dev), torch.zeros((B, T), device=dev)
    init = torch.zeros((B, H, D, D), device=dev)
    qs = q / math.sqrt(D)  # the mixer's pre-scaled q: the call's input, made outside the timed region
    ms = _timed(torch, dev, lambda: dbl.gdn_training_scan(qs, k, v, a, e, e, valid, reset, init, 16),
                reps=3, warm=1)
    del a, e, qs
    return {"workload": f"gdn_training_scan B{B}/H{H}/T{T}/K=V={D} bf16, channel-wise gates, f32 outputs + scores",
            "ms": ms, "mtok_s": B * T / (ms / 1e3) / 1e6, "gpu_launches": 4}


def bench_backward(torch, args, dev):
    """Training shape of the reference's fused scan (B8/T512/H4, K32/V64, f32, chunk 16): the
    backward (gdn_training_backward) and, for context, the forward gdn_training_scan."""
    import delta_block_lm_b200 as dbl

    b, t, h, k_, v_ = 8, 512, 4, 32, 64
    g = torch.Generator(device=dev)
    g.manual_seed(11)
    rn = lambda *s: torch.randn(s, device=dev, generator=g)  # noqa: E731
    q, k = rn(b, t, h, k_) / math.sqrt(k_), rn(b, t, h, k_) / math.sqrt(k_)
    v, w = rn(b, t, h, v_), torch.sigmoid(rn(b, t, h, v_))
    a, e = torch.sigmoid(3.0 + rn(b, t, h, k_)), torch.sigmoid(rn(b, t, h, k_))
    valid, reset = torch.ones(b, t, device=dev), torch.zeros(b, t, device=dev)
    init = torch.zeros(b, h, k_, v_, device=dev)
    go, gf, gs = rn(b, t, h, v_), rn(b, h, k_, v_), rn(b, t, h)
    stream = torch.cuda.current_stream(dev)

    def timed(fn, reps=10):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / reps

    ms_b = timed(lambda: dbl.gdn_training_backward(q, k, v, a, e, w, valid, reset, init, go, gf, gs, chunk_size=16))
    ms_f = timed(lambda: dbl.gdn_training_scan(q, k, v, a, e, w, valid, reset, init, 16))
    # the reference's pairing: the forward saves its context, the backward reads it (a full step)
    args_ = (q, k, v, a, e, w, valid, reset, init)

    def step_saved():
        _, ctx = dbl.gdn_training_scan_saved(*args_, 16)
        dbl.gdn_training_backward_saved(*args_, go, ctx, gf, gs, chunk_size=16)

    ms_step = timed(step_saved)
    tokens = b * t
    line = {"metric": "GDN-2 training scan backward Mtok/s (gdn_training_backward)",
            "value": tokens / (ms_b / 1e3) / 1e6, "unit": "Mtok/s", "ms_per_step": ms_b, "n_gpus": 1,
            "higher_is_better": True, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"B{b}/T{t}/H{h}/K{k_}/V{v_} f32 chunk 16 (the reference's training shape)",
                       "forward_ms": ms_f, "forward_mtok_s": tokens / (ms_f / 1e3) / 1e6,
                       "training_step_saved_context_ms": ms_step,
                       "training_step_recomputing_ms": ms_f + ms_b},
            # chunked forms at this shape: the recomputing backward launches the chunk-map, main,
            # reverse-map, reverse and gradient kernels; the forward the chunk-map, main and score
            # kernels; a saved-context step the forward's three and the backward's last three
            "gpu_launches": 10 * 5 + 10 * 3 + 10 * 6}
    if not args.no_cpu_baseline:
        # the f64 C restatement of the reference's backward on one (b) row of the workload
        sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
        from oracle import oracle as O
        host = [x[:1].double().cpu().numpy() for x in (q, k, v, a, e, w, go, gf, gs)]
        c0 = time.perf_counter()
        O.training_backward(*host[:7], host[7], host[8], valid[:1].cpu().numpy() > 0, reset[:1].cpu().numpy() > 0,
                            init[:1].double().cpu().numpy())
        sec = time.perf_counter() - c0
        line["cpu_baseline"] = {"value": t / sec / 1e6, "unit": "Mtok/s", "cores": 1, "kind": "port",
                                "sample": f"B1/T{t}/H{h}/K{k_}/V{v_}, f64 C restatement of gdn_training.rs:117-284, "
                                          f"{sec:.2f} s"}
    return line


def bench_prologue(torch, args, dev):
    """The GDN-2 mixer prologue (conv + silu + l2 for q, k; conv + silu for v; decay and sigmoid
    gates) at the config-1 shape: B8/T4096/H16, K = V = 128, bf16 projections in, bf16 q, k, v and
    f32 gates out (HBM-bound)."""
    import delta_block_lm_b200 as dbl

    b, t, h, d = B, T, H, D
    g = torch.Generator(device=dev)
    g.manual_seed(13)
    rn = lambda *s, dt=torch.float32: torch.randn(s, device=dev, generator=g).to(dt)  # noqa: E731
    proj = [rn(b, t, h * d, dt=torch.bfloat16) for _ in range(6)]
    conv = [0.3 * rn(4, h * d) for _ in range(3)]
    bias, scale = rn(h * d), 0.3 * rn(h)
    valid, reset = torch.ones(b, t, device=dev), (torch.rand(b, t, device=dev, generator=g) > 0.999).float()
    stream = torch.cuda.current_stream(dev)
    call = lambda: dbl.gdn2_prologue(*proj, *conv, bias, scale, valid, reset, heads=h, out_dtype=torch.bfloat16)  # noqa: E731
    for _ in range(3):
        call()
    torch.cuda.synchronize(dev)
    reps = 20
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        call()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / reps
    hbm, _, src = peaks()
    # per token-head: 6 bf16 projection rows in; q, k, v bf16 and alpha, erase, write f32 out
    alg = b * t * h * (6 * d * 2 + 3 * d * 2 + 3 * d * 4)
    gbs = alg / (ms / 1e3) / 1e9
    line = {"metric": "GDN-2 mixer prologue Mtok/s", "value": b * t / (ms / 1e3) / 1e6, "unit": "Mtok/s",
            "ms_per_step": ms, "n_gpus": 1, "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"B{b}/T{t}/H{h}/K=V={d}, conv width 4, bf16 in/out, f32 gates"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                         "peak_source": src, "algorithmic_bytes_per_launch": alg},
            "gpu_launches": reps}
    if not args.no_cpu_baseline:
        # the numpy restatement of the prologue (f64) on the first 1024 tokens of one row
        sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
        from oracle import oracle as O
        ts = 1024
        host = [x[:1, :ts].float().cpu().numpy() for x in proj]
        c0 = time.perf_counter()
        O.gdn2_prologue(*host, *(x.cpu().numpy() for x in conv), bias.cpu().numpy(), scale.cpu().numpy(),
                        valid[:1, :ts].cpu().numpy(), reset[:1, :ts].cpu().numpy(), heads=h)
        sec = time.perf_counter() - c0
        line["cpu_baseline"] = {"value": ts / sec / 1e6, "unit": "Mtok/s", "cores": 1, "kind": "port",
                                "sample": f"B1/T{ts}/H{h}/K=V={d}, numpy f64 restatement of lib.rs:446-528, {sec:.2f} s"}
    return line


def bench_relay_attn(torch, args, dev, with_cpu=True):
    """Reference-layout relay attention (relay_attention_kernel.rs:38-130: +-128 document window
    plus 16 relay slots, head width 64) at B8/H16/T4096 with 1024-token documents, bf16 on the
    tensor cores; the f32 CUDA-core path and the f64 CPU oracle on a bounded sample for context."""
    import delta_block_lm_b200 as dbl

    b, h, t, dl = 8, 16, 4096, 1024
    nd = b * t // dl
    g = torch.Generator(device=dev)
    g.manual_seed(17)
    rn = lambda *s: torch.randn(s, device=dev, generator=g)  # noqa: E731
    pos = torch.arange(t, device=dev, dtype=torch.int32)
    ds = (pos // dl * dl).expand(b, t).contiguous()
    de = (ds + dl - 1).contiguous()
    di = (torch.arange(b, device=dev, dtype=torch.int32)[:, None] * (t // dl) + pos // dl).contiguous()
    x32 = [rn(b, h, t, 64) for _ in range(3)] + [rn(nd, h, 16, 64) for _ in range(2)]
    x16 = [x.to(torch.bfloat16) for x in x32]
    stream = torch.cuda.current_stream(dev)

    def timed(fn, reps=20):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / reps

    ms = timed(lambda: dbl.relay_attention_forward(*x16, di, ds, de))
    ms32 = timed(lambda: dbl.relay_attention_forward(*x32, di, ds, de), reps=5)
    hbm, _, src = peaks()
    # per query row: q, k, v read and o written (64 bf16 each) and the f32 statistic pair;
    # plus the relay slots once per (document, head)
    alg = b * h * t * (4 * 64 * 2 + 8) + 2 * nd * h * 16 * 64 * 2
    gbs = alg / (ms / 1e3) / 1e9
    # in-window keys per query (document edges clip the +-128 window) for the FLOP count
    win = sum(min(i + 128, dl - 1) - max(i - 128, 0) + 1 for i in range(dl)) / dl
    flops = b * h * t * (win + 16) * 64 * 4
    line = {"metric": "relay attention (reference layout) Mtok/s", "value": b * t / (ms / 1e3) / 1e6,
            "unit": "Mtok/s", "ms_per_step": ms, "n_gpus": 1, "higher_is_better": True, "dtype": "bf16",
            "data": "synthetic (seeded normal q, k, v and relay slots)",
            "config": {"workload": f"B{b}/H{h}/T{t}/hd64, documents of {dl} tokens, 16 relay slots, radius 128",
                       "f32_ms": ms32, "tflops_bf16": flops / (ms / 1e3) / 1e12},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                         "peak_source": src, "algorithmic_bytes_per_launch": alg},
            "gpu_launches": 20 + 5}
    if with_cpu:
        sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
        from oracle import oracle as O
        import numpy as np
        ts = 1024
        sel = [x[:1, :1, :ts].float().cpu().numpy().astype(np.float64) for x in x32[:3]]
        rel = [x[:1, :1].float().cpu().numpy().astype(np.float64) for x in x32[3:]]
        c0 = time.perf_counter()
        O.relay_window(*sel, *rel, di[:1, :ts].cpu().numpy(), ds[:1, :ts].cpu().numpy(), de[:1, :ts].cpu().numpy())
        sec = time.perf_counter() - c0
        line["cpu_baseline"] = {"value": ts / sec / 1e6, "unit": "Mtok/s (one head)", "cores": 1, "kind": "port",
                                "sample": f"B1/H1/T{ts}, one document, f64 C restatement of relay_forward_kernel, "
                                          f"{sec:.2f} s"}
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-secondary", action="store_true", help="skip the decode / relay lines")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["prefill", "long", "decode", "relay", "backward", "prologue", "relay_attn",
                                           "config0", "dropin"],
                    default="prefill",
                    help="prefill: config 1 (the headline, weak-scaled); long: config 4 (time-sharded); "
                         "decode: config 2 alone; relay: config 3 alone; backward: the fused scan's "
                         "backward at the reference's training shape; prologue: the mixer prologue; "
                         "relay_attn: reference-layout relay attention (1 GPU); config0: config 0 alone; "
                         "dropin: the reference's gdn_training_scan call at the config-1 shape (1 GPU)")
    ap.add_argument("--long-tokens", type=int, default=131072)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import datetime

    import torch
    import torch.distributed as dist

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    from delta_block_lm_b200 import _native
    _native.lib()
    if args.workload == "long":
        r = bench_long(torch, dist, args, dev, rank, world)
        line = {"metric": "GDN-2 long-context prefill Mtok/s (config 4, time-sharded)", "value": r["value"],
                "unit": "Mtok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "strong", "dtype": "bf16",
                "data": "synthetic", "config": {k_: v_ for k_, v_ in r.items() if k_ not in ("value", "ms_per_step")}}
        if rank == 0:
            print(json.dumps(line), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return 0
    if args.workload == "prologue":
        if world > 1:
            raise SystemExit("--workload prologue runs on one GPU")
        print(json.dumps(bench_prologue(torch, args, dev)), flush=True)
        return 0
    if args.workload == "relay_attn":
        if world > 1:
            raise SystemExit("--workload relay_attn runs on one GPU")
        print(json.dumps(bench_relay_attn(torch, args, dev, with_cpu=not args.no_cpu_baseline)), flush=True)
        return 0
    if args.workload in ("config0", "dropin"):
        # the headline's `secondary.config0` and `secondary.training_scan_c1_dropin` measurements alone
        if world > 1:
            raise SystemExit("--workload config0/dropin runs on one GPU")
        print(json.dumps(bench_config0(torch, dev) if args.workload == "config0" else bench_dropin_c1(torch, dev)),
              flush=True)
        return 0
    if args.workload == "backward":
        if world > 1:
            raise SystemExit("--workload backward runs on one GPU")
        print(json.dumps(bench_backward(torch, args, dev)), flush=True)
        return 0
    if args.workload in ("decode", "relay"):
        # single-kernel lines (the same measurements as the headline's `secondary` object)
        if world > 1:
            raise SystemExit("--workload decode/relay runs on one GPU")
        if args.workload == "decode":
            r = bench_decode(torch, args, dev)
            line = {"metric": "GDN-2 decode tok/s (config 2)", "value": r["tok_per_s"], "unit": "tok/s",
                    "ms_per_step": r["us_per_step"] / 1e3}
        else:
            r = bench_relay(torch, args, dev)
            line = {"metric": "relay merge (sequence, head) queries/s (config 3)", "value": r["queries_per_s"],
                    "unit": "queries/s", "ms_per_step": r["us_per_call"] / 1e3}
        line.update({"n_gpus": 1, "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
                     "config": {"workload": r["workload"]}, "roofline": r["roofline"],
                     "gpu_launches": r["gpu_launches"]})
        print(json.dumps(line), flush=True)
        return 0
    res = bench_prefill(torch, dist, args, dev, rank, world)
    line = {"metric": METRIC, "value": res["value"], "unit": "Mtok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded normal q/k/v L2-normalised, beta = sigmoid(N(0,1)), "
                    "alpha = exp(logsigmoid(N(3,1))))",
            "config": res["config"], "clocks": res["clocks"], "e2e": res["e2e"],
            "gpu_launches": res["gpu_launches"], "roofline": res["roofline"],
            "kernel_ms_per_launch": res["launch_ms"]}
    if not args.no_secondary:
        # every rank takes part: decode and relay as sequence-sharded replicas, config 4 through the
        # time-sharded hand-off (the only collective)
        sec = {"decode": bench_decode(torch, args, dev, dist, world), "relay": bench_relay(torch, args, dev, dist, world),
               "long": bench_long(torch, dist, argparse.Namespace(**{**vars(args), "steps": 5, "warmup": 3}), dev,
                                  rank, world)}
        if rank == 0:
            line["secondary"] = sec
    if world == 1 and rank == 0:
        if not args.no_secondary:
            line["secondary"]["config0"] = bench_config0(torch, dev)
            line["secondary"]["training_scan_c1_dropin"] = bench_dropin_c1(torch, dev)
            # the training scan at the reference's training shape (the backward workload's line,
            # without its CPU sample)
            tr = bench_backward(torch, argparse.Namespace(**{**vars(args), "no_cpu_baseline": True}), dev)
            line["secondary"]["training_scan"] = {
                "workload": tr["config"]["workload"], "backward_ms": tr["ms_per_step"],
                "backward_mtok_s": tr["value"], "forward_ms": tr["config"]["forward_ms"],
                "training_step_saved_context_ms": tr["config"]["training_step_saved_context_ms"],
                "training_step_recomputing_ms": tr["config"]["training_step_recomputing_ms"],
                "gpu_launches": tr["gpu_launches"]}
        if not args.no_cpu_baseline:
            cores = host_cores()
            v, t_s, secs = cpu_chunk_sample(target_s=4.0, nthreads=cores, reps=3)
            line["cpu_baseline"] = {"value": v / 1e6, "unit": "Mtok/s", "cores": cores, "kind": "port",
                                    "sample": f"B{B}/H{H}/T{t_s}/d{D}, chunk 16, median of 3 x {secs:.1f} s "
                                              "(chunk::scan restated in C, OpenMP)"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
