"""Benchmark: Chronos-2-base encoder forward (bf16, fp32 accumulate) on B200.

Workload (the benchmark's configs[1]): per GPU 256 independent univariate
series, context 2048 (128 patches), prediction_length 64 (4 future patches),
synthetic seeded data (random walk + daily/weekly sinusoids + noise, 2% NaN),
random-init weights (seed 0, N(0, 0.02), RMS weights 1).  One step = one
forward over the batch -> (256, 21, 64) quantile forecasts.  Under torchrun
each rank runs its own 256 series (weak scaling) and the quantile outputs are
gathered to every rank with NCCL all_gather inside the step.

Metric: forecasts/s (whole job).  Timing: CUDA events on the launching stream
per step; L2 is flushed (256 MB write) before every timed step, outside the
event pair; barrier + synchronize around the timed loop; max over ranks.
Per-kernel durations (roofline, kernel shares, launch count) come from a
second, instrumented pass over the same steps, outside the timed region.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

--impl reference times the reference algorithm's CPU path (the CPU oracle
restatement of cutechronos CuteChronos2Model.forward, fp32 torch on all host
cores) on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import ctypes as C
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "forecasts/sec/GPU, Chronos-2-base shape ctx2048 bf16; p50 batch-1 latency"
UNIT = "forecasts/s"
GFLOP_PER_FORECAST = None  # filled from the oracle's FLOP formula


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def log(*a):
    print(*a, file=sys.stderr, flush=True)


class ClockSampler:
    """SM clock, power and throttle reasons of this rank's GPU during the timed
    region: NVML every ~10 ms in a thread (the device found by the UUID torch
    reports, so a remapped CUDA_VISIBLE_DEVICES cannot pick another GPU), plus
    one sample at start and one at stop; nvidia-smi -lms 200 when NVML is
    unavailable."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.rows = []
        self.proc = None
        self.thread = None
        self.nvml = None
        self.handle = None
        self.stop_flag = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(gpu_index).uuid)
            self.handle = pynvml.nvmlDeviceGetHandleByUUID("GPU-" + uuid if not uuid.startswith("GPU-") else uuid)
            self.nvml = pynvml
        except Exception:
            self.nvml = None

    def _sample_nvml(self):
        n = self.nvml
        try:
            sm = n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)
            mx = n.nvmlDeviceGetMaxClockInfo(self.handle, n.NVML_CLOCK_SM)
            pw = n.nvmlDeviceGetPowerUsage(self.handle) / 1000.0
            rs = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
        except Exception:
            return
        flag = lambda bit: "Active" if rs & bit else "Not Active"  # noqa: E731
        self.rows.append([str(self.gpu), str(sm), str(mx), f"{pw:.2f}", hex(rs),
                          flag(n.nvmlClocksEventReasonHwSlowdown), flag(n.nvmlClocksEventReasonHwThermalSlowdown),
                          flag(n.nvmlClocksEventReasonSwThermalSlowdown), flag(n.nvmlClocksEventReasonSwPowerCap)])

    def _loop_nvml(self):
        while not self.stop_flag.wait(0.01):
            self._sample_nvml()

    def start(self):
        if self.nvml is not None:
            self._sample_nvml()
            self.thread = threading.Thread(target=self._loop_nvml, daemon=True)
            self.thread.start()
            return
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def stop(self):
        if self.nvml is not None:
            self.stop_flag.set()
            if self.thread is not None:
                self.thread.join(timeout=2)
            self._sample_nvml()
            return
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=2)
            except Exception:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r[1]) for r in self.rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in self.rows if num(r[2]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows),
                "power_w_max": max((num(r[3]) or 0.0) for r in self.rows)}


def gemm_traffic_per_launch():
    """DRAM bytes per GEMM launch from the committed ncu summary of the same
    workload (profiles/gemm_dram_cfg1.txt); None when it is absent."""
    p = Path(__file__).resolve().parent / "profiles" / "gemm_dram_cfg1.txt"
    try:
        for line in p.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                return int(line.split(":")[1])
    except OSError:
        pass
    return None


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained", d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


class CpuReference:
    """The reference's own CPU implementation of the path on the host cores:
    ``cutechronos.model.CuteChronos2Model`` (its torch fallbacks on CPU
    tensors, fp32, all host threads) as staged into ``oracle/_ref`` by
    ``oracle/stage_reference.py``; when that folder is absent, the CPU oracle
    restatement of the same forward (kind "port")."""

    def __init__(self):
        from cutechronos_b200.model import CuteChronos2Config, CuteChronos2Model
        from cutechronos_b200.workloads import seeded_init_, seeded_state_dict
        from oracle import chronos2_oracle as orc
        from oracle.stage_reference import load_reference_model_class

        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        self.orc = orc
        ref = load_reference_model_class()
        if ref is not None:
            cfg_cls, mod_cls = ref
            self.kind = "reference"
            self.model = seeded_init_(mod_cls(cfg_cls()), seed=0).eval()
            self.W = None
        else:
            self.kind = "port"
            self.model = None
            m = CuteChronos2Model(CuteChronos2Config())
            self.W = seeded_state_dict([(n, tuple(p.shape)) for n, p in m.named_parameters()], seed=0)

    @property
    def what(self) -> str:
        if self.kind == "reference":
            return "reference cutechronos.model.CuteChronos2Model.forward (fp32, torch CPU path, staged in oracle/_ref)"
        return "CPU oracle restatement of CuteChronos2Model.forward (fp32 torch)"

    def forecasts_per_s(self, n_series: int, L: int = 2048, N: int = 4, seed: int = 1) -> float:
        from cutechronos_b200.workloads import series_cfg1

        ctx = series_cfg1(n_series, L, seed)
        with torch.inference_mode():
            t0 = time.perf_counter()
            if self.model is not None:
                self.model(ctx, num_output_patches=N)
            else:
                self.orc.forward(self.orc.OracleConfig(), self.W, ctx, None, N)
            return n_series / (time.perf_counter() - t0)


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    n = 32
    ref = CpuReference()
    for _ in range(args.warmup):
        ref.forecasts_per_s(2)
    vals = [ref.forecasts_per_s(n) for _ in range(args.steps)]
    threads = ref.threads
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * n / value,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (configs[1] generator, seed 1)",
        "config": {"workload": "configs[1]: B=256 univariate, ctx 2048, pred 64 (4 patches), Chronos-2-base",
                   "sample": f"{n} series per step (forecasts are independent per series, so the rate "
                             "scales linearly to the full batch)", "l2": "n/a (CPU)"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": ref.kind,
                         "sample": f"{n} series of configs[1] per step, {ref.what}"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def graph_latency_ms(model, x, N, reps=50):
    """p50 latency of one forward replayed from a CUDA graph (batch-1 serving)."""
    model(x, num_output_patches=N)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        model(x, num_output_patches=N)
        with torch.cuda.graph(g, stream=s):
            model(x, num_output_patches=N)
    torch.cuda.synchronize()
    lats = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        b.synchronize()
        lats.append(a.elapsed_time(b))
    return statistics.median(lats)


def forecasts_per_s(model, ctx, N, gid, flush, steps=5, warmup=2):
    for _ in range(warmup):
        model(ctx, num_output_patches=N, group_ids=gid)
    torch.cuda.synchronize()
    tot = 0.0
    for i in range(steps):
        flush.fill_(i & 0xFF)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        model(ctx, num_output_patches=N, group_ids=gid)
        b.record()
        b.synchronize()
        tot += a.elapsed_time(b)
    return ctx.shape[0] * steps / (tot / 1e3)


def other_configs(model_bf16, dev, flush):
    """The benchmark's other configs on one GPU (their own workloads; not the
    headline line): configs[0] fp32 batch-1 latency (CUDA graph) and
    forecasts/s for configs[2], [3], [4]."""
    from cutechronos_b200.model import CuteChronos2Config, CuteChronos2Model
    from cutechronos_b200.workloads import config0, config2, config3, config4, seeded_init_

    out = {}
    w0 = config0()
    m32 = seeded_init_(CuteChronos2Model(CuteChronos2Config()), seed=0).to(dev, torch.float32).eval()
    out["cfg0_b1_ctx512_f32_p50_ms"] = graph_latency_ms(m32, w0.context.to(dev), w0.num_output_patches)
    del m32
    torch.cuda.empty_cache()
    for name, w in (("cfg2_g64x8_ctx2048", config2()), ("cfg3_b32_ctx8192", config3()),
                    ("cfg4_b4096_ctx512", config4())):
        out[name + "_forecasts_per_s"] = forecasts_per_s(model_bf16, w.context.to(dev), w.num_output_patches,
                                                         w.group_ids, flush)
    # configs[1] with the TurboQuant K/V hook on (4 bits, prod keys, mse values)
    from cutechronos_b200.workloads import series_cfg1
    model_bf16.enable_turboquant_kv(bits=4, key_mode="prod", value_mode="mse")
    try:
        out["cfg1_turboquant_kv4_forecasts_per_s"] = forecasts_per_s(model_bf16, series_cfg1(256, 2048, 1).to(dev),
                                                                     4, None, flush)
    finally:
        model_bf16.disable_turboquant_kv()
    return out


def cfg4_sharded(model_bf16, dev, flush, steps, warmup, grouped=False):
    """configs[4] as the sharding sweep: ONE global batch of 4096 series (ctx
    512, N = 4), identical on every rank; each rank takes its shard of whole
    groups (sharding.partition_groups), runs the forward on it and the (B, 21,
    64) forecasts are all-gathered over NCCL back into the global order inside
    every timed step (sharding.gather_forecasts).  Total work is fixed, so
    this is strong scaling; time = max over ranks of the CUDA-event total.
    grouped: the same series as 512 groups of 8 (group attention inside each
    group; groups never split across ranks)."""
    import torch.distributed as dist

    from cutechronos_b200.sharding import gather_forecasts, partition_groups
    from cutechronos_b200.workloads import config4

    rank, world, _ = dist_env()
    w = config4()
    B = w.context.shape[0]
    gid = torch.arange(B) // 8 if grouped else None
    shards = partition_groups(gid, B, world)
    mine = shards[rank]
    ctx = w.context[mine].to(dev)
    gid_local = gid[mine] if gid is not None else None
    N = w.num_output_patches

    def step():
        y = model_bf16(ctx, num_output_patches=N, group_ids=gid_local)
        return gather_forecasts(y, shards) if world > 1 else y

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(steps):
        flush.fill_(i & 0xFF)
        evs[i][0].record()
        y = step()
        evs[i][1].record()
    torch.cuda.synchronize()
    t = torch.tensor([sum(a.elapsed_time(b) for a, b in evs)], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item()) / steps
    assert y.shape[0] == B
    return {"forecasts_per_s": B / (ms / 1e3), "ms_per_step": ms, "series_per_rank": int(mine.numel()),
            "groups": "512 x 8" if grouped else "4096 x 1", "collective": "NCCL all_gather of the padded "
            "(B_r, 21, 64) bf16 shards" if world > 1 else "none (one GPU)"}


def pipeline_rates(model_bf16, dev, steps=3, warmup=1):
    """The user-facing pipeline on configs[1] inputs, host to host, wall clock
    around synchronised calls: predict_quantiles on a list of 256 CPU series
    (default levels) and predict_df on the same series as a long DataFrame."""
    import pandas as pd

    from cutechronos_b200.pipeline import CuteChronos2Pipeline
    from cutechronos_b200.workloads import series_cfg1

    pipe = CuteChronos2Pipeline(model_bf16, device=str(dev))
    x = series_cfg1(256, 2048, 1)
    series = list(x.unbind(0))
    n, L = x.shape
    df = pd.DataFrame({"item_id": np.repeat(np.arange(n), L), "timestamp": np.tile(np.arange(L), n),
                       "target": x.reshape(-1).numpy()})

    def rate(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(steps):
            fn()
        torch.cuda.synchronize()
        return n * steps / (time.perf_counter() - t0)

    return {
        "predict_quantiles_list_forecasts_per_s": rate(
            lambda: pipe.predict_quantiles(series, prediction_length=64)),
        "predict_df_forecasts_per_s": rate(
            lambda: pipe.predict_df(df, prediction_length=64, quantile_levels=[0.1, 0.5, 0.9])),
    }


def memory_bound_streaming(dev, reps=10):
    """The memory-bound kernels on streaming cases (inputs and outputs well
    above the 126 MB L2), CUDA events, median of `reps` launches: algorithmic
    bytes per launch / duration, against the measured HBM copy bandwidth."""
    from cutechronos_b200 import kernels as kk
    hbm = measured_peaks()[0]
    g = torch.Generator(device=dev).manual_seed(5)
    Bp, Lp, P = 65536, 2048, 128
    ctx = torch.randn(Bp, Lp, generator=g, device=dev)
    pred = torch.randn(Bp, 4, 336, generator=g, device=dev).to(torch.bfloat16)
    loc, sc = torch.zeros(Bp, device=dev), torch.ones(Bp, device=dev)
    rows = torch.randn(136192, 768, generator=g, device=dev).to(torch.bfloat16)
    wln = torch.ones(768, device=dev, dtype=torch.bfloat16)
    cases = {
        "preprocess_65536x2048": (lambda: kk.fused_preprocess(ctx, 16, 8192, True, dtype=torch.bfloat16),
                                  Bp * (4 * Lp + 2 * 48 * P + P + 4 * P + 8)),
        "output_transform_65536x4": (lambda: kk.fused_output_transform(pred, loc, sc, 21, 16, True),
                                     2 * 2 * Bp * 4 * 336 + 8 * Bp),
        "rmsnorm_136192x768": (lambda: kk.rms_layernorm(rows, wln), 2 * 2 * 136192 * 768),
    }
    out = {}
    for name, (fn, nbytes) in cases.items():
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
        for a, b in evs:
            a.record()
            fn()
            b.record()
        torch.cuda.synchronize()
        ms = statistics.median(a.elapsed_time(b) for a, b in evs)
        gbs = nbytes / (ms / 1e3) / 1e9
        out[name] = {"us": round(ms * 1e3, 1), "gbs": round(gbs, 1), "frac_of_measured_hbm": round(gbs / hbm, 3)}
    del ctx, pred, rows
    torch.cuda.empty_cache()
    return out


def e2e_pipelined(step, ctx_host, out_host, flush, steps, dev):
    """End-to-end milliseconds of `steps` forwards with host buffers, the way a
    serving loop runs them: the context of step i+1 goes host -> device and the
    forecasts of step i-1 device -> host on a copy stream while step i
    computes.  Every copy starts inside a timed interval (the copy stream waits
    for the interval's start event); the L2 flush between steps stays outside,
    as in the device-timed loop.  Returns the sum of the intervals."""
    main = torch.cuda.current_stream(dev)
    copy = torch.cuda.Stream(dev)
    xbuf = [torch.empty(ctx_host.shape, dtype=ctx_host.dtype, device=dev) for _ in range(2)]
    h2d = [torch.cuda.Event() for _ in range(2)]
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    ys = [None] * steps
    for i in range(steps):
        flush.fill_(i & 0xFF)
        ev[i][0].record(main)
        with torch.cuda.stream(copy):
            copy.wait_event(ev[i][0])  # also orders after step i-1's forward (same stream, earlier)
            if i >= 1:
                ys[i - 1].record_stream(copy)
                out_host.copy_(ys[i - 1], non_blocking=True)
                ys[i - 1] = None
            for j in ((0, 1) if i == 0 else (i + 1,)):
                if j < steps:  # buffer j % 2 was last read by step j - 2, finished before this interval
                    xbuf[j % 2].copy_(ctx_host, non_blocking=True)
                    h2d[j % 2].record(copy)
        main.wait_event(h2d[i % 2])
        ys[i] = step(xbuf[i % 2])
        if i == steps - 1:  # the last forecasts are read back inside the last interval
            with torch.cuda.stream(copy):
                copy.wait_stream(main)
                ys[i].record_stream(copy)
                out_host.copy_(ys[i], non_blocking=True)
            main.wait_stream(copy)
        ev[i][1].record(main)
    torch.cuda.synchronize()
    return sum(a.elapsed_time(b) for a, b in ev)


def run_b200(args):
    import torch.distributed as dist

    from cutechronos_b200 import _native as nat
    from cutechronos_b200.model import CuteChronos2Config, CuteChronos2Model
    from cutechronos_b200.workloads import seeded_init_, series_cfg1
    from oracle.chronos2_oracle import forecast_flops

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    B, L, N = args.batch, 2048, 4
    P = L // 16
    S = P + 1 + N
    gflop = forecast_flops(S, P, N) / 1e9

    model = seeded_init_(CuteChronos2Model(CuteChronos2Config()), seed=0).to(dev, torch.bfloat16).eval()
    ctx_host = series_cfg1(B, L, 1 + rank).pin_memory()
    ctx = ctx_host.to(dev)
    out_host = torch.empty(B, 21, N * 16, dtype=torch.bfloat16).pin_memory()
    gathered = torch.empty(world * B, 21, N * 16, dtype=torch.bfloat16, device=dev) if world > 1 else None
    flush = torch.empty(256 * 2**20, dtype=torch.uint8, device=dev)
    lib = nat.load()

    def step(x):
        y = model(x, num_output_patches=N)
        if world > 1:
            dist.all_gather_into_tensor(gathered, y)
        return y

    with torch.inference_mode():
        for _ in range(args.warmup):
            step(ctx)
        torch.cuda.synchronize()
        # ---- device-timed region: inputs resident in HBM --------------------
        cap = 256 * args.steps
        clocks = ClockSampler(local)
        clocks.start()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for i in range(args.steps):
            flush.fill_(i & 0xFF)
            evs[i][0].record()
            step(ctx)
            evs[i][1].record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        clocks.stop()
        step_ms = [a.elapsed_time(b) for a, b in evs]
        # the same steps once more with a CUDA-event pair around every launch
        # (per-kernel durations for the roofline and the kernel shares); kept out
        # of the timed region above, whose launches run back to back
        nat.check(lib.cc2_profile_begin(cap), "cc2_profile_begin")
        for i in range(args.steps):
            flush.fill_(i & 0xFF)
            step(ctx)
        torch.cuda.synchronize()
        kinds = (C.c_int * cap)()
        ms = (C.c_float * cap)()
        fl = (C.c_double * cap)()
        by = (C.c_double * cap)()
        cnt = C.c_int()
        nat.check(lib.cc2_profile_read(kinds, ms, fl, by, cap, C.byref(cnt)), "cc2_profile_read")
        total_ms = sum(step_ms)
        t = torch.tensor([total_ms], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
        value = world * B * args.steps / (total_ms / 1e3)

        # ---- end to end through the public API with host buffers --------------
        if world > 1:
            dist.barrier()
        e2e_ms = e2e_pipelined(step, ctx_host, out_host, flush, args.steps, dev)
        t = torch.tensor([e2e_ms], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_value = world * B * args.steps / (float(t.item()) / 1e3)

        # ---- the same two measurements with CUDA-graph replay (compile_mode) ------
        model.enable_cuda_graphs(True)
        try:
            for _ in range(2):
                step(ctx)
            torch.cuda.synchronize()
            gev = []
            for i in range(args.steps):
                flush.fill_(i & 0xFF)
                a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                step(ctx)
                b_.record()
                gev.append((a, b_))
            torch.cuda.synchronize()
            g_e2e_ms = e2e_pipelined(step, ctx_host, out_host, flush, args.steps, dev)
            t = torch.tensor([sum(a.elapsed_time(b_) for a, b_ in gev), g_e2e_ms], device=dev)
            if world > 1:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            graph_mode = {"forecasts_per_s": world * B * args.steps / (float(t[0]) / 1e3),
                          "e2e_forecasts_per_s": world * B * args.steps / (float(t[1]) / 1e3),
                          "path": "CuteChronos2Model.enable_cuda_graphs (compile_mode): one graph replay per step"}
        finally:
            model.enable_cuda_graphs(False)

        # ---- p50 batch-1 latency (CUDA graph of one B=1 forward) ---------------
        lat_p50 = lat_p50_512 = None
        if rank == 0 and not args.no_latency:
            lat_p50 = graph_latency_ms(model, ctx[:1].clone(), N)
            # the reference's published batch-1 configuration: context 512 (README: B=1, L=512)
            lat_p50_512 = graph_latency_ms(model, series_cfg1(1, 512, 7).to(dev), N)
        # ---- configs[4] sharding sweep: one global batch partitioned over the ranks
        sharded = None
        if not args.no_configs:
            sharded = {"univariate": cfg4_sharded(model, dev, flush, max(3, args.steps // 2), 2),
                       "grouped": cfg4_sharded(model, dev, flush, max(3, args.steps // 2), 2, grouped=True),
                       "scaling": "strong (4096 series in total, split over the ranks)"}
        other = pipe_rates = mem_bound = None
        if rank == 0 and not args.no_configs:
            other = other_configs(model, dev, flush)
            pipe_rates = pipeline_rates(model, dev)
            mem_bound = memory_bound_streaming(dev)

    # ---- roofline of the dominant kernel (tcgen05 GEMM), live from the timed region
    n = cnt.value
    agg = {}
    for i in range(min(n, cap)):
        k = nat.KIND_NAMES.get(kinds[i], str(kinds[i]))
        a = agg.setdefault(k, {"launches": 0, "ms": 0.0, "flops": 0.0, "bytes": 0.0})
        a["launches"] += 1
        a["ms"] += ms[i]
        a["flops"] += fl[i]
        a["bytes"] += by[i]
    hbm, tf_burst, tf_sus, peak_src = measured_peaks()
    gemm_names = [nat.KIND_NAMES[k] for k in nat.GEMM_KINDS]
    gemm = {"launches": 0, "ms": 0.0, "flops": 0.0}
    for k in gemm_names:
        for f in gemm:
            gemm[f] += agg.get(k, {}).get(f, 0)
    gemm["ms"] = max(gemm["ms"], 1e-9)
    achieved_tf = gemm["flops"] / (gemm["ms"] / 1e3) / 1e12
    # per role (the GEMMs run inside ~7 ms steps of back-to-back kernels: the
    # burst peak is the one that applies)
    gemm_roles = {k: {"launches_per_step": v["launches"] / args.steps, "us_per_launch": 1e3 * v["ms"] / v["launches"],
                      "tflops": v["flops"] / (v["ms"] / 1e3) / 1e12,
                      "frac": v["flops"] / (v["ms"] / 1e3) / 1e12 / tf_burst}
                  for k, v in agg.items() if k in gemm_names and v["launches"]}
    pre = agg.get("preprocess")
    result = None
    if rank == 0:
        cpu_v, cpu_threads = None, 0
        # the CPU baseline runs at N = 1 only (under torchrun the other ranks'
        # processes share the host cores)
        if not args.no_cpu and world == 1:
            ref = CpuReference()
            ref.forecasts_per_s(1, L, N)
            cpu_v, cpu_threads = ref.forecasts_per_s(32, L, N), ref.threads
        clk = clocks.summary()
        roofline = {
            "bound": "tensor", "kernel": "gemm_pair_kernel / gemm_tc_kernel (tcgen05, all GEMM launches of the step)",
            "achieved": achieved_tf, "peak": tf_burst, "unit": "TFLOP/s", "frac": achieved_tf / tf_burst,
            "peak_source": f"{peak_src} bf16_tflops (burst: each GEMM launch lasts 5-200 us inside a ~7 ms step)",
            "flops_counted": "executed 2*M*N*K of every GEMM launch (the g=1 group block is one folded GEMM)",
            "by_role": gemm_roles,
            "traffic": gemm_traffic_per_launch(),
            "traffic_source": "profiles/gemm_dram_cfg1.txt (ncu dram__bytes_read+write, per GEMM launch of one forward)",
            "launches_per_step": gemm["launches"] / args.steps,
            "avg_launch_us": 1e3 * gemm["ms"] / max(1, gemm["launches"]),
        }
        kernels = {k: {"launches": v["launches"], "ms_total": round(v["ms"], 4),
                       "share": round(v["ms"] / sum(x["ms"] for x in agg.values()), 4)} for k, v in agg.items()}
        if pre:
            kernels["preprocess"]["hbm_gbs"] = pre["bytes"] / (pre["ms"] / 1e3) / 1e9
        result = {
            "metric": METRIC, "value": value, "unit": UNIT,
            "value_is": "whole job: forecasts/s summed over all ranks (per GPU = value / n_gpus)",
            "value_per_gpu": value / world, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (configs[1] generator; random-init weights seed 0)",
            "config": {"workload": "configs[1]: Chronos-2-base encoder forward, B=256 univariate series per GPU, "
                                   "ctx 2048 (128 patches), pred 64 (4 patches), S=133 tokens",
                       "global_batch": world * B, "seq_len": S, "parallelism": f"series sharding x{world}",
                       "l2": "flushed (256 MB write) before every timed step"},
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": B * L * 4,
                    "d2h_bytes_per_step": B * 21 * N * 16 * 2,
                    "path": "CuteChronos2Model.forward on pinned host input, D2H of the (B,21,64) bf16 forecasts; "
                            "copies on a second stream overlap the neighbouring steps' forwards"},
            "gpu_launches": n,
            "roofline": roofline,
            "model_flops_frac": value / world * gflop * 1e9 / (tf_burst * 1e12),
            "gflop_per_forecast": gflop,
            "latency_b1_p50_ms": lat_p50,
            "latency_b1_ctx512_p50_ms": lat_p50_512,
            "latency_path": "bf16, one series, N = 4: a CUDA graph of one CuteChronos2Model.forward (input "
                            "resident), p50 over 50 single replays timed with CUDA events",
            "graph_mode": graph_mode,
            "cfg4_sharded": sharded,
            "other_configs": other,
            "pipeline": pipe_rates,
            "kernels": kernels,
            "memory_bound_streaming": mem_bound,
            "clocks": clk,
            "cpu_baseline": {"value": cpu_v, "unit": UNIT, "cores": cpu_threads,
                             "kind": ref.kind if cpu_v is not None else None,
                             "sample": (f"32 series of configs[1] (ctx 2048, N=4), {ref.what}, one forward")
                             if cpu_v is not None else
                             "not measured at N > 1 (taken on rank 0 of the N = 1 run)"},
        }
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


def run_micro(args):
    """Per-kernel micro-benchmark at the configs[1] shapes (M = B * 133 token
    rows): each GEMM of the forward with its fused epilogue and the time
    attention, timed with CUDA events; cuBLAS on the same GEMM shapes is timed
    beside them as a yardstick (it is not used by the engine)."""
    from cutechronos_b200 import _native as nat
    from cutechronos_b200 import kernels as kk

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    M, d, dff = args.batch * 133, 768, 3072
    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, generator=g, device=dev) * scale).to(torch.bfloat16)

    x, h = rnd(M, d), rnd(M, dff)
    wqkv, wo, wi, wf = rnd(3 * d, d, scale=0.03), rnd(d, d, scale=0.03), rnd(dff, d, scale=0.03), rnd(d, dff, scale=0.02)
    big = rnd(8192, 8192)
    ssq = kk.row_sumsq_parts(x.float()).to(dev)
    so = torch.empty_like(ssq)
    res = x.clone()
    res2 = x.clone()
    res_lo = torch.zeros(kk.lo_numel(M, d), dtype=torch.bfloat16, device=dev)
    res_lo2 = torch.zeros_like(res_lo)
    qkvr = rnd(M, 3 * d, scale=0.5)
    tok = torch.ones(M, dtype=torch.uint8, device=dev)
    att = torch.empty(M, d, dtype=torch.bfloat16, device=dev)
    lib = nat.load()

    def variant(v, fn):
        def run():
            old = lib.cc2_set_attention_variant(v)
            fn()
            lib.cc2_set_attention_variant(old)
        return run

    def gemm_variant(v, fn):
        def run():
            old = lib.cc2_set_gemm_variant(v)
            fn()
            lib.cc2_set_gemm_variant(old)
        return run

    # batch-1 serving shapes (one series, context 2048: 133 token rows)
    x1, h1 = x[:133].contiguous(), h[:133].contiguous()
    res1 = x1.clone()

    B4 = 4096
    qkv4 = rnd(B4 * 37, 3 * d, scale=0.5)
    tok4 = torch.ones(B4 * 37, dtype=torch.uint8, device=dev)
    att4 = torch.empty(B4 * 37, d, dtype=torch.bfloat16, device=dev)
    # memory-bound kernels at a streaming size (HBM-bound; the forward's own
    # launches are a few MB and launch/latency-bound)
    Bp, Lp = 65536, 2048  # the survey's streaming size: inputs and outputs well above the 126 MB L2
    Pp = Lp // 16
    ctxp = torch.randn(Bp, Lp, generator=g, device=dev)
    predp = rnd(Bp, 4, 336)
    locp, scp = torch.zeros(Bp, device=dev), torch.ones(Bp, device=dev)
    predc = torch.empty_like(predp)
    wln = rnd(d)
    x4 = rnd(4 * M, d)
    # group attention as configs[2] runs it: 64 groups x 8 series, S = 133, layout prepared once
    Bg, Sg = 512, 133
    qkvg = rnd(Bg * Sg, 3 * d, scale=0.5)
    tokg = torch.ones(Bg * Sg, dtype=torch.uint8, device=dev)
    attg = torch.empty(Bg * Sg, d, dtype=torch.bfloat16, device=dev)
    gid = torch.arange(Bg) // 8
    mem_h, off_h = (C.c_int32 * Bg)(), (C.c_int32 * (Bg + 1))()
    ngr, mgr = C.c_int(), C.c_int()
    nat.check(lib.cc2_group_layout(gid.data_ptr(), Bg, mem_h, off_h, C.byref(ngr), C.byref(mgr)), "cc2_group_layout")
    mem_d = torch.tensor(list(mem_h), dtype=torch.int32, device=dev)
    off_d = torch.tensor(list(off_h)[: ngr.value + 1], dtype=torch.int32, device=dev)

    def group_attn():
        nat.check(lib.cc2_attention(nat.CC2_BF16, 1, qkvg.data_ptr(), 3 * d, 0, d, 2 * d, attg.data_ptr(), d,
                                    tokg.data_ptr(), Sg * ngr.value, Sg, 12, 64, mem_d.data_ptr(), off_d.data_ptr(),
                                    ngr.value, mgr.value, None, torch.cuda.current_stream().cuda_stream),
                  "cc2_attention")

    # TurboQuant K/V hook on one layer's QKV rows: K prod 4 bits, V mse 4 bits, Hadamard
    from cutechronos_b200 import turboquant as tqm
    kq_p = tqm.TurboQuantParams.build(64, 4, mode="prod", seed=11, device=dev)
    vq_p = tqm.TurboQuantParams.build(64, 4, mode="mse", seed=12, device=dev)
    qkv_tq = rnd(M, 3 * d, scale=0.5)

    # batch-1 forward (bf16, N = 4) replayed from a CUDA graph, built on first use
    b1 = {}

    def b1_forward(L):
        def run():
            if L not in b1:
                from cutechronos_b200.model import CuteChronos2Config, CuteChronos2Model
                from cutechronos_b200.workloads import seeded_init_, series_cfg1
                if "model" not in b1:
                    b1["model"] = seeded_init_(CuteChronos2Model(CuteChronos2Config()), seed=0).to(
                        dev, torch.bfloat16).eval()
                m, xb = b1["model"], series_cfg1(1, L, 7).to(dev)
                m(xb, num_output_patches=4)
                torch.cuda.synchronize()
                gr, st = torch.cuda.CUDAGraph(), torch.cuda.Stream()
                st.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(st):
                    m(xb, num_output_patches=4)
                    with torch.cuda.graph(gr, stream=st):
                        m(xb, num_output_patches=4)
                torch.cuda.synchronize()
                b1[L] = gr
            b1[L].replay()
        return run

    cases = {
        "kv_quant prod4/mse4 M=34048": (
            lambda: tqm.kv_quant(qkv_tq, M, 12, kq_p, vq_p, q_col=0, k_col=d, v_col=2 * d), 0, M * 2 * d * 2 * 2),
        "group attn 64x8 S=133 bf16": (group_attn, 0, Bg * Sg * d * 2 * 4),
        "group attn 64x8 S=133 bf16 (tcgen05)": (
            lambda: kk.group_attention_contig(qkvg.view(Bg, Sg, 3 * d), tokg.view(Bg, Sg), 8, 12), 0,
            Bg * Sg * d * 2 * 4),
        "preprocess B=65536 L=2048 bf16": (
            lambda: kk.fused_preprocess(ctxp, 16, 8192, True, dtype=torch.bfloat16), 0,
            Bp * (4 * Lp + 2 * 48 * Pp + Pp + 4 * Pp + 8)),
        "output transform B=65536 N=4 bf16": (
            lambda: kk.fused_output_transform(predp, locp, scp, 21, 16, True), 0, 2 * 2 * Bp * 4 * 336 + 8 * Bp),
        # yardsticks for the output transform: the same bytes copied by torch, and the
        # transform without the sinh (rearrange and unscale only)
        "output transform B=65536 N=4 bf16 (no sinh)": (
            lambda: kk.fused_output_transform(predp, locp, scp, 21, 16, False), 0, 2 * 2 * Bp * 4 * 336 + 8 * Bp),
        "output transform B=65536 N=4 bf16 (torch copy of the bytes)": (
            lambda: predc.copy_(predp), 0, 2 * 2 * Bp * 4 * 336),
        "rmsnorm M=34048 d=768 bf16": (lambda: kk.rms_layernorm(x, wln), 0, 2 * 2 * M * d),
        "rmsnorm M=136192 d=768 bf16": (lambda: kk.rms_layernorm(x4, wln), 0, 2 * 2 * 4 * M * d),
        "qkv  N=2304 K=768 rowscale": (lambda: kk.linear(x, wqkv, row_ssq=ssq, norm_dim=d), 2 * M * 3 * d * d),
        "o    N=768  K=768 resid+ssq": (lambda: kk.linear(x, wo, residual=res, ssq_out=so, out=res), 2 * M * d * d),
        "ffn1 N=3072 K=768 rowscale+relu": (lambda: kk.linear(x, wi, row_ssq=ssq, norm_dim=d, relu=True),
                                            2 * M * dff * d),
        "ffn2 N=768  K=3072 resid+ssq": (lambda: kk.linear(h, wf, residual=res, ssq_out=so, out=res), 2 * M * d * dff),
        "o    N=768  K=768 resid+ssq+lo": (
            lambda: kk.linear(x, wo, residual=res, residual_lo=res_lo, lo_out=res_lo, ssq_out=so, out=res),
            2 * M * d * d),
        "fold N=768  K=768 rowscale+resid+ssq+lo": (
            lambda: kk.linear(x, wo, row_ssq=ssq, norm_dim=d, residual=res, residual_lo=res_lo, lo_out=res_lo2,
                              ssq_out=so, out=res2), 2 * M * d * d),
        "ffn2 N=768  K=3072 resid+ssq+lo": (
            lambda: kk.linear(h, wf, residual=res, residual_lo=res_lo, lo_out=res_lo, ssq_out=so, out=res),
            2 * M * d * dff),
        "gemm 8192^3 plain": (lambda: kk.linear(big, big), 2 * 8192 ** 3),
        # batch-1 serving latency (graph replay; the "TFLOP/s" column is the forward's FLOPs / latency)
        "b1 forward ctx512 (graph)": (b1_forward(512), 8.644e9),
        "b1 forward ctx2048 (graph)": (b1_forward(2048), 31.481e9),
        # batch-1 FFN down (133 token rows): the micro time of one call is host-bound
        # (tensor maps built per call); the device time comes from ncu
        "b1 ffn2 M=133 N=768 K=3072 (128x64 tiles)": (
            lambda: kk.linear(h1, wf, residual=res1, out=res1), 2 * 133 * d * dff, d * dff * 2),
        "b1 ffn2 M=133 N=768 K=3072 (2-SM tiles)": (
            gemm_variant(2, lambda: kk.linear(h1, wf, residual=res1, out=res1)), 2 * 133 * d * dff, d * dff * 2),
        "attn time S=133 (rope)": (lambda: kk.attention_rows(qkvr, tok, args.batch, 133, 12, True, att),
                                   4 * args.batch * 12 * 133 * 133 * 64),
        "attn time S=133 (no rope)": (lambda: kk.attention_rows(qkvr, tok, args.batch, 133, 12, False, att),
                                      4 * args.batch * 12 * 133 * 133 * 64),
        "attn time S=133 (no rope, mma.sync)": (
            variant(1, lambda: kk.attention_rows(qkvr, tok, args.batch, 133, 12, False, att)),
            4 * args.batch * 12 * 133 * 133 * 64),
        "attn time S=37 B=4096": (lambda: kk.attention_rows(qkv4, tok4, B4, 37, 12, False, att4),
                                  4 * B4 * 12 * 37 * 37 * 64),
        "attn time S=37 B=4096 (one set per tcgen05 tile)": (
            variant(2, lambda: kk.attention_rows(qkv4, tok4, B4, 37, 12, False, att4)), 4 * B4 * 12 * 37 * 37 * 64),
        "attn time S=37 B=4096 (mma.sync)": (
            variant(1, lambda: kk.attention_rows(qkv4, tok4, B4, 37, 12, False, att4)), 4 * B4 * 12 * 37 * 37 * 64),
        "attn time S=521 B=32": (lambda: kk.attention_rows(qkvr, tok, 32, 521, 12, False, att),
                                 4 * 32 * 12 * 521 * 521 * 64),
        "attn time S=521 B=32 (mma.sync)": (
            variant(1, lambda: kk.attention_rows(qkvr, tok, 32, 521, 12, False, att)), 4 * 32 * 12 * 521 * 521 * 64),
        "cublas qkv  N=2304 K=768": (lambda: torch.matmul(x, wqkv.T), 2 * M * 3 * d * d),
        "cublas o    N=768  K=768": (lambda: torch.matmul(x, wo.T), 2 * M * d * d),
        "cublas ffn1 N=3072 K=768": (lambda: torch.matmul(x, wi.T), 2 * M * dff * d),
        "cublas ffn2 N=768  K=3072": (lambda: torch.matmul(h, wf.T), 2 * M * d * dff),
        "cublas 8192^3": (lambda: torch.matmul(big, big), 2 * 8192 ** 3),
    }
    out = {}
    hbm, *_ = measured_peaks()
    trace_buf = torch.zeros(32 * 8, dtype=torch.int64, device=dev) if args.gemm_trace else None
    for name, spec in cases.items():
        fn, flops = spec[0], spec[1]
        nbytes = spec[2] if len(spec) > 2 else 0
        if args.only and args.only not in name:
            continue
        if trace_buf is not None:
            # per-tile event stamps of the 2-SM GEMM's CTA pair 0 (cc2_set_gemm_trace), one
            # traced launch after a warm-up: tile period (MMA warp's accumulator-free stamps),
            # epilogue span (accumulator full -> epilogue done, warp 2), MMA waits on loads
            fn()
            torch.cuda.synchronize()
            trace_buf.zero_()
            nat.check(lib.cc2_set_gemm_trace(trace_buf.data_ptr()), "cc2_set_gemm_trace")
            fn()
            torch.cuda.synchronize()
            nat.check(lib.cc2_set_gemm_trace(None), "cc2_set_gemm_trace")
            t = trace_buf.view(32, 8).cpu().double()
            n = int((t[:, 0] > 0).sum().item())
            if n >= 3:
                period = (t[2:n, 0] - t[1:n - 1, 0]) / 1e3
                epi = (t[1:n, 4] - t[1:n, 3]) / 1e3
                issue_full = (t[1:n, 3] - t[1:n, 2]) / 1e3  # last k-block issued -> accumulator full
                loadw = t[1:n, 6] / 1e3
                tr = {"tiles": n, "period_us": round(period.median().item(), 2),
                      "epilogue_us": round(epi.median().item(), 2),
                      "issue_to_full_us": round(issue_full.median().item(), 2),
                      "mma_load_wait_us": round(loadw.median().item(), 2),
                      # pair 0: first accumulator-free stamp -> last epilogue done, and the
                      # first tile's wait for its first loaded stage
                      "span_us": round((t[n - 1, 4] - t[0, 0]).item() / 1e3, 2),
                      "first_load_us": round((t[0, 1] - t[0, 0]).item() / 1e3, 2)}
                out[name + " [trace]"] = tr
                log(f"{name:36s} trace: {tr}")
        # warm up for at least 30 ms of GPU time so that the SM clock has ramped up
        t_end = time.perf_counter() + 0.03
        n_warm = 0
        while n_warm < 3 or time.perf_counter() < t_end:
            fn()
            n_warm += 1
            if n_warm % 16 == 0:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for a, b in evs:
            a.record()
            fn()
            b.record()
        torch.cuda.synchronize()
        ms = statistics.median(a.elapsed_time(b) for a, b in evs)
        if nbytes:
            gbs = nbytes / (ms / 1e3) / 1e9
            out[name] = {"us": round(ms * 1e3, 2), "gbs": round(gbs, 1), "hbm_frac": round(gbs / hbm, 3)}
            log(f"{name:36s} {ms * 1e3:9.1f} us  {gbs:7.1f} GB/s ({gbs / hbm:.2f} of measured HBM)")
            continue
        out[name] = {"us": round(ms * 1e3, 2), "tflops": round(flops / (ms / 1e3) / 1e12, 1)}
        log(f"{name:36s} {ms * 1e3:9.1f} us  {flops / (ms / 1e3) / 1e12:7.1f} TFLOP/s")
    print(json.dumps({"micro": out, "M": M}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-latency", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the configs[0,2,3,4] measurements")
    ap.add_argument("--micro", action="store_true", help="per-kernel micro-benchmark instead of the step")
    ap.add_argument("--only", default="", help="with --micro: run only cases whose name contains this")
    ap.add_argument("--gemm-trace", action="store_true",
                    help="with --micro: per-tile event trace of the 2-SM GEMM's CTA pair 0 for each case")
    ap.add_argument("--gemm-variant", type=int, default=0, help="0: 2-SM GEMM tiles, 1: 1-SM tiles only, 3: mainloop only (no output)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.gemm_variant:
        from cutechronos_b200 import _native as nat
        nat.load().cc2_set_gemm_variant(args.gemm_variant)
    if args.micro:
        run_micro(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
