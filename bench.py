"""Benchmark of the dequant-GEMM hot path on B200.

Workload: the sharded 28672x8192 int4 symmetric g128 layer (W ~ N(0, 0.015),
x ~ N(0, 1), seeded synthetic data; weight-quantizer_b200/workloads.py), at
batch 4096 by default. One step = the layer applied to one batch: each rank
runs the dequant-GEMM on its row shard, and for N > 1 the kernel's epilogue
stores its rows into the full y [B, M] of every rank over NVLink peer memory
(one-element NCCL all-reduces before and after order the ranks).

Metric: GFLOP/s = 2*B*M*K / t (the reference's convention,
src/ptqkit/measure.py:167, dequantization not counted), whole job, t = max over
ranks of the CUDA-event time of K steps. Also reported: the same layer at the
decode batches 1, 32 and 256 (weight-stream GB/s and GFLOP/s), the end-to-end
number through the public API with host buffers, the dominant kernel's
roofline, the layer saved in ptqkit's compressed format and loaded back
(``loader``), and the reference CPU kernel timed on this host.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

For N > 1 launch with torchrun (one process per GPU).
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from typing import Any

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

M_ROWS, K_COLS, GROUP = 28672, 8192, 128
E2E_CHUNKS = 8
WORKLOAD = "sharded_28672x8192_int4_g128"
METRIC = "dequant-GEMM weight-stream GB/s & GFLOP/s vs B200 roofline, batch 1–4096"


def _peaks() -> dict[str, Any]:
    path = os.path.join(HERE, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc: subprocess.Popen[str] | None = None
        self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def __enter__(self) -> ClockSampler:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.out, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc: object) -> None:
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict[str, Any]:
        self.out.flush()
        self.out.seek(0)
        rows = [ln.split(",") for ln in self.out.read().strip().splitlines() if ln.strip()]
        os.unlink(self.out.name)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
                for name, val in zip(names, r[5:9]):
                    if val.strip().lower() == "active":
                        reasons.add(name)
            except (ValueError, IndexError):
                continue
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        loaded = [s for s in sm if s > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def reference_arm(args: argparse.Namespace) -> None:
    """The reference's own CPU kernel on this host's cores (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np

    import oracle

    wl = importlib.import_module("weight-quantizer_b200.workloads")
    kern = oracle.reference_kernels()
    kind = "reference" if kern is not None else "port"
    layer = wl.sharded_28672x8192(batches=(args.batch,))[0]
    r = oracle.quantize_stored(layer.weight.numpy(), 4, True, GROUP)
    sample = min(args.cpu_sample_rows, args.batch)
    x = np.ascontiguousarray(layer.x[args.batch][:sample].numpy())
    threads = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(threads)

    def call() -> None:
        if kern is not None:
            kern.dequant_gemm(x, r["q"], r["scales"], r["zeros"], None, GROUP, 4, threads)
        else:
            oracle.dequant_gemm(x, r["q"], r["scales"], r["zeros"], None, GROUP, 4, threads)

    for _ in range(args.warmup):
        call()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        call()
        times.append(time.perf_counter() - t0)
    t = sum(times) / len(times)
    gflops = 2.0 * sample * M_ROWS * K_COLS / t / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gflops, 3), "unit": "GFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded)",
        "config": {"workload": WORKLOAD, "M": M_ROWS, "K": K_COLS, "batch": args.batch, "bits": 4,
                   "group_size": GROUP, "symmetric": True},
        "cpu_baseline": {"value": round(gflops, 3), "unit": "GFLOP/s", "cores": threads, "kind": kind,
                         "sample": f"{sample} of the {args.batch} batch rows per step, full layer, "
                                   f"{'oracle/_ref (ptqkit _kernels.dequant_gemm)' if kern else 'C oracle'}"},
        "e2e": {"value": round(gflops, 3), "unit": "GFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline_sample(q: Any, scales: Any, zeros: Any, x: Any, seconds: float) -> dict[str, Any]:
    import numpy as np

    import oracle

    kern = oracle.reference_kernels()
    threads = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(threads)
    x = np.ascontiguousarray(x)

    def call() -> None:
        if kern is not None:
            kern.dequant_gemm(x, q, scales, zeros, None, GROUP, 4, threads)
        else:
            oracle.dequant_gemm(x, q, scales, zeros, None, GROUP, 4, threads)

    call()
    times = []
    t_end = time.perf_counter() + seconds
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        call()
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": round(2.0 * x.shape[0] * M_ROWS * K_COLS / t / 1e9, 3), "unit": "GFLOP/s",
            "cores": threads, "kind": "reference" if kern is not None else "port",
            "sample": f"batch {x.shape[0]} x full {M_ROWS}x{K_COLS} layer, median of {len(times)} calls "
                      f"({'ptqkit _kernels.dequant_gemm built in oracle/_ref' if kern else 'C oracle'})"}


def loader_line(wq: Any, qw: Any, dev: Any, stream: Any, peaks: dict[str, Any]) -> dict[str, Any]:
    """The layer (with an fp32 bias) saved in ptqkit's compressed format and
    loaded back through load_compressed_layers, three times, wall clock with
    the device synchronized (the file is in the page cache); plus the widening
    kernel alone on 64 Mi fp16 values, timed with CUDA events."""
    import torch

    bias = torch.randn(qw.out_features, generator=torch.Generator().manual_seed(5)).to(dev)
    layer = wq.QuantizedLinear(qw, bias, impl="kernel")
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "layer.pt")
        t0 = time.perf_counter()
        size = wq.save_compressed(layer, path)
        t_save = time.perf_counter() - t0
        times = []
        for _ in range(3):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            loaded = wq.load_compressed_layers(path, device=dev)[""]
            torch.cuda.synchronize()
            times.append(time.perf_counter() - t0)
        same = bool(torch.equal(loaded.codes, layer.codes)
                    and torch.equal(loaded.scales, layer.scales.half().float()))
    payload = int(layer.codes.nbytes + 2 * (layer.scales.numel() + layer.zeros.numel()) + 4 * bias.numel())
    t_load = sorted(times)[1]
    n = 64 * 1024 * 1024
    src = torch.randn(n, device=dev).half()
    dst = torch.empty(n, dtype=torch.float32, device=dev)
    ev = []
    for i in range(8):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        wq._kernels.widen_f16_f32(src, dst)
        e1.record(stream)
        if i >= 3:
            ev.append((e0, e1))
    torch.cuda.synchronize()
    t_w = sum(a.elapsed_time(b) for a, b in ev) / len(ev) / 1e3
    widen_gbs = 6.0 * n / t_w / 1e9
    return {"layer": "28672x8192 int4 g128 + fp32 bias", "file_bytes": size, "payload_bytes": payload,
            "save_ms": round(t_save * 1e3, 1), "load_ms": round(t_load * 1e3, 2),
            "load_gbs": round(payload / t_load / 1e9, 2), "loaded_equals_rounded": same,
            "widen": {"values": n, "us": round(t_w * 1e6, 1), "gbs": round(widen_gbs, 1),
                      "frac_hbm": round(widen_gbs / peaks["hbm_gbs"], 4)}}


def _weight_bytes(qw: Any) -> int:
    n = int(qw.codes.nbytes + qw.scales.nbytes + qw.zeros.nbytes)
    return n + (0 if qw.channel_scale is None else int(qw.channel_scale.nbytes))


def config_lines(wq: Any, wl: Any, dev: Any, stream: Any, peaks: dict[str, Any], cpu_seconds: float,
                 reps: int) -> dict[str, Any]:
    """BASELINE's configs 1-4 on one GPU, plus RTN quantize throughput.

    Every timed call starts with L2 holding none of its data (a 256 MB write and
    a 256 MB read of other buffers first), CUDA events around the call alone;
    the median of ``reps`` calls. Beside each line: ptqkit's compiled CPU
    kernel (oracle/_ref) on the same inputs with every host thread."""
    import numpy as np
    import torch

    import oracle

    kern = oracle.reference_kernels()
    threads = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(threads)
    flush_w = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    flush_r = torch.ones(64 * 1024 * 1024, dtype=torch.float32, device=dev)

    def gpu_ms(call: Any) -> float:
        call()
        ts = []
        for i in range(reps):
            flush_w.fill_(float(i))
            flush_r.sum()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            call()
            e1.record(stream)
            ts.append((e0, e1))
        torch.cuda.synchronize()
        return statistics.median(a.elapsed_time(b) for a, b in ts)

    def cpu_ms(call: Any, budget: float) -> float:
        call()
        ts: list[float] = []
        end = time.perf_counter() + budget
        while time.perf_counter() < end or len(ts) < 3:
            t0 = time.perf_counter()
            call()
            ts.append(time.perf_counter() - t0)
        return statistics.median(ts) * 1e3

    def ref_call(qw: Any, x: Any) -> Any:
        q, sc, z = qw.codes.cpu().numpy(), qw.scales.cpu().numpy(), qw.zeros.cpu().numpy()
        ch = None if qw.channel_scale is None else qw.channel_scale.cpu().numpy()
        xn = np.ascontiguousarray(x.numpy())
        if kern is not None:
            return lambda: kern.dequant_gemm(xn, q, sc, z, ch, int(qw.group_size), int(qw.bits), threads)
        return lambda: oracle.dequant_gemm(xn, q, sc, z, ch, int(qw.group_size), int(qw.bits), threads)

    def line(name: str, layers: list[tuple[Any, Any]], batch: int) -> dict[str, Any]:
        xs = [(qw, x.to(dev), torch.empty((x.shape[0], qw.out_features), device=dev)) for qw, x in layers]

        def run() -> None:
            for qw, xd, out in xs:
                wq.dequant_gemm(xd, qw, impl="kernel", out=out)

        # The calls are replayed from a captured CUDA graph, as a serving
        # runtime issues a decode step: the timed region is the GPU's work,
        # not the Python launch overhead of these small layers.
        timing = "CUDA graph replay of the calls, L2 flushed before each replay"
        try:
            run()
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                run()
            ms = gpu_ms(graph.replay)
        except RuntimeError as err:
            timing = f"eager calls (graph capture failed: {str(err)[:80]})"
            ms = gpu_ms(run)
        flops = sum(2.0 * x.shape[0] * qw.out_features * qw.in_features for qw, x in layers)
        wbytes = sum(_weight_bytes(qw) for qw, _ in layers)
        abytes = wbytes + sum(4 * x.shape[0] * (qw.in_features + qw.out_features) for qw, x in layers)
        calls = [ref_call(qw, x) for qw, x in layers]
        cms = cpu_ms(lambda: [c() for c in calls], cpu_seconds)
        return {"config": name, "batch": batch, "layers": len(layers), "ms": round(ms, 4), "timing": timing,
                "gflops": round(flops / ms / 1e6, 1), "weight_gbs": round(wbytes / ms / 1e6, 1),
                "hbm_frac": round(abytes / ms / 1e6 / peaks["hbm_gbs"], 4),
                "cpu_reference": {"ms": round(cms, 3), "gflops": round(flops / cms / 1e6, 2), "cores": threads,
                                  "kind": "reference" if kern is not None else "port"},
                "speedup_vs_cpu": round(cms / ms, 1)}

    out: list[dict[str, Any]] = []
    c1 = wl.gpt2_c_fc_int4_g128()[0]
    out.append(line("1: GPT-2 c_fc 3072x768 int4 sym g128", [(wq.quantize_weight(c1.weight, c1.config), c1.x[8])], 8))
    c2 = wl.gpt2_small_int8_asym()
    qws = [wq.quantize_weight(layer.weight, layer.config) for layer in c2]
    for b in (1, 8):
        out.append(line("2: GPT-2-small 12 blocks (48 linears) int8 asym per-channel, as one sequence",
                        [(qw, layer.x[b]) for qw, layer in zip(qws, c2)], b))
    c3 = wl.awq_11008x4096()[0]
    out.append(line("3: 11008x4096 int4 asym g128 + AWQ channel scale, 1% outlier channels",
                    [(wq.quantize_weight(c3.weight, c3.config, pre_scale=c3.pre_scale), c3.x[16])], 16))
    c4 = wl.oddk_4096x4095_g64()[0]
    qw4 = wq.quantize_weight(c4.weight, c4.config)
    for b in (1, 4, 32):
        out.append(line("4: 4096x4095 int4 sym g64 (odd K)", [(qw4, c4.x[b])], b))

    # RTN quantize + pack of the config-5 and config-3 weights
    rtn = []
    ref_rtn = None
    ref_dir = os.path.join(HERE, "baseline", "_ref")
    if os.path.isdir(os.path.join(ref_dir, "ptqkit")):
        sys.path.insert(0, ref_dir)
        try:
            ref_rtn = importlib.import_module("ptqkit.quant")
        except ImportError:
            ref_rtn = None
    big = wl.sharded_28672x8192(batches=())[0]
    for name, w, cfg, pre in (("5: 28672x8192 int4 sym g128", big.weight, big.config, None),
                              ("3: 11008x4096 int4 asym g128 + AWQ pre-scale", c3.weight, c3.config, c3.pre_scale)):
        wd = w.to(dev)
        pd = None if pre is None else pre.to(dev)
        ms = gpu_ms(lambda: wq.quantize_weight(wd, cfg, pre_scale=pd))
        rows = min(int(w.shape[0]), 2048)
        ws = w[:rows].contiguous()
        if ref_rtn is not None:
            rcfg = ref_rtn.QuantConfig(bits=cfg.bits, symmetric=cfg.symmetric, group_size=cfg.group_size)
            cms = cpu_ms(lambda: ref_rtn.quantize_weight(ws, rcfg, pre_scale=pre), cpu_seconds / 2)
            kind = "reference (ptqkit.quant.quantize_weight, torch CPU)"
        else:
            wn = ws.numpy()
            pn = None if pre is None else pre.numpy()
            cms = cpu_ms(lambda: oracle.quantize_stored(wn, cfg.bits, cfg.symmetric, cfg.group_size, pn), cpu_seconds / 2)
            kind = "port (C oracle)"
        cms_full = cms * int(w.shape[0]) / rows
        read = 4 * w.numel()
        rtn.append({"weight": name, "ms": round(ms, 4), "read_gbs": round(read / ms / 1e6, 1),
                    "hbm_frac": round(read / ms / 1e6 / peaks["hbm_gbs"], 4),
                    "cpu_reference": {"ms_full_weight": round(cms_full, 1), "kind": kind, "cores": threads,
                                      "sample": f"{rows} of {int(w.shape[0])} rows, scaled to the full weight"},
                    "speedup_vs_cpu": round(cms_full / ms, 1),
                    "timed": "GPU RTN + pack and the host read of its status flags"})
        del wd
    # GPTQ on a 4096 x 4096 int4 g128 layer (Hessian of 8192 calibration rows)
    gq = importlib.import_module("weight-quantizer_b200.gptq")
    g = torch.Generator().manual_seed(11)
    kk = 4096
    xc = torch.randn(8192, kk, generator=g)
    hess = (xc.double().t() @ xc.double() / xc.shape[0])
    wg = torch.randn(kk, kk, generator=g) * 0.02
    gcfg = wq.QuantConfig(bits=4, symmetric=True, group_size=128, method=wq.Method.GPTQ)
    hd, wd = hess.to(dev), wg.to(dev)
    gms = gpu_ms(lambda: gq.gptq_quantize(wd, hd, gcfg))
    sample_rows = 256
    gms_sample = gpu_ms(lambda: gq.gptq_quantize(wd[:sample_rows], hd, gcfg))
    gptq = {"layer": "4096x4096 int4 sym g128, Hessian of 8192 rows", "ms": round(gms, 2),
            "timed": "factorization, qparams, sweep and tail kernels (all this library's), host reads of their flags"}
    if ref_rtn is not None:
        ref_gptq = importlib.import_module("ptqkit.gptq")
        rq = ref_rtn.QuantConfig(bits=4, symmetric=True, group_size=128, method=ref_rtn.Method.GPTQ)
        ws = wg[:sample_rows].contiguous()
        cms = cpu_ms(lambda: ref_gptq.gptq_quantize(ws, hess, rq), 0.0)
        gptq["same_work"] = {"rows": sample_rows, "gpu_ms": round(gms_sample, 2), "cpu_ms": round(cms, 1),
                             "cpu": f"ptqkit.gptq.gptq_quantize, torch CPU, {threads} threads",
                             "speedup_vs_cpu": round(cms / gms_sample, 1)}
    del flush_w, flush_r
    return {"configs": out, "rtn": rtn, "gptq": gptq}


def ours(args: argparse.Namespace) -> None:
    import numpy as np
    import torch
    import torch.distributed as dist

    wq = importlib.import_module("weight-quantizer_b200")
    wl = importlib.import_module("weight-quantizer_b200.workloads")
    sharded = importlib.import_module("weight-quantizer_b200.sharded")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))

    def barrier() -> None:
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    peaks = _peaks()
    batches = sorted(set([args.batch] + [b for b in args.sweep if b != args.batch]))
    layer = wl.sharded_28672x8192(batches=tuple(b for b in batches if b in (1, 32, 256, 4096)))[0]
    for b in batches:
        if b not in layer.x:
            layer.x[b] = torch.randn(b, K_COLS, generator=torch.Generator().manual_seed(b))
    mp, ranges = sharded.shard_rows(M_ROWS, world)
    r0, r1 = ranges[rank]
    qw_rows = wq.quantize_weight(layer.weight[r0:r1].to(dev), layer.config)
    full_qw = wq.QuantizedWeight(
        codes=qw_rows.codes, scales=qw_rows.scales, zeros=qw_rows.zeros, bits=4, group_size=GROUP,
        in_features=K_COLS, out_features=r1 - r0, symmetric=True, packed=True, granularity="group")
    shard = sharded.shard_weight(full_qw, 0, 1) if (r1 - r0) == mp else None
    if shard is None:
        pad = mp - (r1 - r0)
        shard = wq.QuantizedWeight(
            codes=torch.cat((full_qw.codes, torch.zeros(pad, full_qw.codes.shape[1], dtype=torch.uint8, device=dev))),
            scales=torch.cat((full_qw.scales, torch.ones(pad, full_qw.scales.shape[1], device=dev))),
            zeros=torch.cat((full_qw.zeros, torch.zeros(pad, full_qw.zeros.shape[1], device=dev))),
            bits=4, group_size=GROUP, in_features=K_COLS, out_features=mp, symmetric=True, packed=True,
            granularity="group")
    lin = sharded.RowParallelDequantLinear(shard, M_ROWS, rank, world)
    weight_bytes_job = (M_ROWS * (K_COLS // 2)) + 2 * 4 * M_ROWS * (K_COLS // GROUP)
    # our kernels per step: batch >= 5 runs the x' prep kernel and the
    # tensor-core kernel, batch <= 4 the decode kernel alone; for N > 1 the
    # tensor-core epilogue stores into every rank's y (the one-element
    # all-reduces that order the ranks are NCCL's)
    launches_per_step = 2 if args.batch > 4 else 1

    stream = torch.cuda.current_stream(dev)
    B = args.batch
    x = layer.x[B].to(dev)

    # ---- main line: K steps of the whole layer at batch B ------------------
    for _ in range(args.warmup):
        lin.forward(x)
    torch.cuda.synchronize()
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(args.steps):
            lin.forward(x)
        end.record(stream)
        torch.cuda.synchronize()
        barrier()
    t_step = max_over_ranks(start.elapsed_time(end) / args.steps / 1e3)
    flops = 2.0 * B * M_ROWS * K_COLS
    value = flops / t_step / 1e9
    clock = clocks.summary()

    # ---- N > 1: the same layer with y left sharded (no exchange) -------------
    # the case where the next layer consumes the row shards (forward(gather=False))
    no_gather = None
    if world > 1:
        for _ in range(args.warmup):
            lin.forward(x, gather=False)
        torch.cuda.synchronize()
        barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for _ in range(args.steps):
            lin.forward(x, gather=False)
        s1.record(stream)
        torch.cuda.synchronize()
        barrier()
        t_ng = max_over_ranks(s0.elapsed_time(s1) / args.steps / 1e3)
        no_gather = {"value": round(flops / t_ng / 1e9, 1), "unit": "GFLOP/s", "ms_per_step": round(t_ng * 1e3, 4),
                     "what": "each rank's row shard of y left in place (forward(gather=False)), max over ranks"}

    # ---- dominant kernel alone (local GEMM), for the roofline --------------
    local_out = torch.empty((max(batches), mp), dtype=torch.float32, device=dev)
    kt = []
    for i in range(args.warmup + args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        lin.forward_local(x, out=local_out[:B])
        e1.record(stream)
        if i >= args.warmup:
            kt.append((e0, e1))
    torch.cuda.synchronize()
    t_kernel = sum(a.elapsed_time(b) for a, b in kt) / len(kt) / 1e3
    kernel_flops = 2.0 * B * mp * K_COLS
    achieved_tflops = kernel_flops / t_kernel / 1e12
    # DRAM bytes (read + write) of one tensor-core launch at batch 4096 on one
    # GPU, from the latest ncu capture of this kernel summarised in
    # profiles/dq_gemm_tc_28672x8192_b4096.md (memory-side counters)
    traffic = 0.746892e9 + 0.454140e9 if (B == 4096 and world == 1) else None
    roofline = {"bound": "tensor", "achieved": round(achieved_tflops, 3), "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": round(achieved_tflops / peaks["bf16_tflops"], 4), "traffic": traffic,
                "traffic_unit": "bytes per launch",
                "kernel": "dequant-GEMM (batch %d, %d rows per GPU; the timed call is the x' prep kernel "
                          "plus the tensor-core kernel)" % (B, mp),
                "kernel_ms": round(t_kernel * 1e3, 4), "peak_source": peaks["source"]}

    # ---- sweep: decode batches, L2 flushed between iterations --------------
    # The flush writes one 256 MB buffer and then reads another, so L2 holds
    # none of the layer's data and no dirty lines whose write-back would
    # compete with the timed kernel's reads.
    flush_w = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    flush_r = torch.ones(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    def flush_l2(i: int) -> None:
        flush_w.fill_(float(i))
        flush_r.sum()

    sweep = []
    for b in args.sweep:
        if b == B:
            continue
        xb = layer.x[b].to(dev)
        for _ in range(args.warmup):
            lin.forward(xb)
        ts = []
        for _ in range(args.steps):
            flush_l2(len(ts))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            barrier()
            e0.record(stream)
            lin.forward(xb)
            e1.record(stream)
            ts.append((e0, e1))
        torch.cuda.synchronize()
        t = max_over_ranks(statistics.median(a.elapsed_time(c) for a, c in ts) / 1e3)
        kt2 = []
        for _ in range(args.steps):
            flush_l2(len(kt2))
            # ~0.5 ms of device-side wait: the host has enqueued the call before
            # the device reaches e0, so the host's launch latency stays outside
            # the kernel's time
            torch.cuda._sleep(1_000_000)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            lin.forward_local(xb, out=local_out[:b])
            e1.record(stream)
            kt2.append((e0, e1))
        torch.cuda.synchronize()
        tk = statistics.median(a.elapsed_time(c) for a, c in kt2) / 1e3
        shard_bytes = mp * (K_COLS // 2) + 2 * 4 * mp * (K_COLS // GROUP) + 4 * b * K_COLS + 4 * b * mp
        back_to_back = None
        if b == 1 and world == 1:
            # a decode step runs layers back to back: two copies of the weights
            # (264 MB, more than twice L2) alternate, 2 x steps launches timed as one
            twin = [lin.shard, wq.QuantizedWeight(
                codes=lin.shard.codes.clone(), scales=lin.shard.scales.clone(), zeros=lin.shard.zeros.clone(),
                bits=4, group_size=GROUP, in_features=K_COLS, out_features=mp, symmetric=True, packed=True,
                granularity="group")]
            for i in range(4):
                wq.dequant_gemm(xb, twin[i & 1], impl="kernel", out=local_out[:1])
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            n_b2b = 2 * args.steps
            e0.record(stream)
            for i in range(n_b2b):
                wq.dequant_gemm(xb, twin[i & 1], impl="kernel", out=local_out[:1])
            e1.record(stream)
            torch.cuda.synchronize()
            tb = e0.elapsed_time(e1) / n_b2b / 1e3
            back_to_back = {"launches": n_b2b, "ms": round(tb * 1e3, 4),
                            "hbm_gbs": round(shard_bytes / tb / 1e9, 1),
                            "hbm_frac": round(shard_bytes / tb / 1e9 / peaks["hbm_gbs"], 4),
                            "how": "two weight copies (264 MB) alternating, launches back to back, one event pair"}
            del twin
        sweep.append({
            "batch": b, "ms": round(t * 1e3, 4), "gflops": round(2.0 * b * M_ROWS * K_COLS / t / 1e9, 1),
            "weight_gbs": round(weight_bytes_job / t / 1e9, 1),
            "kernel_ms": round(tk * 1e3, 4),
            "kernel_hbm_gbs": round(shard_bytes / tk / 1e9, 1),
            "kernel_hbm_frac": round(shard_bytes / tk / 1e9 / peaks["hbm_gbs"], 4),
            "back_to_back": back_to_back,
        })

    # ---- end to end through the public API with pinned host buffers --------
    e2e = None
    if not args.no_e2e:
        # Each rank brings 1/N of the batch rows in from pinned host memory and
        # takes 1/N of the output rows back; for N > 1 an NCCL all-gather
        # assembles the whole x on every rank over NVLink.
        rows_per_rank = (B + world - 1) // world
        b0, b1 = min(rank * rows_per_rank, B), min((rank + 1) * rows_per_rank, B)
        x_h = torch.zeros((rows_per_rank, K_COLS), dtype=torch.float32)
        x_h[: b1 - b0] = layer.x[B][b0:b1]
        x_h = x_h.pin_memory()
        y_h = torch.empty((b1 - b0, M_ROWS), dtype=torch.float32).pin_memory()
        x_all = torch.empty((world * rows_per_rank, K_COLS), dtype=torch.float32, device=dev)
        x_mine = x_all[rank * rows_per_rank:(rank + 1) * rows_per_rank]

        # One GPU: the batch goes through in E2E_CHUNKS chunks on two streams,
        # so one chunk's host->device copy, another's kernels and a third's
        # device->host copy overlap (separate copy engines each way).
        n_chunks = E2E_CHUNKS if (world == 1 and B % E2E_CHUNKS == 0) else 1
        crow = B // n_chunks
        side = [torch.cuda.Stream(dev) for _ in range(2)] if n_chunks > 1 else []
        xbuf = [torch.empty((crow, K_COLS), dtype=torch.float32, device=dev) for _ in side]
        ybuf = [torch.empty((crow, mp), dtype=torch.float32, device=dev) for _ in side]

        def e2e_step() -> None:
            if n_chunks > 1:
                cur = torch.cuda.current_stream(dev)
                for sd in side:
                    sd.wait_stream(cur)
                for c in range(n_chunks):
                    sd = side[c & 1]
                    with torch.cuda.stream(sd):
                        xbuf[c & 1].copy_(x_h[c * crow:(c + 1) * crow], non_blocking=True)
                        wq.dequant_gemm(xbuf[c & 1], lin.shard, impl="kernel", out=ybuf[c & 1])
                        y_h[c * crow:(c + 1) * crow].copy_(ybuf[c & 1][:, :M_ROWS], non_blocking=True)
                for sd in side:
                    cur.wait_stream(sd)
                return
            x_mine.copy_(x_h, non_blocking=True)
            if world > 1:
                dist.all_gather_into_tensor(x_all, x_mine)
            y = lin.forward(x_all[:B])
            y_h.copy_(y[b0:b1], non_blocking=True)

        for _ in range(args.warmup):
            e2e_step()
        torch.cuda.synchronize()
        barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        s1.record(stream)
        torch.cuda.synchronize()
        barrier()
        t_e2e = max_over_ranks(s0.elapsed_time(s1) / args.steps / 1e3)
        e2e = {"value": round(flops / t_e2e / 1e9, 1), "unit": "GFLOP/s",
               "h2d_bytes_per_step": int(world * rows_per_rank * K_COLS * 4),
               "d2h_bytes_per_step": int(B * M_ROWS * 4),
               "ms_per_step": round(t_e2e * 1e3, 3),
               "path": (f"{n_chunks} chunks of {crow} rows on two streams: pinned host -> device, "
                        "dequant_gemm (public API), device -> pinned host, overlapped") if n_chunks > 1 else
                       "each rank: its 1/N of x rows pinned host -> device"
                       + (", NCCL all-gather of x" if world > 1 else "")
                       + ", RowParallelDequantLinear.forward (dequant_gemm kernel"
                       + (" storing y into every rank over NVLink" if world > 1 else "")
                       + "), its 1/N of y rows -> pinned host"}

    # ---- compressed-format loader: this layer written and read back ---------
    loader = None
    if rank == 0 and world == 1 and not args.no_loader:
        loader = loader_line(wq, full_qw, dev, stream, peaks)

    per_config = None
    if rank == 0 and world == 1 and not args.no_configs:
        per_config = config_lines(wq, wl, dev, stream, peaks, args.cpu_seconds / 4, max(args.steps, 5))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sample = min(args.cpu_sample_rows, B)
        cpu = cpu_baseline_sample(full_qw.codes.cpu().numpy(), full_qw.scales.cpu().numpy(),
                                  full_qw.zeros.cpu().numpy(), layer.x[B][:sample].numpy(), args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t_step * 1e3, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16 hi/lo -> f32",
            "data": "synthetic (seeded: W ~ N(0, 0.015), x ~ N(0, 1))",
            "config": {"workload": WORKLOAD, "M": M_ROWS, "K": K_COLS, "batch": B, "bits": 4,
                       "group_size": GROUP, "symmetric": True,
                       "parallelism": f"row-sharded x{world}" + (f" + y stored into every rank ({lin.exchange})"
                                                                   if world > 1 else ""),
                       "l2": "working set larger than L2 (x 134 MB, y 470 MB, weights 132 MB at batch 4096); "
                             "sweep lines flush L2 (256 MB write, then a 256 MB read of another buffer) "
                             "between iterations"},
            "weight_gbs": round(weight_bytes_job / t_step / 1e9, 1),
            "clocks": {"sm_mhz": clock["sm_mhz"], "sm_max_mhz": clock["sm_max_mhz"], "reasons": clock["reasons"]},
            "roofline": roofline,
            "sweep": sweep,
            "e2e": e2e,
            "y_sharded": no_gather,
            "loader": loader,
            "per_config": per_config,
            "cpu_baseline": cpu,
            "gpu_launches": args.steps * launches_per_step,
        }
        print(json.dumps(line), flush=True)
    del np
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--batch", type=int, default=4096)
    ap.add_argument("--sweep", type=lambda s: [int(v) for v in s.split(",") if v], default=[1, 32, 256])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-loader", action="store_true")
    ap.add_argument("--no-configs", action="store_true")
    ap.add_argument("--cpu-sample-rows", type=int, default=64)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        reference_arm(args)
    else:
        ours(args)


if __name__ == "__main__":
    main()
