#!/usr/bin/env python
"""Benchmark of the B200-native Prometheus reactor (driver contract).

Headline metric: fp32 SGEMM TFLOP/s at 8192^3.

  * One step = one C = A*B of the workload through the reactor's device entry
    point (oct_b200_sgemm_device_ld): the TF32 split pass plus the tcgen05
    3xTF32 main kernel.  Inputs (U[-1,1), seeded) are resident in HBM and each
    operand (256 MiB) is larger than the 126 MB L2, so no flush is needed.
  * N > 1 ranks (torchrun, one per GPU): the column-parallel form of the large
    GEMM.  Every rank holds A and its own 8192-column shard of B and writes its
    shard of C (global N = 8192 * world): weak scaling, no data-path
    collective (C stays column-sharded, as a column-parallel layer leaves it).
  * `value` is whole-job TFLOP/s over the max-over-ranks device time of K steps.
  * `e2e` is the same metric through the reference-facing host ABI
    (prometheus_reactor_runtime_sgemm) with pinned host buffers: the host->device
    copy of A and B and the device->host copy of C are inside the timed region.
  * `roofline`: the main kernel's useful flops per launch / its CUDA-event time
    on the launch stream, against the 3xTF32-adjusted tensor peak derived from
    the measured burst dense bf16 peak (tf32 runs at half the bf16 rate, and each
    fp32 product costs three tf32 products): peak = bf16_tflops / 6, scaled by the
    run's median SM clock over the maximum when the part ran below it.
  * `cpu_baseline`: Oct's CPU SGEMM (`cpuSGEMM`, internal/prometheus/runtime.go:319-331,
    restated in oracle/oracle.c) on all host cores, over a bounded row sample.

`--impl reference` times that same CPU restatement as the reference arm (Oct's
reactor needs Vulkan and cannot run on this machine; its Go CPU path is the
reference implementation that exists here).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--m", type=int, default=8192)
    p.add_argument("--n", type=int, default=8192, help="columns per rank")
    p.add_argument("--k", type=int, default=8192)
    p.add_argument("--variant", type=int, default=0,
                   help="0 = AUTO (the library's own choice: at 8192^3 the CTA pair with 32-deep stages), "
                        "16/32 = tcgen05 one CTA per tile with that K stage depth, 216/232 = CTA pair, "
                        "316/332 = CTA pair with the TF32 split inside the kernel, 2 = FMA")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-secondary", action="store_true")
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="target length of the CPU sample")
    p.add_argument("--workload", default="sgemm",
                   choices=["sgemm", "gemma_block", "dit_block", "reductions", "attention", "smallm"],
                   help="sgemm = the driver contract line; the others run one secondary measurement "
                        "alone (for profiling) and print it as JSON")
    return p.parse_args()


def peaks() -> tuple[dict, str]:
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return json.loads(path.read_text()), "measured"
        except Exception:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def nvidia_smi_selector(props) -> str:
    """The `nvidia-smi -i` argument naming the GPU behind a CUDA device.

    nvidia-smi ignores CUDA_VISIBLE_DEVICES and numbers every GPU of the node, so
    the CUDA ordinal would name another GPU whenever the visible set is a subset
    (a lease of GPU 3 is CUDA device 0).  The device's UUID names it on both sides."""
    uuid = str(getattr(props, "uuid", "") or "")
    if not uuid:
        raise ValueError("device properties carry no UUID")
    return uuid if uuid.startswith(("GPU-", "MIG-")) else f"GPU-{uuid}"


def tensor_roofline_peak(pk: dict, pk_kind: str, clock_rec: dict) -> tuple[float, str]:
    """The 3xTF32-adjusted tensor peak a kernel timed in this run is held against.

    The measured burst cuBLAS bf16 figure / 2 (tf32 runs at half the bf16 rate) / 3
    (products per fp32 MAC).  When this run's clock record shows the part below its
    maximum clock (the 1 kW power cap), that figure scaled by the median SM clock is
    also formed, but the larger of the two is the denominator: on this pool's B200s
    the scaling understates what the part delivers at the lower clock (the driver's own
    sustained cuBLAS loop reaches 1363.6 TFLOP/s at a 1297 MHz median, where the
    burst figure scaled by that clock predicts 1063), so the unscaled burst figure is
    the largest measured capability and the most conservative denominator."""
    burst = pk["bf16_tflops"] / 6.0
    note = f"{pk_kind}: bf16_tflops {pk['bf16_tflops']} (burst) / 2 (tf32 rate) / 3 (products)"
    sm, smax = clock_rec.get("sm_mhz"), clock_rec.get("sm_max_mhz") or pk.get("sm_max_mhz")
    if sm and smax and sm < 0.98 * smax:
        ratio = sm / smax
        return burst, note + (f", not scaled: the median SM clock {sm:.0f} / max {smax:.0f} MHz = {ratio:.3f} "
                              f"would give {burst * ratio:.1f}, below what cuBLAS sustains at such clocks")
    return burst, note + (f", part at its maximum clock (median {sm:.0f} MHz)" if sm else ", no clock record")


def clock_scaled_peak(pk: dict, clock_rec: dict) -> float:
    """The burst peak scaled by this run's median SM clock over the maximum (reported beside frac)."""
    burst = pk["bf16_tflops"] / 6.0
    sm, smax = clock_rec.get("sm_mhz"), clock_rec.get("sm_max_mhz") or pk.get("sm_max_mhz")
    return burst * (sm / smax) if sm and smax else burst


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 50 ms during the timed region.

    `gpu` is an nvidia-smi selector (a UUID from nvidia_smi_selector), never a CUDA ordinal."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: str):
        self.gpu = gpu
        self.proc = None
        self.lines: list[str] = []
        self.start = 0

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            # nvidia-smi takes a moment to start: begin the timed region only once it
            # reports, and keep only the samples taken from then on
            t0 = time.time()
            while not self.lines and time.time() - t0 < 5.0:
                time.sleep(0.01)
            self.start = len(self.lines)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            # at least one sample after the region started (short regions end between samples)
            t0 = time.time()
            while len(self.lines) <= self.start and time.time() - t0 < 2.0:
                time.sleep(0.01)
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in (self.lines[self.start:] or self.lines):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                smax.append(float(parts[1]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[4:8]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "gpu": self.gpu}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm), "gpu": self.gpu}


def cpu_sgemm_sample(m: int, n: int, k: int, seconds: float, threads: int) -> dict:
    """Oct's cpuSGEMM restated (oracle port) on a bounded sample of output rows."""
    from oracle import oracle as O
    a = O.uniform_matrix(m, k, 1000).ravel()
    b = O.uniform_matrix(k, n, 1001).ravel()
    probe_rows = max(1, threads)
    t0 = time.perf_counter()
    O.cpu_sgemm_f32(a, b, m, n, k, rows=slice(0, probe_rows), threads=threads)
    t_probe = time.perf_counter() - t0
    rows = probe_rows * max(1, int(seconds / max(t_probe, 1e-6)))
    rows = min(rows, m)
    t0 = time.perf_counter()
    O.cpu_sgemm_f32(a, b, m, n, k, rows=slice(0, rows), threads=threads)
    t = time.perf_counter() - t0
    return {"value": 2.0 * rows * n * k / t / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"cpuSGEMM (fp32 i-j-k, runtime.go:319-331, C restatement) on {rows} of {m} output rows of "
                      f"{m}x{n}x{k}, {t:.1f} s on {threads} threads, extrapolated per flop",
            "seconds": t, "rows": rows}


def cpu_baseline_table(threads: int, budget_s: float = 2.0) -> list[dict]:
    """The reference's CPU paths, restated in C / numpy (oracle/, the checker), each timed
    with one thread and with all host threads: cpuSGEMM (runtime.go:319-331) and the fp64
    `@` __octMatMulMM (emit_go_runtime.go:168-200) on output-row samples of 8192^3 sized to
    ~budget_s; prom_reduction_cpu_reference (reactor_vulkan_fused_reduction.c:996-1114) for
    sum / max / softmax and CanonicalRMSNorm (canonical_contract.go:91-105) over all of
    32768 x {256, 2048, 4096}; the binary64 block pipelines (oracle/blocks.py) at a reduced
    token count."""
    import numpy as np
    from oracle import oracle as O
    from oracle import blocks as OB
    out = []

    def timed(fn):
        t0 = time.perf_counter()
        fn()
        return time.perf_counter() - t0

    m = n = k = 8192
    a = O.uniform_matrix(m, k, 1000).ravel()
    b = O.uniform_matrix(k, n, 1001).ravel()
    for th in (1, threads):
        probe = timed(lambda: O.cpu_sgemm_f32(a, b, m, n, k, rows=slice(0, th), threads=th))
        rows = min(m, th * max(1, int(budget_s / max(probe, 1e-6))))
        t = timed(lambda: O.cpu_sgemm_f32(a, b, m, n, k, rows=slice(0, rows), threads=th))
        out.append({"path": "cpuSGEMM fp32 (runtime.go:319-331)", "kind": "port (C restatement)", "cores": th,
                    "shape": f"{m}x{n}x{k}", "sample_rows": rows, "TFLOP/s": 2.0 * rows * n * k / t / 1e12})
    a64, b64 = a.astype(np.float64), b.astype(np.float64)
    probe = timed(lambda: O.oct_matmul_f64(a64, b64, m, n, k, rows=slice(0, 1)))
    rows = min(m, max(1, int(budget_s / max(probe, 1e-6))))
    t = timed(lambda: O.oct_matmul_f64(a64, b64, m, n, k, rows=slice(0, rows)))
    out.append({"path": "Oct `@` __octMatMulMM[float64] (emit_go_runtime.go:168-200)", "kind": "port (C restatement)",
                "cores": 1, "shape": f"{m}x{n}x{k}", "sample_rows": rows, "TFLOP/s": 2.0 * rows * n * k / t / 1e12})
    del a, b, a64, b64
    # Row reductions and RMSNorm over all 32768 rows of the reference tests' deterministic
    # input, GB/s of algorithmic bytes
    for width in (256, 2048, 4096):
        x = O.reduction_input(32768, width)
        w = (np.random.default_rng(width + 1).random(width) + 0.5).astype(np.float32)
        r = x.shape[0]
        for th in (1, threads):
            for name, op in (("sum", 1), ("max", 2), ("softmax", 3), ("rmsnorm", 0)):
                if op == 0:
                    t = timed(lambda: O.rmsnorm_f32(x, w, 1e-5, threads=th, form="canonical"))
                    nbytes = 8 * r * width
                    path = "CanonicalRMSNorm (canonical_contract.go:91-105)"
                else:
                    t = timed(lambda: O.reduction_cpu_reference(x, op, threads=th))
                    nbytes = (8 if op == 3 else 4) * r * width + (0 if op == 3 else 4 * r)
                    path = f"prom_reduction_cpu_reference {name} (reactor_vulkan_fused_reduction.c)"
                out.append({"path": path, "kind": "port (C restatement)", "cores": th,
                            "shape": f"{r}x{width}", "GB/s": nbytes / t / 1e9, "rows/s": r / t})
        del x
    # Block pipelines in binary64 at a reduced token count (numpy BLAS on every host thread)
    for name, cfg, ts in (("gemma_block", OB.gemma_config(seq_len=128), None),
                          ("dit_block", OB.dit_config(seq_len=256, grid_w=16), [500.0])):
        wts = OB.random_weights(cfg, seed=3)
        xb = np.random.default_rng(4).standard_normal((cfg.seq_len, cfg.hidden)).astype(np.float32)
        t = timed(lambda: OB.forward(cfg, wts, xb, ts))
        out.append({"path": f"{name} pipeline, binary64 numpy restatement (oracle/blocks.py)",
                    "kind": "port (numpy, BLAS threads)", "cores": threads,
                    "shape": f"1 x {cfg.seq_len} tokens at the benchmark hidden / head / FFN dims",
                    "tokens/s": cfg.seq_len / t,
                    "note": "reduced token count: attention is a smaller share than at the benchmark length"})
    for r in out:
        for key in ("TFLOP/s", "GB/s", "rows/s", "tokens/s"):
            if key in r:
                r[key] = round(r[key], 6 if key == "TFLOP/s" else 2)
    return out


def ragged_sgemm_measurements(rt, torch, stream) -> list[dict]:
    """The reference's smaller SGEMM configurations (512^3, 1000^3 and the ragged
    4097 x 4095 x 1023) on the device (the auto-selected kernel) and end to end through
    prometheus_reactor_runtime_sgemm with host buffers (copies included)."""
    import numpy as np
    from oct_b200 import reactor as R
    out = []
    for (m, n, k) in ((512, 512, 512), (1000, 1000, 1000), (4097, 4095, 1023)):
        g = torch.Generator(device="cuda").manual_seed(m + n)
        a = torch.rand(m, k, device="cuda", generator=g) * 2 - 1
        b = torch.rand(k, n, device="cuda", generator=g) * 2 - 1
        c = torch.empty(m, n, device="cuda")
        iters = 50
        for _ in range(5):
            rt.sgemm_device(a, b, c, m, n, k, R.SGEMM_AUTO, stream)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(iters):
            rt.sgemm_device(a, b, c, m, n, k, R.SGEMM_AUTO, stream)
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / iters
        ha, hb = a.cpu().numpy().ravel(), b.cpu().numpy().ravel()
        hc = np.empty(m * n, dtype=np.float32)
        for _ in range(3):
            rt.sgemm_with_status(m, n, k, ha, hb, out=hc)
        t0 = time.perf_counter()
        for _ in range(10):
            _, st = rt.sgemm_with_status(m, n, k, ha, hb, out=hc)
        e2e_ms = (time.perf_counter() - t0) * 100.0
        if not st.ok:
            raise RuntimeError(f"sgemm {m}x{n}x{k} failed: {st}")
        flops = 2.0 * m * n * k
        out.append({"kernel": f"sgemm_{m}x{n}x{k}", "variant": "auto", "ms": round(ms, 4),
                    "TFLOP/s": round(flops / (ms * 1e-3) / 1e12, 2), "e2e_ms": round(e2e_ms, 4),
                    "e2e_TFLOP/s": round(flops / (e2e_ms * 1e-3) / 1e12, 3),
                    "e2e_path": "prometheus_reactor_runtime_sgemm, pageable host buffers"})
        del a, b, c
    return out


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # the reference arm runs on rank 0 only
    from oracle import oracle as O
    O.build()
    threads = O.max_threads()
    m, n, k = args.m, args.n, args.k
    a = O.uniform_matrix(m, k, 1000).ravel()
    b = O.uniform_matrix(k, n, 1001).ravel()
    # Size one step as a bounded row sample so the whole run stays within minutes.
    t0 = time.perf_counter()
    O.cpu_sgemm_f32(a, b, m, n, k, rows=slice(0, threads), threads=threads)
    t_probe = time.perf_counter() - t0
    budget = 150.0 / max(1, args.steps + args.warmup)
    rows = min(m, max(1, int(threads * budget / max(t_probe, 1e-6))))
    for _ in range(args.warmup):
        O.cpu_sgemm_f32(a, b, m, n, k, rows=slice(0, rows), threads=threads)
    times = []
    for s in range(args.steps):
        r0 = (s * rows) % max(1, m - rows + 1)
        t0 = time.perf_counter()
        O.cpu_sgemm_f32(a, b, m, n, k, rows=slice(r0, r0 + rows), threads=threads)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = 2.0 * rows * n * k * args.steps / total / 1e12
    sample = (f"cpuSGEMM (fp32 i-j-k, internal/prometheus/runtime.go:319-331; C restatement, Oct's Go/Vulkan "
              f"reactor cannot run here) on {rows} of {m} rows of {m}x{n}x{k} per step, {threads} threads")
    line = {
        "impl": "reference", "metric": "fp32 SGEMM TFLOP/s at 8192^3", "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"sgemm {m}x{n}x{k} (row sample per step)", "m": m, "n": n, "k": k},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def reduction_measurements(rt, torch, hbm_peak: float) -> list[dict]:
    """Row reductions and RMSNorm at the benchmark shapes (32768 rows x 256 / 2048 / 4096)."""
    from oct_b200 import reactor as R
    out = []
    stream = torch.cuda.current_stream()
    rows = 32768
    l2_bytes = 126 * 2 ** 20
    for width in (256, 2048, 4096):
        g = torch.Generator(device="cuda").manual_seed(width)
        # back-to-back launches rotate over enough inputs that each one was evicted from L2
        # (126 MB) by the launches before it: 12 x 33.5 MB at W = 256, 2 at the larger widths
        nbuf = max(2, -(-3 * l2_bytes // (4 * rows * width)))
        xs = [torch.randn(rows, width, device="cuda", generator=g) for _ in range(nbuf)]
        w = torch.rand(width, device="cuda", generator=g) + 0.5
        y_row = torch.empty(rows, device="cuda")
        y_full = torch.empty_like(xs[0])
        inv = torch.empty(rows, device="cuda")
        for name, fn, nbytes in (
            ("row_sum", lambda x: rt.reduction_device(x, y_row, rows, width, R.OP_SUM, stream),
             4 * rows * width + 4 * rows),
            ("row_max", lambda x: rt.reduction_device(x, y_row, rows, width, R.OP_MAX, stream),
             4 * rows * width + 4 * rows),
            ("softmax", lambda x: rt.reduction_device(x, y_full, rows, width, R.OP_SOFTMAX, stream),
             8 * rows * width),
            ("rmsnorm", lambda x: rt.rmsnorm_device(x, w, y_full, inv, rows, width, 1e-6, stream),
             8 * rows * width + 4 * width),
        ):
            for i in range(max(3, nbuf)):
                fn(xs[i % nbuf])
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            iters = 24
            e0.record(stream)
            for i in range(iters):
                fn(xs[i % nbuf])
            e1.record(stream)
            e1.synchronize()
            ms = e0.elapsed_time(e1) / iters
            gbs = nbytes / (ms * 1e-3) / 1e9
            out.append({"kernel": name, "rows": rows, "width": width, "ms": round(ms, 5), "GB/s": round(gbs, 1),
                        "frac_of_hbm": round(gbs / hbm_peak, 3), "bytes": nbytes,
                        "l2": f"inputs rotate over {nbuf} buffers ({nbuf * 4 * rows * width / 1e6:.0f} MB)"})
        st = rt.sync_status()
        if not st.ok:
            raise RuntimeError(f"reduction status {st}")
        del xs, y_full, y_row, inv
    return out


def smallm_measurements(rt, torch, stream, hbm_peak: float) -> list[dict]:
    """Small-M products (Gemma per-token shapes): HBM-bound on B; B = 134 MB > L2, no flush needed."""
    from oct_b200 import reactor as R
    out = []
    for (m, n, k) in ((1, 16384, 2048), (8, 16384, 2048), (16, 8192, 4096)):  # B = 134 MB > L2
        g = torch.Generator(device="cuda").manual_seed(11)
        a = torch.rand(m, k, device="cuda", generator=g) * 2 - 1
        b = torch.rand(k, n, device="cuda", generator=g) * 2 - 1
        c = torch.empty(m, n, device="cuda")
        for variant, label in ((R.SGEMM_AUTO, "sgemm_smallm"), (R.SGEMM_SMALLM, "sgemm_smallm_cuda_cores"),
                               (R.SGEMM_SMALLM_TC, "sgemm_smallm_tensor_cores")):
            for _ in range(3):
                rt.sgemm_device(a, b, c, m, n, k, variant, stream)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            iters = 20
            e0.record(stream)
            for _ in range(iters):
                rt.sgemm_device(a, b, c, m, n, k, variant, stream)
            e1.record(stream)
            e1.synchronize()
            ms = e0.elapsed_time(e1) / iters
            nbytes = 4 * (k * n + m * k + m * n)
            out.append({"kernel": label, "m": m, "n": n, "k": k, "ms": round(ms, 4),
                        "GB/s": round(nbytes / (ms * 1e-3) / 1e9, 1),
                        "frac_of_hbm": round(nbytes / (ms * 1e-3) / 1e9 / hbm_peak, 3),
                        "bytes": nbytes, "l2": "B larger than L2, no flush"})
    return out


def secondary_measurements(rt, torch, hbm_peak: float) -> list[dict]:
    """Reductions, the transformer blocks, the FMA control and the 32-deep tensor-core variant."""
    from oct_b200 import reactor as R
    out = reduction_measurements(rt, torch, hbm_peak)
    stream = torch.cuda.current_stream()
    # Transformer blocks at the benchmark shapes (random init, synthetic tokens)
    out.extend(block_measurements(rt, torch, stream))
    out.extend(attention_measurements(rt, torch, stream))
    out.extend(smallm_measurements(rt, torch, stream, hbm_peak))
    out.extend(ragged_sgemm_measurements(rt, torch, stream))
    # FMA control and the 32-deep tensor-core variant at the headline shape
    m = n = k = 8192
    g = torch.Generator(device="cuda").manual_seed(7)
    a = torch.rand(m, k, device="cuda", generator=g) * 2 - 1
    b = torch.rand(k, n, device="cuda", generator=g) * 2 - 1
    c = torch.empty(m, n, device="cuda")
    for variant, label, iters in ((R.SGEMM_FMA, "sgemm_fma_control", 3), (R.SGEMM_TC_BK16, "sgemm_3xtf32_bk16", 5),
                                  (R.SGEMM_TC_BK32, "sgemm_3xtf32_bk32", 5),
                                  (R.SGEMM_TC_PAIR16, "sgemm_3xtf32_pair16", 5),
                                  (R.SGEMM_TC_PAIR32, "sgemm_3xtf32_pair32", 5),
                                  (R.SGEMM_TC_INSM16, "sgemm_3xtf32_insm16", 5),
                                  (R.SGEMM_TC_INSM32, "sgemm_3xtf32_insm32", 5)):
        rt.sgemm_device(a, b, c, m, n, k, variant, stream)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(iters):
            rt.sgemm_device(a, b, c, m, n, k, variant, stream)
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / iters
        out.append({"kernel": label, "m": m, "n": n, "k": k, "ms": round(ms, 3),
                    "TFLOP/s": round(2.0 * m * n * k / (ms * 1e-3) / 1e12, 2)})
    rt.set_kernel_timing(False)
    return out


def attention_measurements(rt, torch, stream, iters: int = 5) -> list[dict]:
    """The fused attention kernel alone at the DiT block's shape (2 items x 4096 tokens x 24 heads of 128)."""
    from oracle import blocks as OB  # used only for the shape
    pk, _ = peaks()
    peak = pk["bf16_tflops"] / 6.0  # burst 3xTF32-adjusted peak
    cfg, items = OB.dit_config(), 2
    seq, heads, hd = cfg.seq_len, cfg.heads, cfg.head_dim
    g = torch.Generator(device="cuda").manual_seed(5)
    q, k, v = (torch.randn(items * seq, heads * hd, device="cuda", generator=g) for _ in range(3))
    o = torch.empty_like(q)
    for _ in range(2):
        rt.attention_device(q, k, v, o, items, seq, heads, hd, stream=stream)
    rt.set_kernel_timing(True)
    rt.read_kernel_timing()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(iters):
        rt.attention_device(q, k, v, o, items, seq, heads, hd, stream=stream)
    e1.record(stream)
    e1.synchronize()
    split_ms, main_ms, launches = rt.read_kernel_timing()
    rt.set_kernel_timing(False)
    st = rt.sync_status()
    if not st.ok:
        raise RuntimeError(f"attention status {st}")
    ms = e0.elapsed_time(e1) / iters
    kms = main_ms / max(1, launches)
    flops = 4.0 * items * heads * seq * seq * hd  # Q K^T and P V
    return [{"kernel": "flash_attention_3xtf32", "items": items, "seq": seq, "heads": heads, "head_dim": hd,
             "ms": round(ms, 3), "kernel_ms": round(kms, 3), "split_ms": round(split_ms / max(1, launches), 3),
             "TFLOP/s": round(flops / (kms * 1e-3) / 1e12, 2),
             "frac_of_3xtf32_peak": round(flops / (kms * 1e-3) / 1e12 / peak, 3)}]


def block_measurements(rt, torch, stream, iters: int = 5, only: str | None = None) -> list[dict]:
    """Tokens/s of one block forward at the benchmark shapes, plus its tensor-peak fraction."""
    from oct_b200 import reactor as R
    from oracle import blocks as OB  # used only for the shapes and the flop count
    pk, _ = peaks()
    peak = pk["bf16_tflops"] / 6.0  # burst 3xTF32-adjusted peak
    res = []
    for name, cfg, batch in (("gemma_block", OB.gemma_config(), 4), ("dit_block", OB.dit_config(), 2)):
        if only is not None and name != only:
            continue
        fam = R.BLOCK_GEMMA if cfg.family == OB.GEMMA else R.BLOCK_DIT
        blk = rt.block(fam, hidden=cfg.hidden, heads=cfg.heads, kv_heads=cfg.kv_heads, head_dim=cfg.head_dim,
                       ffn=cfg.ffn, seq_len=cfg.seq_len, max_batch=batch, eps=cfg.eps, rope_base=cfg.rope_base,
                       grid_w=cfg.grid_w, rope_frame=cfg.rope_frame)
        g = torch.Generator(device="cuda").manual_seed(99)
        weights = {}
        for wname, shape in OB.weight_shapes(cfg).items():
            t = torch.randn(*shape, device="cuda", generator=g)
            weights[wname] = (t * 0.02 + 1.0) if len(shape) == 1 and wname != "ada_b" else t * 0.02
        blk.set_weights(weights)
        del weights
        T = batch * cfg.seq_len
        x = torch.randn(T, cfg.hidden, device="cuda", generator=g)
        y = torch.empty_like(x)
        ts = [500.0, 250.0][:batch] if cfg.family == OB.DIT else None
        for _ in range(2):
            blk.forward_device(x, y, batch, ts, stream)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(iters):
            blk.forward_device(x, y, batch, ts, stream)
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / iters
        flops = OB.flops_per_forward(cfg, batch)
        res.append({"kernel": name, "batch": batch, "seq": cfg.seq_len, "hidden": cfg.hidden, "ms": round(ms, 3),
                    "tokens/s": round(T / (ms * 1e-3), 1), "TFLOP/s": round(flops / (ms * 1e-3) / 1e12, 2),
                    "frac_of_3xtf32_peak": round(flops / (ms * 1e-3) / 1e12 / peak, 3)})
        blk.close()
        del x, y
        torch.cuda.empty_cache()
    st = rt.sync_status()
    if not st.ok:
        raise RuntimeError(f"block status {st}")
    return res


def sharded_sgemm_measurements(rt, torch, dist, rank: int, world: int, stream, iters: int = 5) -> list[dict]:
    """The column-parallel SGEMM with the gather (oct_b200_sgemm_tp_device): the ragged
    sweep's two largest products at a FIXED global size (strong scaling).  Every rank holds
    the same A and N / world columns of B and ends with all of C; time = max over ranks.
    Each collective is timed; rank 0 also times the one-GPU product of the full size for
    the strong-scaling efficiency t1 / (world * tN).  Before timing, every rank's gathered
    C is compared with its own one-GPU product of the full size."""
    from oct_b200 import reactor as R
    from oct_b200 import tp
    res = []
    pk, _ = peaks()
    peak = pk["bf16_tflops"] / 6.0  # burst 3xTF32-adjusted peak
    for (m, n, k) in ((8192, 8192, 8192), (16384, 16384, 4096)):
        if n % (4 * world):
            continue
        g = torch.Generator(device="cuda").manual_seed(17)  # the same A and B on every rank
        a = torch.rand(m, k, device="cuda", generator=g) * 2 - 1
        b = torch.rand(k, n, device="cuda", generator=g) * 2 - 1
        b_shard = tp.shard_columns(b, rank, world)
        # one-GPU reference product of the full size (every rank: parity; rank 0: t1)
        c1 = torch.empty(m, n, device="cuda")
        for _ in range(2):
            rt.sgemm_device(a, b, c1, m, n, k, R.SGEMM_TC_BK16, stream)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(iters):
            rt.sgemm_device(a, b, c1, m, n, k, R.SGEMM_TC_BK16, stream)
        e1.record(stream)
        e1.synchronize()
        t1 = torch.tensor([e0.elapsed_time(e1) / iters], dtype=torch.float64)
        dist.broadcast(t1, src=0)
        del b
        for collective, cname in ((R.TP_COLLECTIVE_PEER, "peer_stores"), (R.TP_COLLECTIVE_NCCL, "nccl_allgather")):
            ids = [R.nccl_unique_id(rt.lib) if rank == 0 else None]
            dist.broadcast_object_list(ids, src=0)
            t = rt.tp_sgemm(rank, world, max_m=m, max_n=n, nccl_id=ids[0], collective=collective)
            c = torch.full((m, n), float("nan"), device="cuda")
            t.run_device(a, b_shard, c, m, n, k, stream)
            if t.sync(stream) != 0:
                raise RuntimeError(f"tp sgemm {cname} failed")
            err = float((c - c1).abs().max() / c1.abs().max())
            te = torch.tensor([err], dtype=torch.float64)
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
            del c
            for _ in range(2):
                t.run_device(a, b_shard, None, m, n, k, stream)
            torch.cuda.synchronize()
            dist.barrier()
            e0.record(stream)
            for _ in range(iters):
                t.run_device(a, b_shard, None, m, n, k, stream)
            e1.record(stream)
            e1.synchronize()
            if t.sync(stream) != 0:
                raise RuntimeError(f"tp sgemm {cname} failed")
            tt = torch.tensor([e0.elapsed_time(e1) / iters], dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t.close()
            ms, ms1 = float(tt.item()), float(t1.item())
            tf = 2.0 * m * n * k / (ms * 1e-3) / 1e12
            parity = {"vs_1gpu_normwise": float(te.item()), "ok": bool(te.item() <= 1e-6)}
            if not parity["ok"]:
                raise RuntimeError(f"tp sgemm {cname} parity failed: {parity}")
            res.append({"kernel": f"sgemm_tp_{m}x{n}x{k}", "collective": cname, "ranks": world,
                        "n_per_rank": n // world, "ms": round(ms, 3), "ms_1gpu": round(ms1, 3),
                        "TFLOP/s": round(tf, 2), "frac_of_3xtf32_peak_all_gpus": round(tf / (peak * world), 3),
                        "strong_scaling_efficiency": round(ms1 / (world * ms), 3),
                        "scaling": "strong (fixed global product, C gathered on every rank)", "parity": parity})
        del a, b_shard, c1
        torch.cuda.empty_cache()
    return res


def tp_block_measurements(rt, torch, dist, rank: int, world: int, stream, iters: int = 5) -> list[dict]:
    """Gemma / DiT blocks over all ranks, global tokens/s: pure tensor parallel (tp = world), and
    tensor parallel within groups of ranks plus data parallel across the groups (each group runs
    its share of the batch) when the batch divides."""
    from oracle import blocks as OB  # shapes and flop counts only
    res = []
    for name, cfg, batch in (("gemma_block", OB.gemma_config(), 4), ("dit_block", OB.dit_config(), 2)):
        layouts = [world]
        dp = max(d for d in range(1, world + 1) if world % d == 0 and batch % d == 0 and world // d >= 2)
        if dp > 1:
            layouts.append(world // dp)
        for tp_size in layouts:
            r = _block_group_measure(rt, torch, dist, rank, world, stream, iters, name, cfg, batch, tp_size)
            if r is not None:
                res.append(r)
    return res


def _block_group_measure(rt, torch, dist, rank, world, stream, iters, name, cfg, batch, tp_size):
    from oct_b200 import reactor as R
    from oct_b200 import tp
    from oracle import blocks as OB
    if cfg.heads % tp_size or cfg.ffn % tp_size:
        return None
    pk, _ = peaks()
    peak = pk["bf16_tflops"] / 6.0  # burst 3xTF32-adjusted peak
    dp = world // tp_size
    group, tp_rank = rank // tp_size, rank % tp_size
    local_batch = batch // dp
    rcfg = tp.rank_config(cfg, tp_rank, tp_size)
    fam = R.BLOCK_GEMMA if cfg.family == OB.GEMMA else R.BLOCK_DIT
    # one NCCL unique id seeds exactly one communicator: a fresh id per group and block
    ids = [[R.nccl_unique_id(rt.lib) for _ in range(dp)] if rank == 0 else None]
    dist.broadcast_object_list(ids, src=0)
    blk = rt.block(fam, hidden=rcfg.hidden, heads=rcfg.heads, kv_heads=rcfg.kv_heads, head_dim=rcfg.head_dim,
                   ffn=rcfg.ffn, seq_len=rcfg.seq_len, max_batch=local_batch, eps=rcfg.eps, rope_base=rcfg.rope_base,
                   grid_w=rcfg.grid_w, rope_frame=rcfg.rope_frame, tp_rank=tp_rank, tp_world=tp_size,
                   nccl_id=ids[0][group] if tp_size > 1 else b"")
    # one full weight set (same seed on every rank), sharded for this rank
    g = torch.Generator(device="cuda").manual_seed(99)
    full = {}
    for wname, shape in OB.weight_shapes(cfg).items():
        t = torch.randn(*shape, device="cuda", generator=g)
        full[wname] = (t * 0.02 + 1.0) if len(shape) == 1 and wname != "ada_b" else t * 0.02
    shard = (tp.shard_weights(cfg.family, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, full, tp_rank,
                              tp_size) if tp_size > 1 else full)
    blk.set_weights(shard)
    del shard
    T_local = local_batch * cfg.seq_len
    x = torch.randn(T_local, cfg.hidden, device="cuda", generator=torch.Generator(device="cuda").manual_seed(7 + group))
    y = torch.empty_like(x)
    ts = ([500.0, 250.0][group * local_batch:(group + 1) * local_batch] if cfg.family == OB.DIT else None)
    for _ in range(2):
        blk.forward_device(x, y, local_batch, ts, stream)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(iters):
        blk.forward_device(x, y, local_batch, ts, stream)
    e1.record(stream)
    e1.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / iters], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    T = batch * cfg.seq_len
    flops = OB.flops_per_forward(cfg, batch)
    label = f"{name}_tp{tp_size}" if dp == 1 else f"{name}_tp{tp_size}_dp{dp}"
    blk.close()
    # parity of this layout at the benchmark configuration: each group's leader runs the
    # same items through one GPU with the full weights (outside the timed region)
    err = 0.0
    if tp_rank == 0:
        one = rt.block(fam, hidden=cfg.hidden, heads=cfg.heads, kv_heads=cfg.kv_heads, head_dim=cfg.head_dim,
                       ffn=cfg.ffn, seq_len=cfg.seq_len, max_batch=local_batch, eps=cfg.eps, rope_base=cfg.rope_base,
                       grid_w=cfg.grid_w, rope_frame=cfg.rope_frame)
        one.set_weights(full)
        y1 = torch.empty_like(x)
        one.forward_device(x, y1, local_batch, ts, stream)
        torch.cuda.synchronize()
        one.close()
        err = float((y - y1).abs().max() / y1.abs().max())
        del y1
    te = torch.tensor([err], dtype=torch.float64)
    dist.all_reduce(te, op=dist.ReduceOp.MAX)
    small = _tp_small_parity(rt, torch, dist, rank, world, cfg.family, tp_size)
    parity = {"vs_1gpu_normwise": float(te.item()), "oracle_small_normwise": small,
              "ok": bool(te.item() <= 1e-4 and small <= 1e-4)}
    if not parity["ok"]:
        raise RuntimeError(f"tensor-parallel parity failed for {label}: {parity}")
    del x, y, full
    torch.cuda.empty_cache()
    return {"kernel": label, "tp": tp_size, "dp": dp, "batch": batch, "seq": cfg.seq_len, "ms": round(ms, 3),
            "tokens/s": round(T / (ms * 1e-3), 1), "TFLOP/s": round(flops / (ms * 1e-3) / 1e12, 2),
            "frac_of_3xtf32_peak_all_gpus": round(flops / (ms * 1e-3) / 1e12 / (peak * world), 3),
            "parity": parity}


def _tp_small_parity(rt, torch, dist, rank, world, family, tp_size) -> float:
    """One tensor-parallel layout at a small configuration against the binary64 oracle
    (oracle/blocks.py, the checker): max normwise error over every rank."""
    from oct_b200 import reactor as R
    from oct_b200 import tp
    from oracle import blocks as OB
    dp = world // tp_size
    group, tp_rank = rank // tp_size, rank % tp_size
    if family == OB.GEMMA:
        cfg, ts = OB.gemma_config(seq_len=128, hidden=1024, heads=8, head_dim=128, ffn=2048), None
    else:
        cfg, ts = OB.dit_config(seq_len=256, hidden=1024, heads=8, ffn=2048, grid_w=16), [300.0 + 50.0 * group]
    w = OB.random_weights(cfg, seed=41)
    x = np.random.default_rng(42 + group).standard_normal((cfg.seq_len, cfg.hidden)).astype(np.float32)
    ids = [[R.nccl_unique_id(rt.lib) for _ in range(dp)] if rank == 0 else None]
    dist.broadcast_object_list(ids, src=0)
    shard = (tp.shard_weights(cfg.family, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, w, tp_rank,
                              tp_size) if tp_size > 1 else w)
    rcfg = tp.rank_config(cfg, tp_rank, tp_size)
    fam = R.BLOCK_GEMMA if family == OB.GEMMA else R.BLOCK_DIT
    blk = rt.block(fam, hidden=rcfg.hidden, heads=rcfg.heads, kv_heads=rcfg.kv_heads, head_dim=rcfg.head_dim,
                   ffn=rcfg.ffn, seq_len=rcfg.seq_len, max_batch=1, eps=rcfg.eps, rope_base=rcfg.rope_base,
                   grid_w=rcfg.grid_w, rope_frame=rcfg.rope_frame, tp_rank=tp_rank, tp_world=tp_size,
                   nccl_id=ids[0][group] if tp_size > 1 else b"")
    blk.set_weights(shard)
    y = blk.forward(x, 1, ts)
    blk.close()
    ref = OB.forward(cfg, w, x, ts)
    t = torch.tensor([float(np.max(np.abs(y - ref)) / np.max(np.abs(ref)))], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_ours(args) -> None:
    import torch
    from oct_b200 import reactor as R

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        # Control plane only (barriers, the max-over-ranks time, the NCCL id
        # broadcast) runs over gloo; the data-path collectives of the
        # tensor-parallel block use the library's own NCCL communicator over NVLink.
        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=timedelta(seconds=180))
    rt = R.Runtime()
    m, n, k = args.m, args.n, args.k
    stream = torch.cuda.current_stream()
    g = torch.Generator(device="cuda").manual_seed(1234 + rank)
    a = torch.rand(m, k, device="cuda", generator=g) * 2 - 1
    b = torch.rand(k, n, device="cuda", generator=g) * 2 - 1
    c = torch.empty(m, n, device="cuda")
    flops = 2.0 * m * n * k

    def step():
        rt.sgemm_device(a, b, c, m, n, k, args.variant, stream)

    # the kernel AUTO runs for this shape (the library's resolve_variant: m > 16 and
    # m*n*k >= 4e6 here; CTA pair with 32-deep stages from 2048 x 2048 up)
    kid = args.variant
    if kid == 0:
        kid = 232 if (m >= 2048 and n >= 2048) else 16

    for _ in range(max(3, args.warmup)):
        step()
    st = rt.sync_status(stream)
    if not st.ok:
        raise RuntimeError(f"warm-up failed: {st}")

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    rt.set_kernel_timing(True)
    rt.read_kernel_timing()  # reset the launch count
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with ClockSampler(nvidia_smi_selector(torch.cuda.get_device_properties(local))) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        barrier()
    ms_total = e0.elapsed_time(e1)
    split_ms, main_ms, launches = rt.read_kernel_timing()
    rt.set_kernel_timing(False)
    st = rt.sync_status(stream)
    if not st.ok:
        raise RuntimeError(f"timed run failed: {st}")
    t = torch.tensor([ms_total], dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    value = flops * world * args.steps / (ms_max * 1e-3) / 1e12

    pk, pk_kind = peaks()
    clock_rec = clocks.summary()
    tensor_peak, peak_note = tensor_roofline_peak(pk, pk_kind, clock_rec)
    tensor_peak_burst = pk["bf16_tflops"] / 6.0
    tensor_peak_sustained = pk.get("bf16_tflops_sustained", pk["bf16_tflops"]) / 6.0
    # The FMA control records no per-kernel events: its whole step is the kernel.
    main_per_launch_ms = main_ms / launches if launches > 0 and main_ms > 0 else ms_max / args.steps
    achieved = flops / (main_per_launch_ms * 1e-3) / 1e12
    traffic = None
    tpath = REPO / "profiles" / "traffic.json"
    if tpath.exists():
        try:
            key = "sgemm3x_pair_kernel_8192" if kid in (216, 232) else "sgemm3x_kernel_8192"
            entry = json.loads(tpath.read_text()).get(key)
            if entry is not None:
                traffic = entry.get("bytes_per_launch")
        except Exception:
            traffic = None

    # ---- end to end through the reference-facing host ABI (pinned buffers)
    e2e = None
    if not args.no_e2e:
        ha = torch.empty(m * k, dtype=torch.float32, pin_memory=True)
        hb = torch.empty(k * n, dtype=torch.float32, pin_memory=True)
        hc = torch.empty(m * n, dtype=torch.float32, pin_memory=True)
        ha.copy_(a.reshape(-1).cpu())
        hb.copy_(b.reshape(-1).cpu())
        na, nb, nc = ha.numpy(), hb.numpy(), hc.numpy()
        for _ in range(max(3, args.warmup // 2)):
            _, s = rt.sgemm_with_status(m, n, k, na, nb, out=nc)
            if not s.ok:
                raise RuntimeError(f"e2e warm-up failed {s}")
        barrier()
        t0 = time.perf_counter()
        e2e_steps = max(3, min(args.steps, 10))
        for _ in range(e2e_steps):
            _, s = rt.sgemm_with_status(m, n, k, na, nb, out=nc)
            if not s.ok:
                raise RuntimeError(f"e2e step failed {s}")
        tt = torch.tensor([time.perf_counter() - t0], dtype=torch.float64)
        if dist is not None:
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e = {"value": flops * world * e2e_steps / float(tt.item()) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": 4 * (m * k + k * n) * world, "d2h_bytes_per_step": 4 * m * n * world,
               "steps": e2e_steps, "path": "prometheus_reactor_runtime_sgemm, pinned host buffers"}

    secondary = None
    cpu = None
    if world > 1 and not args.no_secondary:
        secondary = sharded_sgemm_measurements(rt, torch, dist, rank, world, stream)
        secondary += tp_block_measurements(rt, torch, dist, rank, world, stream)
    if rank == 0 and world == 1:
        if not args.no_secondary:
            secondary = secondary_measurements(rt, torch, pk["hbm_gbs"])
        if not args.no_cpu_baseline:
            from oracle import oracle as O
            O.build()
            cpu = cpu_sgemm_sample(m, n, k, args.cpu_seconds, O.max_threads())
            cpu.pop("seconds", None)
            cpu.pop("rows", None)
            cpu["reference_paths"] = cpu_baseline_table(O.max_threads())

    if rank == 0:
        line = {
            "metric": "fp32 SGEMM TFLOP/s at 8192^3",
            "value": value,
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": max(3, args.warmup),
            "ms_per_step": ms_max / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic",
            "config": {
                "workload": (f"sgemm {m}x{n}x{k} per rank: independent products, A and B seeded per rank, no data "
                             "exchange (weak scaling); the column-parallel product with replicated A and the "
                             "gathered C is the sgemm_tp secondary lines (strong scaling)"),
                "m": m, "n_per_rank": n, "k": k,
                "variant_id": args.variant, "kernel_id": kid,
                "variant": ("tcgen05 3xTF32" + (" CTA pair" if kid in (216, 232, 316, 332) else "")
                            + (", TF32 split inside the kernel" if kid in (316, 332) else ", split pass"))
                if kid in (1, 16, 32, 216, 232, 316, 332) else "fp32 FMA",
                "stage_depth_k": kid % 100 if kid in (16, 32, 216, 232, 316, 332) else None,
                "parallelism": f"independent replicas x{world}",
                "l2": "no flush: every operand (256 MiB) exceeds the 126 MB L2",
                "input": "U[-1,1) fp32, seeded per rank",
            },
            "roofline": {
                "bound": "tensor",
                "kernel": ("sgemm3x_insm_kernel" if kid in (316, 332) else
                           "sgemm3x_pair_kernel" if kid in (216, 232) else "sgemm3x_kernel")
                          + " (tcgen05 kind::tf32, 3 products per k-step)",
                "achieved": achieved,
                "peak": tensor_peak,
                "unit": "TFLOP/s",
                "frac": achieved / tensor_peak,
                "traffic": traffic,
                "peak_source": peak_note,
                "frac_of_burst_peak": achieved / tensor_peak_burst,
                "burst_peak": tensor_peak_burst,
                "frac_of_sustained_peak": achieved / tensor_peak_sustained,
                "sustained_peak": tensor_peak_sustained,
                "frac_of_clock_scaled_peak": achieved / clock_scaled_peak(pk, clock_rec),
                "algorithmic_flops_per_launch": flops,
                "main_kernel_ms_per_launch": main_per_launch_ms,
                "split_pass_ms_per_launch": split_ms / max(1, launches),
            },
            "e2e": e2e,
            "cpu_baseline": cpu,
            # FMA and the in-kernel split: one kernel per step; the others: 2 split passes + main
            "gpu_launches": (1 if kid in (2, 316, 332) else 3) * args.steps,
            "clocks": clock_rec,
            "secondary": secondary,
        }
        print(json.dumps(line), flush=True)
    rt.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_single_workload(args) -> None:
    """One secondary measurement alone, e.g. under ncu; prints it as JSON."""
    import torch
    from oct_b200 import reactor as R
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    rt = R.Runtime()
    pk, _ = peaks()
    if args.workload == "reductions":
        res = reduction_measurements(rt, torch, pk["hbm_gbs"])
    elif args.workload == "smallm":
        res = smallm_measurements(rt, torch, torch.cuda.current_stream(), pk["hbm_gbs"])
    elif args.workload == "attention":
        res = attention_measurements(rt, torch, torch.cuda.current_stream(), iters=max(1, args.steps))
    else:
        res = block_measurements(rt, torch, torch.cuda.current_stream(), iters=max(1, args.steps), only=args.workload)
    print(json.dumps({"workload": args.workload, "results": res}), flush=True)
    rt.close()


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload != "sgemm":
        run_single_workload(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
