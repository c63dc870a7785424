"""Benchmark: inferences/s of one workload graph through the B200 launch plan.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

One step = one inference = one invocation of the workload graph at its full
batch (default workload: the int8 ResNet-style stack, X uint8 [32,64,56,56],
4 x QLinearConv 3x3 64->64 + 2 x QLinearAdd).  Under torchrun every rank runs
its own independent inferences on its own GPU with a full weight replica
(weak scaling, no collective on the data path); the reported time is the max
over ranks.

* ``value``  -- inputs/outputs resident in HBM, device time per step from CUDA
  events on the launching stream, L2 flushed (256 MiB write) before every
  timed step, max over ranks.
* ``e2e``    -- the same step through the C-ABI with pinned HOST buffers:
  host->device input copy, the plan, device->host output copy, all inside the
  timed region.  ``--host-io overlap`` (what ``auto``, the default, picks when
  a step moves at least 1 MiB): K steps issued back to back
  with the library's overlapped-runs mode (step k+1's upload and step k-1's
  download overlap step k's kernels), timed from an event before the first
  step to an event after the last step's download (emx_b200_join), / K;
  ``--host-io slices``: each step on its own, its batch cut into slices whose
  copies overlap its kernels, timed step by step.
* ``roofline`` -- the dominant kernel's algorithmic work per launch / its mean
  CUDA-event duration (per-op events inside the library), against the
  measured peaks.
* ``cpu_baseline`` -- the reference's own generated C (``oracle/_ref``, gcc
  -O2) on the host cores (one row-slice per core), rank 0 at N=1 only, on a
  bounded sample; ``single_thread`` inside it: the same C on one core.

``--impl reference`` times that reference C as the whole arm (rank 0 only).
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
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

L2_FLUSH_BYTES = 256 << 20


# ----------------------------------------------------------------------------- workloads
def workload_spec(name: str):
    """(workload, per-launch algorithmic model of the dominant kernel)."""
    from emx_onnx_cgen_b200 import workloads as W
    if name == "qconv_stack_int8":
        wl = W.qconv_stack_int8()
        p = wl.params
        n, c, h, w = p["batch"], p["channels"], p["height"], p["width"]
        ops_per_conv = 2 * n * h * w * c * c * 9
        act = n * c * h * w
        # per conv launch: activation in + out, residual read for the 2 fused adds, weights
        bytes_all = 4 * (2 * act + c * c * 9) + 2 * act
        dom = {"kernel": "qconv_tc", "launches": 4, "ops_total": 4 * ops_per_conv,
               "bytes_total": bytes_all, "engine": "int8", "unit_ops": "TOP/s", "dtype": "u8/s8 -> s32",
               "ref_tag": "ref_qconv_b1", "ref_rows": 1, "full_rows": n}
        return wl, dom
    if name == "llama_mlp_int4":
        wl = W.llama_mlp_int4()
        p = wl.params
        m, h, f, bs = p["m"], p["hidden"], p["inter"], p["block"]
        flops = 3 * 2 * m * h * f  # gate, up, down
        w_bytes = 3 * h * f // 2 + 3 * f * (h // bs) * 2  # int4 weights + fp16 scales
        # A read (by the fused gate/up launch), P written and read back, Y written
        act_bytes = 2 * (m * h + 2 * m * f + m * h)
        dom = {"kernel": "nbits_gemm", "launches": 2, "ops_total": flops, "bytes_total": w_bytes + act_bytes,
               "engine": "f16", "unit_ops": "TFLOP/s", "dtype": "f16 x int4 -> f32 acc -> f16",
               "ref_tag": "ref_nbits_m1", "ref_rows": 1, "full_rows": m}
        return wl, dom
    if name == "mlp_fp32":
        wl = W.mlp_fp32()
        p = wl.params
        m, k, h = p["m"], p["k"], p["hidden"]
        flops = 2 * m * k * h * 2
        byts = 4 * (2 * k * h + m * k + m * k + k + h)
        dom = {"kernel": "gemm_f32", "launches": 2, "ops_total": flops, "bytes_total": byts, "engine": "fp32",
               "unit_ops": "TFLOP/s", "dtype": "f32 (reference accumulation order)", "ref_tag": "ref_mlp_m64",
               "ref_rows": 64, "full_rows": m}
        return wl, dom
    if name == "attention_fp16":
        wl = W.attention_fp16()
        p = wl.params
        b, h, t, d = p["batch"], p["heads"], p["seq"], p["head_dim"]
        flops = 2 * (2 * b * h * t * t * d) // 2  # causal: QK^T and PV over the unmasked half
        byts = 4 * b * h * t * d * 2
        dom = {"kernel": "attention_f16", "launches": 1, "ops_total": flops, "bytes_total": byts, "engine": "f16",
               "unit_ops": "TFLOP/s", "dtype": "f16 (reference statement rounding)", "ref_tag": "ref_attn_b1h1",
               "ref_rows": 1, "full_rows": b * h}
        return wl, dom
    if name == "lstm_fp32":
        wl = W.lstm_fp32()
        p = wl.params
        t, b, i, h = p["seq"], p["batch"], p["input_size"], p["hidden"]
        flops = 2 * t * b * 4 * h * (i + h)
        byts = 4 * (t * b * i + t * b * h + 4 * h * (i + h) + 2 * b * h)
        dom = {"kernel": "lstm_f32", "launches": 1, "ops_total": flops, "bytes_total": byts, "engine": "fp32",
               "unit_ops": "TFLOP/s", "dtype": "f32", "ref_tag": "ref_lstm_b1", "ref_rows": 1, "full_rows": b}
        return wl, dom
    raise SystemExit(f"unknown workload {name}")


# ----------------------------------------------------------------------------- peaks
def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def measure_fp32_peak(torch) -> float:
    """fp32 CUDA-core throughput of cuBLAS SGEMM (TF32 off), best of 10, TFLOP/s."""
    n = 8192
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    a = torch.randn(n, n, device="cuda")
    b = torch.randn(n, n, device="cuda")
    for _ in range(2):
        a @ b
    best = 1e30
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        a @ b
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1))
    torch.backends.cuda.matmul.allow_tf32 = prev
    del a, b
    return 2 * n ** 3 / (best * 1e-3) / 1e12


def measure_int8_peak(torch) -> float:
    """Dense int8 tensor throughput of cuBLASLt (torch._int_mm), best of 10, TOP/s."""
    n = 8192
    a = torch.randint(-127, 127, (n, n), dtype=torch.int8, device="cuda")
    b = torch.randint(-127, 127, (n, n), dtype=torch.int8, device="cuda").t()
    for _ in range(3):
        torch._int_mm(a, b)
    best = 1e30
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1))
    del a, b
    return 2 * n ** 3 / (best * 1e-3) / 1e12


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- CPU reference
def cpu_reference_sample(dom: dict, seconds: float, steps: int | None = None, warmup: int = 0,
                         threads: int | None = None):
    """Run the reference's generated C (oracle/_ref) on all host cores (or on
    ``threads`` of them; 1 = the generated C single-threaded, as emitted).

    Returns (list of per-step seconds, rows per step, threads).  One step runs
    ``threads`` independent row-slices in parallel, one per thread; ctypes
    releases the GIL for the duration of each call."""
    from oracle.refc import RefCModel
    from emx_onnx_cgen_b200 import workloads as W
    import json as _json
    idx = _json.loads((ROOT / "oracle" / "_ref" / "index.json").read_text())[dom["ref_tag"]]
    model = RefCModel(dom["ref_tag"])
    wl = W.BUILDERS[idx["builder"]](**idx["kwargs"])
    cores = len(os.sched_getaffinity(0))
    threads = max(1, min(threads or cores, dom["full_rows"] // dom["ref_rows"]))
    per_thread = [wl.make_inputs(s) for s in range(threads)]
    outs = [None] * threads

    def one(i):
        outs[i] = model.run(per_thread[i])

    def step():
        ts = [threading.Thread(target=one, args=(i,)) for i in range(threads)]
        t0 = time.perf_counter()
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        return time.perf_counter() - t0

    for _ in range(warmup):
        step()
    times = []
    t_start = time.perf_counter()
    while True:
        times.append(step())
        if steps is not None and len(times) >= steps:
            break
        if seconds and time.perf_counter() - t_start >= seconds:
            break
    return times, threads * dom["ref_rows"], threads


# ----------------------------------------------------------------------------- arms
def single_thread_baseline(dom: dict, seconds: float = 6.0) -> dict:
    """The generated C single-threaded on a bounded sample (at least one row-slice)."""
    times, rows, _ = cpu_reference_sample(dom, seconds, threads=1)
    sec = sum(times) / len(times)
    return {"value": rows / dom["full_rows"] / sec, "unit": "inferences/s", "cores": 1,
            "sample": f"{len(times)} steps x {rows} of {dom['full_rows']} batch rows, one thread"}


def reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    wl, dom = workload_spec(args.workload)
    # one step = one row-slice per host thread; the run stops after K steps or
    # ~150 s of CPU time, whichever comes first (the line reports the steps run)
    times, rows, threads = cpu_reference_sample(dom, 150.0, steps=args.steps, warmup=min(args.warmup, 1))
    args.steps = len(times)
    sec = sum(times) / len(times)
    value = rows / dom["full_rows"] / sec
    line = {
        "impl": "reference", "metric": "inferences/s", "value": value, "unit": "inferences/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dom["dtype"],
        "data": "synthetic", "config": {"workload": args.workload, **_config(wl)},
        "cpu_baseline": {"value": value, "unit": "inferences/s", "cores": threads, "kind": "reference",
                         "sample": f"{rows} of {dom['full_rows']} batch rows per step, reference generated C "
                                   f"(gcc -std=c99 -O2), one row-slice per thread",
                         "single_thread": single_thread_baseline(dom)},
        "e2e": {"value": value, "unit": "inferences/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _config(wl) -> dict:
    cfg = {k: (list(v) if isinstance(v, tuple) else v) for k, v in wl.params.items()}
    cfg["parallelism"] = "replicas (batch of independent inferences per GPU)"
    cfg["l2"] = "flushed (256 MiB write) before every timed step"
    return cfg


def ours_arm(args) -> None:
    import torch
    import torch.distributed as dist
    from emx_onnx_cgen_b200 import lowering
    from emx_onnx_cgen_b200.plan import B200PlanEmitter
    from emx_onnx_cgen_b200.runtime import Session

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))

    wl, dom = workload_spec(args.workload)
    plan = B200PlanEmitter().emit_plan(lowering.lower(wl.graph))
    sess = Session(plan, device=local)
    if args.io_chunks is not None:
        sess.set_host_io_chunks(args.io_chunks)
    # a real (non-legacy) stream: its handle is what the library launches on and
    # what the timing events are recorded on
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sptr = stream.cuda_stream
    assert sptr != 0

    x_np = wl.make_inputs(rank)
    host_in = [torch.from_numpy(np.ascontiguousarray(x_np[n])).pin_memory() for n in plan.input_names]
    dev_in = [t.to("cuda") for t in host_in]
    from emx_onnx_cgen_b200.plan import NP
    dev_out = [torch.empty(s, dtype=getattr(torch, np.dtype(NP[d]).name), device="cuda")
               for s, d in zip(plan.output_shapes, plan.output_dtypes)]
    host_out = [torch.empty_like(t, device="cpu").pin_memory() for t in dev_out]
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = sum(t.numel() * t.element_size() for t in host_out)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    in_d, out_d = [t.data_ptr() for t in dev_in], [t.data_ptr() for t in dev_out]
    in_h, out_h = [t.data_ptr() for t in host_in], [t.data_ptr() for t in host_out]

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    def timed_overlap(ins, outs, steps):
        # K steps back to back; the stream waits for the last download before e1
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            flush.fill_(1)
            sess.run_ptrs(ins, outs, stream=sptr)
        sess.join(sptr)
        e1.record(stream)
        torch.cuda.synchronize()
        sess.sync()
        return e0.elapsed_time(e1) / steps

    def timed(ins, outs, steps):
        ev = []
        for _ in range(steps):
            flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            sess.run_ptrs(ins, outs, stream=sptr)
            e1.record(stream)
            ev.append((e0, e1))
        torch.cuda.synchronize()
        sess.sync()
        return sum(a.elapsed_time(b) for a, b in ev) / steps

    from emx_onnx_cgen_b200.distributed import check_same_plan, max_over_ranks as _max_over_ranks

    def max_over_ranks(v: float) -> float:
        return _max_over_ranks(v, device="cuda")

    if not check_same_plan(plan.plan_bytes, plan.weight_bytes, device="cuda"):
        raise SystemExit("ranks emitted different plans")

    with ClockSampler(local) as clk:
        # warm-up: at least W steps and at least ~1 s of back-to-back work so the
        # SM clock has ramped before the timed region
        t0 = time.perf_counter()
        done = 0
        while done < args.warmup or time.perf_counter() - t0 < 1.0:
            flush.fill_(3)
            sess.run_ptrs(in_d, out_d, stream=sptr)
            sess.run_ptrs(in_h, out_h, stream=sptr)
            done += 1
            if done % 16 == 0:
                sess.sync()
        sess.sync()
        launches_before = sess.launch_count()
        barrier()
        ms = timed(in_d, out_d, args.steps)
        launches = sess.launch_count() - launches_before
    barrier()
    host_io = args.host_io
    if host_io == "auto":  # overlapping runs pays when copies are worth hiding (the library's 1 MiB slicing threshold)
        host_io = "overlap" if h2d + d2h >= (1 << 20) else "slices"
    if host_io == "overlap":
        sess.set_host_io_overlap(True)
        for _ in range(max(4, args.warmup)):  # both staging sets' graphs
            flush.fill_(3)
            sess.run_ptrs(in_h, out_h, stream=sptr)
        sess.join(sptr)
        torch.cuda.synchronize()
        sess.sync()
        barrier()
        ms_e2e = timed_overlap(in_h, out_h, args.steps)
        sess.set_host_io_overlap(False)
    else:
        ms_e2e = timed(in_h, out_h, args.steps)
    barrier()
    ms = max_over_ranks(ms)
    ms_e2e = max_over_ranks(ms_e2e)

    # per-kernel durations from the library's per-op events (outside the timed region)
    sess.set_profiling(True)
    for _ in range(max(3, args.steps)):
        flush.fill_(2)
        sess.run_ptrs(in_d, out_d, stream=sptr)
        sess.sync()
    op_ms, runs = sess.op_times()
    sess.set_profiling(False)
    from emx_onnx_cgen_b200 import kernel_ids as K
    dom_ops = [(t / runs, op) for t, op in zip(op_ms, plan.ops) if K.NAMES[op.kernel] == dom["kernel"]]
    dom_total_ms = sum(t for t, _ in dom_ops)
    # chained convolutions run as one launch timed on the chain's first op (members launch nothing)
    dom_ms = [t for t, op in dom_ops if op.ip.get(K.QC_CHAIN, 0) >= 0 or op.kernel != K.K_QCONV_TC]
    launch_ms = dom_total_ms / len(dom_ms)
    peaks = measured_peaks()
    if dom["engine"] == "int8":
        eng_peak = measure_int8_peak(torch) if rank == 0 else None
        eng_src = "int8 dense, cuBLASLt torch._int_mm 8192^3 best of 10, measured in this run"
    elif dom["engine"] == "fp32":
        eng_peak = measure_fp32_peak(torch) if rank == 0 else None
        eng_src = "fp32 CUDA cores, cuBLAS SGEMM (TF32 off) 8192^3 best of 10, measured in this run"
    else:
        eng_peak = peaks["bf16_tflops"]
        eng_src = f"dense bf16 (= fp16 rate) burst, MEASURED_PEAKS.json ({peaks['source']})"
    achieved_ops = dom["ops_total"] / (dom_total_ms * 1e-3) / 1e12
    achieved_bw = dom["bytes_total"] / (dom_total_ms * 1e-3) / 1e9
    t_compute = dom["ops_total"] / (eng_peak * 1e12) if eng_peak else 0
    t_mem = dom["bytes_total"] / (peaks["hbm_gbs"] * 1e9)
    if t_compute >= t_mem:
        roof = {"bound": "tensor", "achieved": achieved_ops, "peak": eng_peak, "unit": dom["unit_ops"],
                "frac": achieved_ops / eng_peak, "peak_source": eng_src}
    else:
        roof = {"bound": "hbm", "achieved": achieved_bw, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved_bw / peaks["hbm_gbs"], "peak_source": f"MEASURED_PEAKS.json ({peaks['source']})"}
    roof.update({"traffic": _ncu_traffic(dom["kernel"], args.workload), "kernel": dom["kernel"],
                 "launches_per_step": len(dom_ms), "launch_ms": launch_ms,
                 "ops_per_launch": dom["ops_total"] / len(dom_ms),
                 "bytes_per_launch": dom["bytes_total"] / len(dom_ms),
                 "hbm_frac_at_same_time": achieved_bw / peaks["hbm_gbs"],
                 "tensor_frac_at_same_time": achieved_ops / eng_peak if eng_peak else None})

    line = {
        "metric": "inferences/s", "value": world * 1000.0 / ms, "unit": "inferences/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": dom["dtype"], "data": "synthetic",
        "config": {"workload": args.workload, **_config(wl),
                   "host_io": ("overlapped runs (two staging sets)" if host_io == "overlap"
                               else f"one run at a time ({args.io_chunks or 4} batch slices when >= 1 MiB moves)")},
        "e2e": {"value": world * 1000.0 / ms_e2e, "unit": "inferences/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": ms_e2e},
        "gpu_launches": int(launches), "roofline": roof, "clocks": clk.summary(),
        "per_op_ms": {f"{i}:{K.NAMES[op.kernel]}": t / runs for i, (t, op) in enumerate(zip(op_ms, plan.ops))},
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            times, rows, threads = cpu_reference_sample(dom, seconds=12.0)
            sec = sum(times) / len(times)
            line["cpu_baseline"] = {
                "value": rows / dom["full_rows"] / sec, "unit": "inferences/s", "cores": threads,
                "kind": "reference",
                "sample": f"{len(times)} steps x {rows} of {dom['full_rows']} batch rows, reference generated C "
                          f"(gcc -std=c99 -O2), one row-slice per thread",
                "single_thread": single_thread_baseline(dom)}
        except Exception as exc:  # the GPU number stands without it
            line["cpu_baseline"] = {"value": None, "error": str(exc)[:200]}
    if rank == 0:
        print(json.dumps(line), flush=True)
    sess.close()
    if world > 1:
        dist.destroy_process_group()


def _ncu_traffic(kernel: str, workload: str):
    """DRAM bytes per launch from the committed ncu summary, if there is one."""
    f = ROOT / "profiles" / f"{kernel}_{workload}.md"
    if not f.exists():
        return None
    for ln in f.read_text().splitlines():
        if ln.startswith("traffic_bytes_per_launch:"):
            try:
                return float(ln.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="qconv_stack_int8")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--host-io", choices=["auto", "overlap", "slices"], default="auto",
                    help="e2e host copies: overlap consecutive steps, or one step at a time (its batch sliced); "
                         "auto: overlap when a step moves >= 1 MiB")
    ap.add_argument("--io-chunks", type=int, default=None,
                    help="batch slices for the e2e run's pipelined host copies (library default 4; 1 = off)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        reference_arm(args)
    else:
        ours_arm(args)


if __name__ == "__main__":
    main()
