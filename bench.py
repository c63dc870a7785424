"""Benchmark: inferences/s of the five workload graphs through the B200 launch plan.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME | --workloads a,b,...]

One step = one inference = one invocation of a workload graph at its full
batch.  The printed JSON line is the headline workload (the int8 ResNet-style
stack, X uint8 [32,64,56,56], 4 x QLinearConv 3x3 64->64 + 2 x QLinearAdd);
its ``per_workload`` key holds the same measurement for every other workload
(fp32 MLP, int4 Llama MLP, fp16 causal attention in both modes, fp32 LSTM).

Under torchrun every rank runs its own independent inferences on its own GPU
with a full weight replica (weak scaling, no collective on the data path);
the reported time is the max over ranks.  With N > 1 each workload also gets a
``strong`` entry: ONE inference split along its batch dimension over the N
GPUs (each rank runs the same graph at batch/N), and a ``copy_ceiling``: the
same host<->device copies as the e2e step, all ranks at once, no kernels.

* ``value``  -- inputs/outputs resident in HBM, device time per step from CUDA
  events on the launching stream, L2 flushed (256 MiB write) between timed
  steps outside the event windows, max over ranks.
* ``e2e``    -- the same step through the C-ABI with pinned HOST buffers:
  host->device input copy, the plan, device->host output copy, all inside the
  timed region.  K steps are issued back to back in the library's
  overlapped-runs mode (step k+1's upload and step k-1's download overlap step
  k's kernels), timed from an event before the first step to an event after
  the last download (emx_b200_join), / K; the L2 is flushed once before that
  window, not inside it.
* ``roofline`` -- the dominant kernel's algorithmic work per launch / its mean
  CUDA-event duration (per-op events inside the library, chain members that
  launch nothing excluded), against the measured peaks.
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
HEADLINE = "qconv_stack_int8"
ALL_WORKLOADS = ("qconv_stack_int8", "llama_mlp_int4", "mlp_fp32", "attention_fp16", "attention_fp16_tc", "lstm_fp32")


# ----------------------------------------------------------------------------- workloads
def workload_spec(name: str, shard: int = 1):
    """(workload, per-launch algorithmic model of the dominant kernel, plan emitter options).

    ``shard`` > 1 builds the same graph at 1/shard of its batch dimension (the
    slice one rank runs when one inference is split over ``shard`` GPUs)."""
    from emx_onnx_cgen_b200 import workloads as W
    if name == "qconv_stack_int8":
        wl = W.qconv_stack_int8(batch=32 // shard)
        p = wl.params
        n, c, h, w = p["batch"], p["channels"], p["height"], p["width"]
        ops_per_conv = 2 * n * h * w * c * c * 9
        act = n * c * h * w
        # activation in + out per conv, residual read for the 2 fused adds, weights
        bytes_all = 4 * (2 * act + c * c * 9) + 2 * act
        dom = {"kernel": "qconv_tc", "ops_total": 4 * ops_per_conv, "bytes_total": bytes_all,
               "engine": "int8", "unit_ops": "TOP/s", "dtype": "u8/s8 -> s32",
               "ref_tag": "ref_qconv_b1", "ref_rows": 1, "full_rows": n}
        return wl, dom, {}
    if name == "llama_mlp_int4":
        wl = W.llama_mlp_int4(m=2048 // shard)
        p = wl.params
        m, h, f, bs = p["m"], p["hidden"], p["inter"], p["block"]
        flops = 3 * 2 * m * h * f  # gate, up, down
        w_bytes = 3 * h * f // 2 + 3 * f * (h // bs) * 2  # int4 weights + fp16 scales
        # A read (by the fused gate/up launch), P written and read back, Y written
        act_bytes = 2 * (m * h + 2 * m * f + m * h)
        dom = {"kernel": "nbits_gemm", "ops_total": flops, "bytes_total": w_bytes + act_bytes,
               "engine": "f16", "unit_ops": "TFLOP/s", "dtype": "f16 x int4 -> f32 acc -> f16",
               "ref_tag": "ref_nbits_m1", "ref_rows": 1, "full_rows": m}
        return wl, dom, {}
    if name == "mlp_fp32":
        wl = W.mlp_fp32(m=64 // shard)
        p = wl.params
        m, k, h = p["m"], p["k"], p["hidden"]
        flops = 2 * m * k * h * 2
        byts = 4 * (2 * k * h + m * k + m * k + k + h)
        dom = {"kernel": "gemm_f32", "ops_total": flops, "bytes_total": byts, "engine": "fp32",
               "unit_ops": "TFLOP/s", "dtype": "f32 (reference accumulation order)", "ref_tag": "ref_mlp_m64",
               "ref_rows": 64, "full_rows": m}
        return wl, dom, {}
    if name in ("attention_fp16", "attention_fp16_tc"):
        wl = W.attention_fp16(batch=8 // shard)
        p = wl.params
        b, h, t, d = p["batch"], p["heads"], p["seq"], p["head_dim"]
        flops = 2 * (2 * b * h * t * t * d) // 2  # causal: QK^T and PV over the unmasked half
        byts = 4 * b * h * t * d * 2
        tc = name.endswith("_tc")
        dom = {"kernel": "attention_tc" if tc else "attention_f16", "ops_total": flops, "bytes_total": byts,
               "engine": "f16", "unit_ops": "TFLOP/s",
               "dtype": ("f16 in, tcgen05 f16 MMAs, f32 accumulation and online softmax" if tc
                         else "f16 (reference statement rounding)"),
               "ref_tag": "ref_attn_b1h1", "ref_rows": 1, "full_rows": b * h}
        return wl, dom, ({"attention_mode": "tensor"} if tc else {})
    if name == "lstm_fp32":
        wl = W.lstm_fp32(batch=256 // shard)
        p = wl.params
        t, b, i, h = p["seq"], p["batch"], p["input_size"], p["hidden"]
        flops = 2 * t * b * 4 * h * (i + h)
        byts = 4 * (t * b * i + t * b * h + 4 * h * (i + h) + 2 * b * h)
        dom = {"kernel": "lstm_f32", "ops_total": flops, "bytes_total": byts, "engine": "fp32",
               "unit_ops": "TFLOP/s", "dtype": "f32", "ref_tag": "ref_lstm_b1", "ref_rows": 1, "full_rows": b}
        return wl, dom, {}
    raise SystemExit(f"unknown workload {name}")


# ----------------------------------------------------------------------------- peaks
def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def _best_ms(torch, fn, reps: int = 10) -> float:
    best = 1e30
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        best = min(best, e0.elapsed_time(e1))
    return best


def measure_fp32_peak(torch) -> float:
    """fp32 CUDA-core throughput of cuBLAS SGEMM (TF32 off), best of 10, TFLOP/s."""
    n = 8192
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    a = torch.randn(n, n, device="cuda")
    b = torch.randn(n, n, device="cuda")
    for _ in range(2):
        a @ b
    best = _best_ms(torch, lambda: a @ b)
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
    best = _best_ms(torch, lambda: torch._int_mm(a, b))
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
    releases the GIL for the duration of each call.  At least one step runs,
    however long it takes."""
    from oracle.refc import RefCModel
    from emx_onnx_cgen_b200 import workloads as W
    idx = json.loads((ROOT / "oracle" / "_ref" / "index.json").read_text())[dom["ref_tag"]]
    model = RefCModel(dom["ref_tag"])
    wl = W.BUILDERS[idx["builder"]](**idx["kwargs"])
    cores = len(os.sched_getaffinity(0))
    # one slice per thread; a slice that is a whole inference (the MLP) runs once per thread
    threads = max(1, threads or cores)
    if dom["ref_rows"] < dom["full_rows"]:
        threads = min(threads, dom["full_rows"] // dom["ref_rows"])
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


def single_thread_baseline(dom: dict, seconds: float = 5.0) -> dict:
    """The generated C single-threaded on a bounded sample (at least one row-slice)."""
    times, rows, _ = cpu_reference_sample(dom, seconds, threads=1)
    sec = sum(times) / len(times)
    return {"value": rows / dom["full_rows"] / sec, "unit": "inferences/s", "cores": 1,
            "sample": f"{len(times)} steps x {rows} of {dom['full_rows']} batch rows, one thread"}


def cpu_baseline(dom: dict, seconds: float) -> dict:
    times, rows, threads = cpu_reference_sample(dom, seconds=seconds)
    sec = sum(times) / len(times)
    out = {"value": rows / dom["full_rows"] / sec, "unit": "inferences/s", "cores": threads,
           "kind": "reference",
           "sample": f"{len(times)} steps x {rows} of {dom['full_rows']} batch rows, reference generated C "
                     f"(gcc -std=c99 -O2), one row-slice per thread"}
    if min(times) * threads <= 4 * seconds:
        out["single_thread"] = single_thread_baseline(dom, seconds=seconds / 2)
    else:
        # one slice alone would outlast the sample budget: report the per-thread rate of
        # the parallel run (each thread ran one whole slice on its own core)
        out["single_thread"] = {"value": out["value"] / threads, "unit": "inferences/s", "cores": 1,
                                "sample": "per-thread rate of the parallel run above (one slice per core)"}
    return out


# ----------------------------------------------------------------------------- arms
def reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    names = _workload_list(args)
    lines = {}
    for name in names:
        if name.endswith("_tc"):
            continue  # the reference has one attention; its line is attention_fp16's
        wl, dom, _ = workload_spec(name)
        # one step = one row-slice per host thread; the run stops after K steps or the
        # sample budget, whichever comes first (the line reports the steps run)
        budget = 60.0 if name == HEADLINE else 20.0
        times, rows, threads = cpu_reference_sample(dom, budget, steps=args.steps,
                                                    warmup=min(args.warmup, 1) if name == HEADLINE else 0)
        sec = sum(times) / len(times)
        value = rows / dom["full_rows"] / sec
        lines[name] = {
            "impl": "reference", "metric": "inferences/s", "value": value, "unit": "inferences/s",
            "n_gpus": args.gpus, "steps": len(times), "warmup": args.warmup, "ms_per_step": sec * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dom["dtype"],
            "data": "synthetic", "config": {"workload": name, **_config(wl)},
            "cpu_baseline": {"value": value, "unit": "inferences/s", "cores": threads, "kind": "reference",
                             "sample": f"{rows} of {dom['full_rows']} batch rows per step, reference generated "
                                       f"C (gcc -std=c99 -O2), one row-slice per thread"},
            "e2e": {"value": value, "unit": "inferences/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
    head = names[0] if names[0] in lines else next(iter(lines))
    line = dict(lines[head])
    others = {k: v for k, v in lines.items() if k != head}
    if others:
        line["per_workload"] = others
    print(json.dumps(line), flush=True)


def _config(wl) -> dict:
    cfg = {k: (list(v) if isinstance(v, tuple) else v) for k, v in wl.params.items()}
    cfg["parallelism"] = "replicas (batch of independent inferences per GPU)"
    cfg["l2"] = "flushed (256 MiB write) between timed device steps, outside the event windows"
    return cfg


class Ctx:
    """Per-process GPU context shared by the workload measurements."""

    def __init__(self, args):
        import torch
        import torch.distributed as dist
        self.torch, self.dist, self.args = torch, dist, args
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        # under torchrun: this rank's host threads and page-locked buffers on
        # its GPU's NUMA node (first touch), next to that GPU's PCIe root
        self.host_binding = None
        if self.world > 1:
            from emx_onnx_cgen_b200.distributed import bind_host_to_gpu
            try:
                self.host_binding = bind_host_to_gpu(self.local)
            except Exception as exc:  # placement is an optimisation, never a reason to stop
                self.host_binding = {"numa_node": None, "error": str(exc)[:120]}
        if self.world > 1:
            from datetime import timedelta
            dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                    device_id=torch.device("cuda", self.local))
        # a real (non-legacy) stream: its handle is what the library launches on and
        # what the timing events are recorded on
        self.stream = torch.cuda.Stream()
        torch.cuda.set_stream(self.stream)
        self.sptr = self.stream.cuda_stream
        assert self.sptr != 0
        self.flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
        self.peaks = measured_peaks()
        self.engine_peaks = {}

    def barrier(self):
        self.torch.cuda.synchronize()
        if self.world > 1:
            self.dist.barrier()

    def max_over_ranks(self, v: float) -> float:
        from emx_onnx_cgen_b200.distributed import max_over_ranks
        return max_over_ranks(v, device="cuda")

    def engine_peak(self, engine: str):
        """Measured engine peak (rank 0 measures; every rank gets the value)."""
        if engine in self.engine_peaks:
            return self.engine_peaks[engine]
        torch = self.torch
        if engine == "int8":
            v = measure_int8_peak(torch)
            src = "int8 dense, cuBLASLt torch._int_mm 8192^3 best of 10, measured in this run"
        elif engine == "fp32":
            v = measure_fp32_peak(torch)
            src = "fp32 CUDA cores, cuBLAS SGEMM (TF32 off) 8192^3 best of 10, measured in this run"
        else:
            v = self.peaks["bf16_tflops"]
            src = f"dense bf16 (= fp16 rate) burst, MEASURED_PEAKS.json ({self.peaks['source']})"
        # every rank measured its own GPU; the roof is the best of them
        if self.world > 1:
            v = self.max_over_ranks(v)
        self.engine_peaks[engine] = (v, src)
        return v, src


def run_workload(ctx: Ctx, name: str, shard: int = 1) -> dict:
    """Measure one workload on this rank (max over ranks applied); returns its line."""
    torch, args = ctx.torch, ctx.args
    from emx_onnx_cgen_b200 import lowering, kernel_ids as K
    from emx_onnx_cgen_b200.plan import B200PlanEmitter, NP
    from emx_onnx_cgen_b200.runtime import Session
    from emx_onnx_cgen_b200.distributed import check_same_plan

    wl, dom, emit_opts = workload_spec(name, shard)
    plan = B200PlanEmitter(**emit_opts).emit_plan(lowering.lower(wl.graph))
    if not check_same_plan(plan.plan_bytes, plan.weight_bytes, device="cuda"):
        raise SystemExit("ranks emitted different plans")
    sess = Session(plan, device=ctx.local)
    stream, sptr, flush = ctx.stream, ctx.sptr, ctx.flush

    x_np = wl.make_inputs(ctx.rank)
    host_in = [torch.from_numpy(np.ascontiguousarray(x_np[n])).pin_memory() for n in plan.input_names]
    del x_np
    dev_in = [t.to("cuda") for t in host_in]
    dev_out = [torch.empty(s, dtype=getattr(torch, np.dtype(NP[d]).name), device="cuda")
               for s, d in zip(plan.output_shapes, plan.output_dtypes)]
    host_out = [torch.empty_like(t, device="cpu").pin_memory() for t in dev_out]
    h2d = sum(t.numel() * t.element_size() for t in host_in)
    d2h = sum(t.numel() * t.element_size() for t in host_out)
    in_d, out_d = [t.data_ptr() for t in dev_in], [t.data_ptr() for t in dev_out]
    in_h, out_h = [t.data_ptr() for t in host_in], [t.data_ptr() for t in host_out]

    def timed(ins, outs, steps, flush_between=True):
        ev = []
        for _ in range(steps):
            if flush_between:
                flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            sess.run_ptrs(ins, outs, stream=sptr)
            e1.record(stream)
            ev.append((e0, e1))
        torch.cuda.synchronize()
        sess.sync()
        return sum(a.elapsed_time(b) for a, b in ev) / steps

    def timed_overlap(ins, outs, steps):
        # K steps back to back; the stream waits for the last download before e1
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            sess.run_ptrs(ins, outs, stream=sptr)
        sess.join(sptr)
        e1.record(stream)
        torch.cuda.synchronize()
        sess.sync()
        return e0.elapsed_time(e1) / steps

    with ClockSampler(ctx.local) as clk:
        # warm-up: at least W steps and at least ~1 s of back-to-back work so the
        # SM clock has ramped before the timed region
        t0 = time.perf_counter()
        done = 0
        while done < args.warmup or time.perf_counter() - t0 < 1.0:
            flush.fill_(3)
            sess.run_ptrs(in_d, out_d, stream=sptr)
            sess.run_ptrs(in_h, out_h, stream=sptr)
            done += 1
            if done % 4 == 0:
                sess.sync()
        sess.sync()
        launches_before = sess.launch_count()
        ctx.barrier()
        ms = timed(in_d, out_d, args.steps)
        launches = sess.launch_count() - launches_before
    ctx.barrier()
    # every step crosses the bus in both directions: the serving mode overlaps them
    overlap = h2d + d2h > 0
    if overlap:
        sess.set_host_io_overlap(True)
        for _ in range(max(4, args.warmup)):  # both staging sets' graphs
            sess.run_ptrs(in_h, out_h, stream=sptr)
        sess.join(sptr)
        torch.cuda.synchronize()
        sess.sync()
        ctx.barrier()
        ms_e2e = timed_overlap(in_h, out_h, args.steps)
        sess.set_host_io_overlap(False)
    else:
        ms_e2e = timed(in_h, out_h, args.steps, flush_between=False)
    ctx.barrier()
    ms_copy = copy_ceiling_ms(ctx, host_in, dev_in, host_out, dev_out, args.steps) if ctx.world > 1 else None
    ms = ctx.max_over_ranks(ms)
    ms_e2e = ctx.max_over_ranks(ms_e2e)
    if ms_copy is not None:
        ms_copy = ctx.max_over_ranks(ms_copy)

    # per-kernel durations from the library's per-op events (outside the timed region)
    sess.set_profiling(True)
    for _ in range(max(3, min(args.steps, 20))):
        flush.fill_(2)
        sess.run_ptrs(in_d, out_d, stream=sptr)
        sess.sync()
    op_ms, runs = sess.op_times()
    sess.set_profiling(False)
    # chained convolutions run as one launch timed on the chain's first op; chain
    # members (QC_CHAIN < 0) launch nothing and their empty event windows are skipped
    dom_ms = [t / runs for t, op in zip(op_ms, plan.ops)
              if K.NAMES[op.kernel] == dom["kernel"]
              and not (op.kernel == K.K_QCONV_TC and op.ip.get(K.QC_CHAIN, 0) < 0)]
    dom_total_ms = sum(dom_ms)
    peaks = ctx.peaks
    eng_peak, eng_src = ctx.engine_peak(dom["engine"])
    achieved_ops = dom["ops_total"] / (dom_total_ms * 1e-3) / 1e12
    achieved_bw = dom["bytes_total"] / (dom_total_ms * 1e-3) / 1e9
    t_compute = dom["ops_total"] / (eng_peak * 1e12)
    t_mem = dom["bytes_total"] / (peaks["hbm_gbs"] * 1e9)
    # attainable = min(engine peak, AI x HBM peak); frac = achieved work rate / attainable
    attainable_ops = min(eng_peak, dom["ops_total"] / dom["bytes_total"] * peaks["hbm_gbs"] * 1e9 / 1e12)
    if t_compute >= t_mem:
        roof = {"bound": "tensor" if dom["engine"] in ("int8", "f16") else "fp32",
                "achieved": achieved_ops, "peak": eng_peak, "unit": dom["unit_ops"],
                "frac": achieved_ops / attainable_ops, "peak_source": eng_src + " (of measured)"}
    else:
        roof = {"bound": "hbm", "achieved": achieved_bw, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved_bw / peaks["hbm_gbs"],
                "peak_source": f"MEASURED_PEAKS.json ({peaks['source']}) (of measured)"}
    roof.update({"traffic": _ncu_traffic(dom["kernel"], name), "kernel": dom["kernel"],
                 "launches_per_step": len(dom_ms), "launch_ms": dom_total_ms / max(1, len(dom_ms)),
                 "ops_per_launch": dom["ops_total"] / max(1, len(dom_ms)),
                 "bytes_per_launch": dom["bytes_total"] / max(1, len(dom_ms)),
                 "hbm_frac_at_same_time": achieved_bw / peaks["hbm_gbs"],
                 "engine_frac_at_same_time": achieved_ops / eng_peak})

    per = ctx.world if shard == 1 else 1  # weak: N inferences per step; strong: one split over N
    line = {
        "metric": "inferences/s", "value": per * 1000.0 / ms, "unit": "inferences/s", "n_gpus": ctx.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak" if shard == 1 else "strong", "vs_baseline": None, "dtype": dom["dtype"],
        "data": "synthetic", "config": {"workload": name, **_config(wl),
                                        "host_io": ("overlapped runs (two staging sets)" if overlap
                                                    else "one run at a time")},
        "e2e": {"value": per * 1000.0 / ms_e2e, "unit": "inferences/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": ms_e2e,
                "l2": "flushed once before the K back-to-back steps, not between them"},
        "gpu_launches": int(launches), "roofline": roof, "clocks": clk.summary(),
        "per_op_ms": {f"{i}:{K.NAMES[op.kernel]}": t / runs for i, (t, op) in enumerate(zip(op_ms, plan.ops))},
    }
    if shard > 1:
        line["config"]["parallelism"] = f"one inference split along its batch dimension over {shard} GPUs"
    if ctx.host_binding is not None:
        line["config"]["host_numa"] = ctx.host_binding
    if ms_copy is not None:
        line["copy_ceiling"] = {
            "value": per * 1000.0 / ms_copy, "unit": "inferences/s", "ms_per_step": ms_copy,
            "what": "the step's H2D and D2H copies alone (same pinned buffers, two copy streams, all ranks at "
                    "once, max over ranks)",
            "e2e_frac": ms_copy / ms_e2e}
    sess.close()
    del dev_in, dev_out, host_in, host_out
    torch.cuda.empty_cache()
    line["_dom"] = dom
    return line


def copy_ceiling_ms(ctx: Ctx, host_in, dev_in, host_out, dev_out, steps: int) -> float:
    """Per-step time of the e2e step's copies alone: uploads on one stream and
    downloads on another, K steps back to back, every rank at the same time."""
    torch = ctx.torch
    up, down = torch.cuda.Stream(), torch.cuda.Stream()

    def copies(k):
        for _ in range(k):
            with torch.cuda.stream(up):
                for h, d in zip(host_in, dev_in):
                    d.copy_(h, non_blocking=True)
            with torch.cuda.stream(down):
                for h, d in zip(host_out, dev_out):
                    h.copy_(d, non_blocking=True)

    copies(2)
    torch.cuda.synchronize()
    ctx.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ctx.stream)
    up.wait_stream(ctx.stream)
    down.wait_stream(ctx.stream)
    copies(steps)
    ctx.stream.wait_stream(up)
    ctx.stream.wait_stream(down)
    e1.record(ctx.stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def _workload_list(args) -> list[str]:
    if args.workloads:
        return [w for w in args.workloads.split(",") if w]
    if args.workload:
        return [args.workload]
    return list(ALL_WORKLOADS)


def ours_arm(args) -> None:
    ctx = Ctx(args)
    names = _workload_list(args)
    lines = {}
    for name in names:
        lines[name] = run_workload(ctx, name)
        if ctx.world > 1:
            strong = run_workload(ctx, name, shard=ctx.world)
            strong.pop("_dom")
            lines[name]["strong"] = {k: strong[k] for k in ("value", "unit", "ms_per_step", "scaling", "e2e",
                                                           "roofline", "gpu_launches", "config")}
    if ctx.rank == 0 and ctx.world == 1 and not args.no_cpu_baseline:
        for name, line in lines.items():
            if name.endswith("_tc") and name[:-3] in lines and "cpu_baseline" in lines[name[:-3]]:
                line["cpu_baseline"] = lines[name[:-3]]["cpu_baseline"]
                continue
            try:
                line["cpu_baseline"] = cpu_baseline(line["_dom"], seconds=10.0 if name == HEADLINE else 6.0)
            except Exception as exc:  # the GPU number stands without it
                line["cpu_baseline"] = {"value": None, "error": str(exc)[:200]}
    for line in lines.values():
        line.pop("_dom", None)
    if ctx.rank == 0:
        head = names[0]
        out = dict(lines[head])
        others = {k: v for k, v in lines.items() if k != head}
        if others:
            out["per_workload"] = others
        print(json.dumps(out), flush=True)
    if ctx.world > 1:
        ctx.dist.destroy_process_group()


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
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default=None, help="measure one workload only")
    ap.add_argument("--workloads", default=None, help="comma-separated list; the first is the headline line")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        reference_arm(args)
    else:
        ours_arm(args)


if __name__ == "__main__":
    main()
