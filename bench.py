#!/usr/bin/env python
"""Benchmark: compiled inference of a gawee graph on B200, data parallel over N GPUs.

Default workload (the one the headline metric is quoted on and that fits one
GPU): ResNet-18 fp32, batch 256 of 3x224x224 ~N(0,1), Kaiming-normal conv
weights with BatchNorm folded into the conv bias, graph in the gawee dialect
as the ONNX emitter prints it.  Batch rows are independent, so the job
partitions: every GPU runs its own batch of 256 (seeded per rank), weights
replicated, with no collective on the data path (weak scaling; the process
group only aligns and times the ranks).  `--workload decoder135m` runs the
135M GQA decoder prefill (batch 64 x 512 tokens per GPU) instead.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl gawee|reference]

One JSON line on rank 0:
  value       whole-job images/s (or tokens/s), inputs resident in HBM, device
              time of K forwards (CUDA events on the launch stream, max over ranks)
  e2e         same metric through the C ABI with pinned host buffers: each step
              copies its input in, runs the forward and copies its output back;
              consecutive steps are pipelined (upload, compute and download on
              three streams, two staging buffers each way)
  roofline    tensor-core kernels: algorithmic FLOPs / their device time in an
              eagerly profiled forward, against the measured peaks
  cpu_baseline  the CPU oracle (a C++ port of the reference lowering semantics)
              on a bounded sample on this host, N=1 only
`--impl reference` times that CPU implementation alone (the reference's own
MLIR/LLVM toolchain is not available, so its AOT binary cannot be built).
"""
from __future__ import annotations

import argparse
import atexit
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    # name: (builder(batch), total batch, unit items per batch row, metric, unit)
    "resnet18": ("ResNet-18 fp32 images/s (batch 256, 3x224x224)", "images/s", 256, 1),
    "decoder135m": ("decoder-135M GQA fp32 prefill tokens/s (batch 64 x seq 512)", "tokens/s", 64, 512),
}


def build_graph(workload: str, batch: int):
    from gawee_b200 import synth
    if workload == "resnet18":
        return synth.resnet18(batch)
    return synth.smollm135m(batch, 512)


def full_inputs(workload: str, batch: int, rank: int = 0):
    """Seeded batched inputs of one rank's partition."""
    rng = np.random.default_rng(43 + rank)
    if workload == "resnet18":
        return rng.standard_normal((batch, 3, 224, 224), dtype=np.float32)
    return rng.integers(0, 49152, (batch, 512), dtype=np.int64)


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"bf16": d.get("bf16_tflops"), "hbm": d.get("hbm_gbs"), "source": "measured"}
    return {"bf16": 1590.0, "hbm": 6650.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed regions.

    nvidia-smi is started and its first row awaited before the region opens
    (that row, taken right after the warm-up, is dropped), so a timed region
    of a few hundred milliseconds still gets samples at the 100 ms period."""

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.skip = 0
        self.path = os.path.join("/tmp", f"gawee_clocks_{os.getpid()}.csv")

    def _rows(self):
        try:
            with open(self.path) as f:
                return [ln for ln in f if ln.strip()]
        except OSError:
            return []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=clocks.sm,clocks.max.sm,power.draw,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return self
        atexit.register(self.__exit__, None, None, None)
        t0 = time.perf_counter()
        while not self._rows() and time.perf_counter() - t0 < 10.0 and self.proc.poll() is None:
            time.sleep(0.01)
        self.skip = len(self._rows())
        return self

    def __exit__(self, *a):
        if self.proc:
            proc, self.proc = self.proc, None
            proc.terminate()
            try:
                proc.wait(5)
            except Exception:
                proc.kill()

    def summary(self):
        if not os.path.exists(self.path):
            return None
        rows = []
        for line in self._rows()[self.skip:]:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                rows.append((float(parts[0]), float(parts[1]), parts[3:7]))
            except ValueError:
                continue
        os.remove(self.path)
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "samples": len(rows), "reasons": reasons}


def cpu_baseline(workload: str, seconds_hint: float = 20.0):
    """The oracle on one batch row (1 image / 1 sequence) with every host thread."""
    import oracle
    g = build_graph(workload, 1)
    args = g.make_args()
    o = oracle.Oracle(g.mlir)
    threads = os.cpu_count() or 1
    reps, t_total = 0, 0.0
    while reps == 0 or (t_total < seconds_hint and reps < 8):
        t0 = time.perf_counter()
        o.run(args, threads=threads)
        t_total += time.perf_counter() - t0
        reps += 1
    per_row = t_total / reps
    _, unit, _, items = WORKLOADS[workload]
    return {"value": items / per_row, "unit": unit, "cores": threads, "kind": "port",
            "sample": f"{reps} run(s) of a batch-1 slice ({'1 image' if workload == 'resnet18' else '1 sequence x 512 tokens'}) "
                      f"of the same graph on the C++ oracle, {threads} threads; whole batch extrapolates linearly"}


def run_reference(a):
    """--impl reference: the CPU implementation of the path on this host."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import oracle
    metric, unit, total, items = WORKLOADS[a.workload]
    g = build_graph(a.workload, 1)
    args = g.make_args()
    o = oracle.Oracle(g.mlir)
    threads = os.cpu_count() or 1
    for _ in range(a.warmup):
        o.run(args, threads=threads)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        o.run(args, threads=threads)
    dt = time.perf_counter() - t0
    value = items * a.steps / dt
    sample = (f"each step: a batch-1 slice of the {a.workload} workload on the C++ oracle "
              f"(the reference's lowering semantics; its own MLIR/LLVM AOT toolchain is absent), {threads} threads")
    line = {"metric": metric, "value": value, "unit": unit, "impl": "reference", "n_gpus": a.gpus, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": dt / a.steps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": a.workload, "global_batch": total,
                       "sample_per_step": "a batch-1 slice; throughput extrapolates linearly over the batch"},
            "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="gawee", choices=["gawee", "reference"])
    ap.add_argument("--workload", default="resnet18", choices=list(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=0, help="override the global batch (small profiling runs)")
    a = ap.parse_args()
    if a.impl == "reference":
        return run_reference(a)

    import torch
    import torch.distributed as dist

    from gawee_b200.runtime import Model

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != a.gpus:
        raise SystemExit(f"--gpus {a.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))

    metric, unit, per_gpu, items = WORKLOADS[a.workload]
    if a.batch:
        per_gpu = a.batch
        metric += f" [batch overridden to {a.batch}]"
    total_batch = per_gpu * world
    g = build_graph(a.workload, per_gpu)
    args = g.make_args()
    args[0] = np.ascontiguousarray(full_inputs(a.workload, per_gpu, rank))
    m = Model(g.mlir, device=local)
    m.set_args(args)
    stream = torch.cuda.Stream(local)
    sp = stream.cuda_stream

    out_dt, out_shape = m.output_specs[0]
    out_bytes = int(np.prod(out_shape)) * out_dt.itemsize

    def step():
        m.forward(sp)

    # first forward (eager) + status check, then warm-up (CUDA graph capture on the second)
    step()
    m.synchronize(sp)
    for _ in range(a.warmup):
        step()
    m.synchronize(sp)

    def timed(fn, k):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(local)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(k):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(local)
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=f"cuda:{local}")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    clk = ClockSampler(local).__enter__()
    ms = timed(step, a.steps)
    m.synchronize(sp)
    value = total_batch * items * a.steps / (ms / 1e3)

    # End to end through the C ABI, every step: the step's input from pinned
    # host memory to the GPU, gawee_set_arg_device + gawee_forward, the result
    # back to pinned host memory.  Steps are pipelined the way a serving loop
    # would run them: step i+1's upload (its own stream) overlaps step i's
    # forward and step i's download (another stream) overlaps step i+1's, with
    # two device staging buffers each way and events ordering the hand-offs.
    from cuda.bindings import runtime as cudart
    in_bytes = args[0].nbytes
    h_in = torch.from_numpy(args[0]).pin_memory().view(torch.uint8).reshape(-1)
    h_out = [torch.empty(out_bytes, dtype=torch.uint8).pin_memory() for _ in range(2)]
    dev = f"cuda:{local}"
    d_in = [torch.empty(in_bytes, dtype=torch.uint8, device=dev) for _ in range(2)]
    d_out = [torch.empty(out_bytes, dtype=torch.uint8, device=dev) for _ in range(2)]
    up, down = torch.cuda.Stream(local), torch.cuda.Stream(local)
    in_ready = [torch.cuda.Event() for _ in range(2)]
    in_free = [torch.cuda.Event() for _ in range(2)]
    out_ready = [torch.cuda.Event() for _ in range(2)]
    out_free = [torch.cuda.Event() for _ in range(2)]
    out_ptr = m.output_ptr(0)
    d2d = cudart.cudaMemcpyKind.cudaMemcpyDeviceToDevice

    def e2e_steps(k):
        for i in range(k):
            b = i & 1
            if i >= 2:
                up.wait_event(in_free[b])      # step i-2 has consumed this staging buffer
            with torch.cuda.stream(up):
                d_in[b].copy_(h_in, non_blocking=True)
            in_ready[b].record(up)
            stream.wait_event(in_ready[b])
            m._check(m._lib.gawee_set_arg_device(m._h, 0, d_in[b].data_ptr(), in_bytes, sp))
            in_free[b].record(stream)
            step()
            if i >= 2:
                stream.wait_event(out_free[b])  # step i-2's result has reached the host
            err, = cudart.cudaMemcpyAsync(d_out[b].data_ptr(), out_ptr, out_bytes, d2d, cudart.cudaStream_t(sp))
            if err != cudart.cudaError_t.cudaSuccess:
                raise RuntimeError(f"cudaMemcpyAsync: {err}")
            out_ready[b].record(stream)
            down.wait_event(out_ready[b])
            with torch.cuda.stream(down):
                h_out[b].copy_(d_out[b], non_blocking=True)
            out_free[b].record(down)

    e2e_steps(2)
    torch.cuda.synchronize(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(up)
    e2e_steps(a.steps)
    e1.record(down)                              # after the last step's download
    torch.cuda.synchronize(local)
    ms_e2e = e0.elapsed_time(e1)
    clk.__exit__(None, None, None)
    clocks = clk.summary()
    if world > 1:
        t = torch.tensor([ms_e2e], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_e2e = float(t.item())
    e2e_value = total_batch * items * a.steps / (ms_e2e / 1e3)

    # per-kernel device times of one eager forward -> tensor-core roofline
    kern = m.kernels()
    prof = m.profile(sp)
    tc_ms = sum(t for (n, tc, f), t in zip(kern, prof) if tc)
    tc_flops = sum(f for (n, tc, f) in kern if tc)
    fwd_ms = sum(prof)
    peaks = load_peaks()
    achieved = tc_flops / (tc_ms / 1e3) / 1e12 if tc_ms > 0 else 0.0
    peak = peaks["bf16"]
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak if peak else None, "traffic": None,
                "peak_source": f"{peaks['source']} bf16 dense (cuBLAS); fp32 here is 3 TF32 passes at half the bf16 rate",
                "fp32_emulated_ceiling": peak / 6.0, "frac_of_fp32_emulated_ceiling": achieved / (peak / 6.0),
                "kernel": "conv_gemm_tc_kernel (tcgen05 kind::tf32, 3 passes)",
                "tc_share_of_forward": tc_ms / fwd_ms if fwd_ms else None,
                "tc_ms_per_forward": tc_ms, "tc_flops_per_forward": tc_flops}

    line = {"metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": ms / a.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded; architecture and init as the config, no pretrained weights)",
            "config": {"workload": a.workload, "global_batch": total_batch, "per_gpu_batch": per_gpu,
                       "parallelism": f"dp{world} (each GPU runs its own batch; weights replicated; "
                                      "no collective on the data path)",
                       "l2": "inputs larger than L2 (ResNet input 154 MB per step at N=1)"
                       if a.workload == "resnet18" else "activations larger than L2"},
            "e2e": {"value": e2e_value, "unit": unit, "h2d_bytes_per_step": in_bytes * world,
                    "d2h_bytes_per_step": out_bytes * world},
            "roofline": roofline, "clocks": clocks,
            "gpu_launches": m.num_kernels() * a.steps}
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(a.workload)
    if rank == 0:
        sys.stderr.write("per-kernel ms (one eager forward):\n")
        for (n, tc, f), t in sorted(zip(kern, prof), key=lambda x: -x[1])[:12]:
            sys.stderr.write(f"  {t:8.3f} ms  {'TC' if tc else '  '} {f / 1e9:9.2f} GFLOP  {n}\n")
        groups = {}
        for (n, tc, f), t in zip(kern, prof):
            g = groups.setdefault(n, [0, 0.0, 0.0])
            g[0] += 1
            g[1] += t
            g[2] += f
        sys.stderr.write("by op (launches, total ms, GFLOP):\n")
        for n, (c, t, f) in sorted(groups.items(), key=lambda x: -x[1][1]):
            sys.stderr.write(f"  {t:9.3f} ms  {c:5d}  {f / 1e9:9.2f} GFLOP  {n}\n")
        print(json.dumps(line), flush=True)
    m.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
