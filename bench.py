#!/usr/bin/env python
"""Benchmark: compiled inference of a gawee graph on B200, data parallel over N GPUs.

Default workload (the metric's first half, configuration 3): ResNet-18 fp32,
a global batch of 256 images of 3x224x224 ~N(0,1), Kaiming-normal conv
weights with BatchNorm folded into the conv bias, graph in the gawee dialect
as the ONNX emitter prints it.  On N GPUs the batch is split in contiguous
row blocks (256/N images per GPU), weights are replicated, and every step
ends with the NCCL gather of each rank's logits to rank 0 (strong scaling:
the total work is fixed).  `--workload decoder135m` runs the 135M GQA decoder
prefill (global batch 64 x 512 tokens) the same way.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl gawee|reference]

One JSON line on rank 0:
  value       whole-job images/s (or tokens/s): device time of K steps
              (forward + gather to rank 0), inputs resident in HBM, CUDA events
              on the launch stream, max over ranks
  value_no_gather  the same without the gather
  e2e         same metric through the C ABI with pinned host buffers: each step
              copies each rank's input rows in, runs the forward, gathers to
              rank 0 and copies the gathered logits back to the host;
              consecutive steps are pipelined (upload, compute and download on
              three streams, two staging buffers each way)
  roofline    tensor-core kernels: algorithmic FLOPs / their device time in an
              eagerly profiled forward, against the measured peaks
  cpu_baseline  the CPU oracle (a C++ port of the reference lowering semantics)
              on a bounded sample on this host, N=1 only (all threads, and
              one thread as the reference's generated code runs)
  extra       N=1 only: the metric's other configurations -- the decoder-135M
              prefill (configuration 4, tokens/s) and the batch-1 latencies of
              ResNet-18, BERT-tiny and Llama-15M (configurations 0-2; Llama-15M
              both as the reference binding's KV-cache decode step and as a
              256-token prefill) -- each with its own e2e, roofline and CPU
              baseline; and `precision_modes`: the ResNet-18 b256 and
              decoder-135M b64 forwards again in the single-pass TF32 and
              BF16 modes (reduced precision, not the headline)
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
    # name: metric, unit, global batch (rows split across the GPUs), units per batch row
    "resnet18": ("ResNet-18 fp32 images/s (global batch 256 of 3x224x224 sharded over the GPUs, "
                 "logits gathered to rank 0)", "images/s", 256, 1),
    "decoder135m": ("decoder-135M GQA fp32 prefill tokens/s (global batch 64 x seq 512 sharded over the GPUs, "
                    "logits gathered to rank 0)", "tokens/s", 64, 512),
}


def build_graph(workload: str, batch: int):
    from gawee_b200 import synth
    if workload == "resnet18":
        return synth.resnet18(batch)
    return synth.smollm135m(batch, 512)


def global_inputs(workload: str, batch: int):
    """Seeded inputs of the whole global batch (every rank builds the same
    array and keeps its own rows)."""
    rng = np.random.default_rng(43)
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


def _time_oracle(g, threads: int, seconds_hint: float, max_reps: int = 8):
    import oracle
    args = g.make_args()
    o = oracle.Oracle(g.mlir)
    reps, t_total = 0, 0.0
    while reps == 0 or (t_total < seconds_hint and reps < max_reps):
        t0 = time.perf_counter()
        o.run(args, threads=threads)
        t_total += time.perf_counter() - t0
        reps += 1
    return t_total / reps, reps


def cpu_baseline(workload: str, seconds_hint: float = 15.0):
    """The oracle on one batch row (1 image / 1 sequence of 512 tokens), with
    every host thread, and single-threaded as the reference's generated code
    runs (scalar, one thread)."""
    _, unit, _, items = WORKLOADS[workload]
    g = build_graph(workload, 1)
    threads = os.cpu_count() or 1
    per_row, reps = _time_oracle(g, threads, seconds_hint)
    out = {"value": items / per_row, "unit": unit, "cores": threads, "kind": "port",
           "sample": f"{reps} run(s) of a batch-1 slice "
                     f"({'1 image' if workload == 'resnet18' else '1 sequence x 512 tokens'}) of the same graph "
                     f"on the C++ oracle, {threads} threads; the whole batch extrapolates linearly"}
    if workload == "resnet18":
        per1, reps1 = _time_oracle(g, 1, 4.0, max_reps=2)
        out["single_thread"] = {"value": items / per1, "unit": unit, "cores": 1,
                                "sample": f"{reps1} run(s) of 1 image, 1 thread"}
    return out


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
            "warmup": a.warmup, "ms_per_step": dt / a.steps * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": a.workload, "global_batch": total,
                       "sample_per_step": "a batch-1 slice; throughput extrapolates linearly over the batch"},
            "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# DRAM bytes (read + write) of the tensor-core kernels per batch row, from one
# ncu capture (dram__bytes_read.sum + dram__bytes_write.sum over one forward):
# workload -> (bytes per row, batch captured, summary).  Scaled to the bench's
# batch, where traffic grows with the rows (batches at least as large as the
# captured one; smaller batches keep more of their activations in L2).
TC_DRAM_BYTES = {
    "resnet18": (968.2e6 / 64, 64, "profiles/resnet18_b64_dram.md"),
}


def tc_traffic(workload, rows):
    if workload not in TC_DRAM_BYTES:
        return None, None
    per_row, cap_rows, src = TC_DRAM_BYTES[workload]
    if rows < cap_rows:
        return None, None
    return per_row * rows, (f"{src}: ncu DRAM bytes of the tensor-core kernels of one batch-{cap_rows} forward, "
                            f"x {rows}/{cap_rows}")


def tc_roofline(m, sp, peaks, workload=None, rows=0):
    """Tensor-core kernels of one eagerly profiled forward: algorithmic FLOPs
    over their CUDA-event device time, against the measured peaks."""
    kern = m.kernels()
    prof = m.profile(sp)
    tc_ms = sum(t for (n, tc, f), t in zip(kern, prof) if tc)
    tc_flops = sum(f for (n, tc, f) in kern if tc)
    fwd_ms = sum(prof)
    achieved = tc_flops / (tc_ms / 1e3) / 1e12 if tc_ms > 0 else 0.0
    peak = peaks["bf16"]
    tf32, tf32_src = tf32_mma_rate(m.device)
    traffic, traffic_src = tc_traffic(workload, rows)
    r = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
         "frac": achieved / peak if peak else None, "traffic": traffic, "traffic_source": traffic_src,
         "peak_source": f"{peaks['source']} bf16 dense (cuBLAS burst); fp32 here is 3 TF32 passes",
         "tf32_mma_tflops": tf32, "tf32_mma_source": tf32_src,
         "fp32_3xtf32_ceiling": tf32 / 3.0,
         "frac_of_fp32_3xtf32_ceiling": achieved / (tf32 / 3.0),
         "kernel": "conv_gemm_tma_kernel + conv_gemm_tc_kernel (tcgen05 kind::tf32, 3 passes)",
         "tc_share_of_forward": tc_ms / fwd_ms if fwd_ms else None,
         "tc_ms_per_forward": tc_ms, "tc_flops_per_forward": tc_flops, "forward_ms_eager": fwd_ms}
    return r, kern, prof


# Raw tcgen05.mma kind::tf32 rate: measured at run time by gawee_probe_tf32_mma
# (back-to-back M = 128, N = 128, K = 8 MMAs on every SM).  The fallback is the
# same shape's cost measured on this pool's B200s, 64 cycles per MMA: 4096
# FLOP per cycle per SM, 148 SMs at 1965 MHz.  The fp32 path issues three
# TF32 MMAs per product, so its tensor ceiling is a third of the rate.
TF32_MMA_TFLOPS_FALLBACK = 4096 * 148 * 1.965e9 / 1e12


def tf32_mma_rate(device):
    import ctypes
    from gawee_b200.runtime import load_library
    out = ctypes.c_double(0.0)
    if load_library().gawee_probe_tf32_mma(device, ctypes.byref(out)) == 0 and out.value > 0:
        return out.value, "measured now (gawee_probe_tf32_mma)"
    return TF32_MMA_TFLOPS_FALLBACK, "64 cycles per 128x128x8 MMA at 1965 MHz (earlier measurement)"


def l2_flush_buffer(dev):
    import torch
    return torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # 256 MB > 126 MB L2


def latency_entry(name, g, metric, published_ms, published_src, peaks, local, steps):
    """Batch-1 latency of one config: CUDA-graph replays timed one by one with
    CUDA events, L2 flushed between replays (outside the events)."""
    import torch
    from gawee_b200.runtime import Model
    args = g.make_args()
    m = Model(g.mlir, device=local)
    try:
        m.set_args(args)
        stream = torch.cuda.Stream(local)
        sp = stream.cuda_stream
        flush = l2_flush_buffer(f"cuda:{local}")
        for _ in range(5):
            m.forward(sp)
        m.synchronize(sp)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for e0, e1 in ev:
            with torch.cuda.stream(stream):
                flush.fill_(1)
            e0.record(stream)
            m.forward(sp)
            e1.record(stream)
        m.synchronize(sp)
        times = sorted(e0.elapsed_time(e1) for e0, e1 in ev)
        ms = statistics.median(times)
        # end to end: input from pinned host memory, forward, logits back to pinned host memory
        in_bytes = sum(a.nbytes for a, spec in zip(args, g.args) if spec.kind == "input")
        hosts = [torch.from_numpy(a).pin_memory() if spec.kind == "input" else None for a, spec in zip(args, g.args)]
        out_dt, out_shape = m.output_specs[0]
        h_out = torch.empty(int(np.prod(out_shape)) * out_dt.itemsize, dtype=torch.uint8).pin_memory()
        e2e = []
        for _ in range(steps):
            with torch.cuda.stream(stream):
                flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for i, h in enumerate(hosts):
                if h is not None:
                    m._check(m._lib.gawee_set_arg(m._h, i, h.data_ptr(), h.numel() * h.element_size(), sp))
            m.forward(sp)
            m._check(m._lib.gawee_get_output(m._h, 0, h_out.data_ptr(), h_out.numel(), sp))
            e1.record(stream)
            m.synchronize(sp)
            e2e.append(e0.elapsed_time(e1))
        roof, kern, prof = tc_roofline(m, sp, peaks)
        n_launch = m.num_launches()
    finally:
        m.close()
    per, reps = _time_oracle(g, os.cpu_count() or 1, 5.0, max_reps=4)
    per1, reps1 = _time_oracle(g, 1, 5.0, max_reps=2)
    return {"metric": metric, "value": ms, "unit": "ms", "higher_is_better": False, "steps": steps,
            "min_ms": times[0], "p90_ms": times[int(0.9 * (len(times) - 1))],
            "l2": "flushed (256 MB write) before every replay, outside the timed events",
            "e2e": {"value": statistics.median(e2e), "unit": "ms", "h2d_bytes_per_step": in_bytes,
                    "d2h_bytes_per_step": int(h_out.numel())},
            "gpu_launches_per_step": n_launch, "roofline": roof,
            "cpu_baseline": {"value": per * 1e3, "unit": "ms", "cores": os.cpu_count() or 1, "kind": "port",
                             "sample": f"{reps} run(s) of the whole batch-1 graph on the C++ oracle",
                             "single_thread_ms": per1 * 1e3},
            "reference_published_ms": published_ms, "reference_published_source": published_src}


def precision_modes(m, stream, steps, units):
    """Device time of `steps` forwards of an already warmed model in each
    reduced-precision mode (single-pass TF32, BF16), as units per second;
    the model is left in fp32.  Neither is a parity mode: their error bounds
    are stated with gawee_set_precision in include/gawee_cuda.h."""
    import torch
    sp = stream.cuda_stream
    out = {}
    try:
        for mode in ("tf32", "bf16"):
            m.set_precision(mode)
            for _ in range(3):
                m.forward(sp)
            m.synchronize(sp)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(steps):
                m.forward(sp)
            e1.record(stream)
            m.synchronize(sp)
            ms = e0.elapsed_time(e1) / steps
            out[mode] = {"value": units / ms * 1e3, "ms_per_step": ms}
    finally:
        m.set_precision("fp32")
    return out


def decoder_entry(peaks, local, steps):
    """Config 4 at N=1: decoder-135M prefill, batch 64 x 512, tokens/s."""
    import torch
    from gawee_b200.runtime import Model
    g = build_graph("decoder135m", 64)
    args = g.make_args()
    args[0] = np.ascontiguousarray(global_inputs("decoder135m", 64))
    m = Model(g.mlir, device=local)
    try:
        m.set_args(args)
        stream = torch.cuda.Stream(local)
        sp = stream.cuda_stream
        for _ in range(3):
            m.forward(sp)
        m.synchronize(sp)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            m.forward(sp)
        e1.record(stream)
        m.synchronize(sp)
        ms = e0.elapsed_time(e1) / steps
        h_in = torch.from_numpy(args[0]).pin_memory()
        out_dt, out_shape = m.output_specs[0]
        out_bytes = int(np.prod(out_shape)) * out_dt.itemsize
        h_out = torch.empty(out_bytes, dtype=torch.uint8).pin_memory()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            m._check(m._lib.gawee_set_arg(m._h, 0, h_in.data_ptr(), args[0].nbytes, sp))
            m.forward(sp)
            m._check(m._lib.gawee_get_output(m._h, 0, h_out.data_ptr(), out_bytes, sp))
        e1.record(stream)
        m.synchronize(sp)
        ms_e2e = e0.elapsed_time(e1) / steps
        roof, kern, prof = tc_roofline(m, sp, peaks)
        n_launch = m.num_launches()
        modes = precision_modes(m, stream, steps, 64 * 512)
    finally:
        m.close()
    tokens = 64 * 512
    cpu = cpu_baseline("decoder135m")
    return {"metric": "decoder-135M GQA fp32 prefill tokens/s (batch 64 x seq 512, 1 GPU)", "value": tokens / ms * 1e3,
            "unit": "tokens/s", "higher_is_better": True, "ms_per_step": ms, "steps": steps,
            "l2": "weights (538 MB) and activations larger than L2",
            "e2e": {"value": tokens / ms_e2e * 1e3, "unit": "tokens/s", "h2d_bytes_per_step": int(args[0].nbytes),
                    "d2h_bytes_per_step": out_bytes,
                    "note": "serial: upload, forward and the 6.4 GB logits download in one stream"},
            "gpu_launches_per_step": n_launch, "roofline": roof, "cpu_baseline": cpu,
            "precision_modes": modes}


def run_extra(peaks, local, resnet_modes=None):
    from gawee_b200 import synth
    out = {"decoder135m_prefill": decoder_entry(peaks, local, steps=5)}
    out["precision_modes"] = {
        "note": "the same workloads in the reduced-precision modes (not parity modes; bounds with "
                "gawee_set_precision in include/gawee_cuda.h): single-pass TF32 everywhere, or BF16 "
                "products on the TMA contraction kernel with single-pass TF32 elsewhere",
        "resnet18_b256": dict(resnet_modes or {}, unit="images/s"),
        "decoder135m_b64x512": dict(out["decoder135m_prefill"].pop("precision_modes"), unit="tokens/s")}
    cfgs = [("resnet18_b1_latency", synth.resnet18(1), "ResNet-18 fp32 batch-1 latency (1x3x224x224)", 6814.2),
            ("bert_tiny_s128_latency", synth.bert_tiny(), "BERT-tiny fp32 encoder latency (batch 1, seq 128)", 354.0),
            ("llama15m_decode_step_latency", synth.llama15m_decode(1, 1),
             "Llama-15M fp32 KV-cache decode step latency (batch 1, 1 new token over a past of 1: the reference "
             "tinyllama binding's shapes)", 107.6),
            ("llama15m_s256_prefill_latency", synth.llama15m(),
             "Llama-15M fp32 prefill latency (batch 1, seq 256)", None)]
    for name, g, metric, pub in cfgs:
        src = ("middle/delta.md:22-24 (Gawee CPU AOT p50 on an Apple M1-class CPU, 1 thread, process launch "
               "and npy I/O included)" if pub else
               "none: the reference publishes the tinyllama_15m decode step (see llama15m_decode_step_latency), "
               "not a 256-token prefill")
        out[name] = latency_entry(name, g, metric, pub, src, peaks, local, steps=30)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="gawee", choices=["gawee", "reference"])
    ap.add_argument("--workload", default="resnet18", choices=list(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the other configs of the metric (N=1 only)")
    ap.add_argument("--batch", type=int, default=0, help="override the global batch (small profiling runs)")
    a = ap.parse_args()
    if a.impl == "reference":
        return run_reference(a)

    import torch
    import torch.distributed as dist

    from gawee_b200 import dp
    from gawee_b200.runtime import Model

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    # NCCL_DEBUG is left as the caller set it: at any level from VERSION up
    # NCCL prints its version banner on stdout, where the JSON line goes
    # (unset, it prints nothing)
    if world != a.gpus:
        raise SystemExit(f"--gpus {a.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))

    metric, unit, global_batch, items = WORKLOADS[a.workload]
    if a.batch:
        global_batch = a.batch
        metric += f" [global batch overridden to {a.batch}]"
    s0, s1 = dp.shard_range(global_batch, world, rank)
    local_batch = s1 - s0
    g = build_graph(a.workload, local_batch)
    args = g.make_args()
    args[0] = np.ascontiguousarray(global_inputs(a.workload, global_batch)[s0:s1])
    m = Model(g.mlir, device=local)
    m.set_args(args)
    stream = torch.cuda.Stream(local)
    sp = stream.cuda_stream
    dev = f"cuda:{local}"

    out_dt, out_shape = m.output_specs[0]
    out_bytes = int(np.prod(out_shape)) * out_dt.itemsize
    gathered_bytes = out_bytes
    if world > 1:
        uid = dp.share_nccl_id(Model.dp_unique_id() if rank == 0 else bytes(128), rank)
        m.dp_init(world, rank, uid)
        gathered_bytes = m.dp_output_bytes(0)
    # rank 0's gather destinations (two, for the pipelined end-to-end loop)
    d_out = [torch.empty(gathered_bytes if rank == 0 else 1, dtype=torch.uint8, device=dev) for _ in range(2)]

    def step(dst=None):
        m.forward(sp)
        if world > 1:  # every rank, every step: the rows go to rank 0
            m.dp_gather_output(0, (dst if dst is not None else d_out[0]).data_ptr() if rank == 0 else None, sp)

    def forward_only():
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
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    clk = ClockSampler(local).__enter__()
    ms = timed(step, a.steps)
    m.synchronize(sp)
    value = global_batch * items * a.steps / (ms / 1e3)
    ms_ng = timed(forward_only, a.steps) if world > 1 else ms
    m.synchronize(sp)
    value_no_gather = global_batch * items * a.steps / (ms_ng / 1e3)

    # End to end through the C ABI, every step: this rank's input rows from
    # pinned host memory to the GPU, gawee_set_arg_device + gawee_forward, the
    # gather of every rank's rows to rank 0 (N > 1), and rank 0 reads the
    # gathered result back to pinned host memory.  Steps are pipelined the way
    # a serving loop runs them: step i+1's upload (its own stream) overlaps
    # step i's forward, and step i's download (another stream) overlaps step
    # i+1's, with two device staging buffers each way and events ordering the
    # hand-offs.
    from cuda.bindings import runtime as cudart
    in_bytes = args[0].nbytes
    h_in = torch.from_numpy(args[0]).pin_memory().view(torch.uint8).reshape(-1)
    h_out = [torch.empty(gathered_bytes, dtype=torch.uint8).pin_memory() for _ in range(2)]
    d_in = [torch.empty(in_bytes, dtype=torch.uint8, device=dev) for _ in range(2)]
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
            if i >= 2:
                stream.wait_event(out_free[b])  # step i-2's result has reached the host
            if world > 1:
                step(d_out[b])
            else:
                forward_only()
                err, = cudart.cudaMemcpyAsync(d_out[b].data_ptr(), out_ptr, out_bytes, d2d,
                                              cudart.cudaStream_t(sp))
                if err != cudart.cudaError_t.cudaSuccess:
                    raise RuntimeError(f"cudaMemcpyAsync: {err}")
            out_ready[b].record(stream)
            down.wait_event(out_ready[b])
            if rank == 0:
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
    e2e_value = global_batch * items * a.steps / (ms_e2e / 1e3)

    peaks = load_peaks()
    roofline, kern, prof = tc_roofline(m, sp, peaks, a.workload, s1 - s0)
    n_kern = m.num_launches()
    m.synchronize(sp)

    line = {"metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": ms / a.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "value_no_gather": value_no_gather,
            "dtype": "f32", "data": "synthetic (seeded; architecture and init as the config, no pretrained weights)",
            "config": {"workload": a.workload, "global_batch": global_batch, "per_gpu_batch": local_batch,
                       "parallelism": f"dp{world}: the global batch is split in contiguous row blocks, weights "
                                      "replicated; each step ends with the NCCL gather of every rank's output "
                                      "rows to rank 0" if world > 1 else "dp1 (one GPU holds the whole batch)",
                       "l2": "inputs larger than L2 (ResNet input 154 MB per step over all GPUs)"
                       if a.workload == "resnet18" else "weights and activations larger than L2"},
            "e2e": {"value": e2e_value, "unit": unit, "h2d_bytes_per_step": in_bytes * world
                    if global_batch % world == 0 else None,
                    "d2h_bytes_per_step": gathered_bytes},
            "roofline": roofline, "clocks": clocks,
            "gpu_launches": n_kern * a.steps}
    if world > 1:
        t = torch.tensor([in_bytes], device=dev, dtype=torch.int64)
        dist.all_reduce(t)
        line["e2e"]["h2d_bytes_per_step"] = int(t.item())
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(a.workload)
    extra_on = rank == 0 and world == 1 and not a.no_extra and a.workload == "resnet18" and not a.batch
    resnet_modes = precision_modes(m, stream, a.steps, global_batch * items) if extra_on else None
    m.close()
    if extra_on:
        line["extra"] = run_extra(peaks, local, resnet_modes)
    if rank == 0:
        sys.stderr.write("per-kernel ms (one eager forward):\n")
        for (n, tc, f), t in sorted(zip(kern, prof), key=lambda x: -x[1])[:12]:
            sys.stderr.write(f"  {t:8.3f} ms  {'TC' if tc else '  '} {f / 1e9:9.2f} GFLOP  {n}\n")
        groups = {}
        for (n, tc, f), t in zip(kern, prof):
            gg = groups.setdefault(n, [0, 0.0, 0.0])
            gg[0] += 1
            gg[1] += t
            gg[2] += f
        sys.stderr.write("by op (launches, total ms, GFLOP):\n")
        for n, (c, t, f) in sorted(groups.items(), key=lambda x: -x[1][1]):
            sys.stderr.write(f"  {t:9.3f} ms  {c:5d}  {f / 1e9:9.2f} GFLOP  {n}\n")
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
