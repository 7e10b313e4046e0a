#!/usr/bin/env python
"""Benchmark of manifesto's dtype/convert + fused-elementwise hot path on B200.

Headline workload (one JSON line on rank 0): whole-checkpoint FP8 E4M3
quantisation of a Llama-3-8B layout (291 BF16 tensors, 8,030,261,248 params,
values N(0, 0.02)) with per-tensor amax scales, every tensor row-split over the
N ranks (strong scaling: the checkpoint is fixed).  --path picks the step
(default auto: twopass on one GPU, passes on several):
  twopass  mf_ckpt_quant_fp8: amax pass, NCCL max all-reduce, cast pass
  passes   mf_ckpt_plan_run_passes: the amax pass, whose last CTA publishes the
           rank's maxima into every rank's exchange buffer over NVLink peer
           memory, then the cast pass, which waits for every rank's flag inside
           the kernel (two launches, no collective call)
  plan     mf_ckpt_plan_run: one launch, per group of tensors an amax phase and
           a cast phase that re-reads the group from L2, the per-group amax
           exchanged inside the kernel

  value      params quantised per second, whole job (max-over-ranks device time)
  e2e        the same through the C ABI with host buffers: pinned host BF16 ->
             device, quantise, FP8 + scales -> host, every step, beside the bare
             pinned-copy ceiling of the same bytes (link_ceiling_gbs)
  roofline   the step's kernel timed alone with CUDA events: 3 B/param (BF16 read
             once, E4M3 written once: the single-pass bound) / launch time vs the
             measured HBM copy peak and vs the measured ceiling of its 2:1
             read:write mix (mf_bw_probe)
  two_pass   the two-pass path on the same buffers: each pass alone and the step's
             phases (memset, pass 1, all-reduce, pass 2) with events between them,
             max over ranks
  kernels    (N=1) every other benchmark config as its own kernel line: FP8->FP32
             decode, Int4 group dequant, axpy f32/bf16, fused SwiGLU->FP8, each with
             the measured ceiling of its read:write mix
  cpu_baseline  (N=1, rank 0) the C oracle port of the Go loops on the host cores,
             on a bounded sample (the embedding matrix + decoder layer 0: 743,448,576
             params); each kernel line carries its own config's port timing under "cpu"
  parity     (every N, after the timed region) the amax vector against a
             torch.distributed all-reduce of each rank's own max|v|, and four tensors'
             FP8 shards against the CPU oracle; exit status 3 on a mismatch

--impl reference times that CPU port alone (the reference is Go; no Go toolchain
exists on these machines, so the port stands in for it).
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "achieved HBM GB/s and % of 8 TB/s roofline per kernel; elems/s at 1/2/4/8 B200"
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0
E4M3 = 5
BF16 = 4
F32 = 2


def hbm_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def traffic_table() -> dict:
    """Per-unit DRAM bytes measured with ncu (profiles/traffic.txt: kernel bytes_per_elem)."""
    out = {}
    p = ROOT / "profiles" / "traffic.txt"
    if p.exists():
        for line in p.read_text().splitlines():
            parts = line.split()
            if len(parts) >= 2 and not line.startswith("#"):
                try:
                    out[parts[0]] = float(parts[1])
                except ValueError:
                    pass
    return out


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi samples of this GPU's clocks during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines: list[str] = []

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
            time.sleep(0.3)
        except Exception:
            self.proc = None

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                mx.append(float(f[1]))
            except ValueError:
                continue
            for name, val in zip(names, f[4:8]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------- our arm

class Dist:
    def __init__(self, world: int, rank: int, local_rank: int):
        self.world, self.rank, self.local_rank = world, rank, local_rank
        self.pg = None

    def init(self, torch) -> None:
        if self.world > 1:
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                    device_id=torch.device("cuda", self.local_rank))
            self.pg = dist

    def barrier(self, torch) -> None:
        if self.pg:
            self.pg.barrier()
        torch.cuda.synchronize()

    def max(self, torch, v: float) -> float:
        if not self.pg:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def all_gather_bytes(self, data: bytes) -> list[bytes]:
        if not self.pg:
            return [data]
        out = [None] * self.world
        self.pg.all_gather_object(out, data)
        return out

    def broadcast_bytes(self, data: bytes | None) -> bytes:
        if not self.pg:
            return data
        obj = [data]
        self.pg.broadcast_object_list(obj, src=0)
        return obj[0]

    def close(self) -> None:
        if self.pg:
            self.pg.destroy_process_group()


def fill_normal_bf16(torch, t, seed: int, mu: float, sigma: float) -> None:
    """Fill a bf16 tensor with N(mu, sigma) from a seeded device generator (one launch)."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    t.view(-1).normal_(mu, sigma, generator=g)


def time_launches(torch, fn, reps: int, flush=None) -> list[float]:
    """Per-launch device times (ms) with CUDA events on torch's current stream.

    All (flush, start, launch, end) sets are queued before one synchronisation,
    so the device never idles waiting for the host between an event and its
    launch (the host-side call overhead stays outside the measured interval).
    """
    torch.cuda.synchronize()
    pairs = []
    for _ in range(reps):
        if flush is not None:
            flush()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        pairs.append((s, e))
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in pairs]


def kernel_line(name: str, alg_bytes: float, times_ms: list[float], peak: float, elems: int,
                ceiling: dict | None = None) -> dict:
    ms = statistics.median(times_ms)
    gbs = alg_bytes / (ms * 1e-3) / 1e9
    line = {"kernel": name, "ms": round(ms, 4), "alg_bytes": int(alg_bytes), "gbs": round(gbs, 1),
            "frac_of_measured": round(gbs / peak, 4), "frac_of_8tbs": round(gbs / NOMINAL_HBM_GBS, 4),
            "elems_per_s": elems / (ms * 1e-3), "reps": len(times_ms)}
    if ceiling:
        line["direction_ceiling"] = ceiling
        line["frac_of_direction_ceiling"] = round(gbs / ceiling["gbs"], 4)
    return line


PROBE_MIXES = {(1, 0): "read-only", (0, 1): "write-only", (1, 1): "copy 1:1", (1, 4): "read 1 : write 4",
               (2, 1): "read 2 : write 1"}


def probe_ceiling(torch, stream_handle: int, src_ptr: int, a: int, dst_ptr: int, b: int, n_steps: int, flush=None,
                  reps: int = 20) -> dict:
    """DRAM ceiling of one read:write mix, measured with mf_bw_probe (bulk-copy loads and stores, no other
    work) on the given buffers: median of `reps` launches, L2 flushed before each."""
    from manifesto_b200._abi import call
    f = lambda: call("mf_bw_probe", src_ptr, a, dst_ptr, b, n_steps, stream_handle)
    _warm(f)
    ms = statistics.median(time_launches(torch, f, reps, flush))
    nbytes = 16 * n_steps * (a + b)
    return {"mix": PROBE_MIXES[(a, b)], "bytes": int(nbytes), "ms": round(ms, 4),
            "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1), "kernel": f"bw_probe_kernel<{a},{b}>"}


KERNEL_CONFIGS = ("c1", "c2", "c3", "c3s", "c4", "c4g")


def bench_kernels(torch, stream_handle: int, peak: float, which=KERNEL_CONFIGS, reps: int = 50) -> dict:
    """Configs 1-4 on one GPU, each kernel timed alone with L2 flushed before every launch."""
    flush_buf = torch.empty(512 << 20, dtype=torch.uint8, device="cuda")
    flush_words = flush_buf.view(torch.int64)

    def flush():
        # Write a buffer 4x the L2, then read it back: the read evicts the
        # write's dirty lines, so the timed kernel starts with a cold L2 that
        # holds none of its inputs and no write-backs owed by someone else.
        flush_buf.fill_(1)
        torch.amax(flush_words)
    out = {}
    for name in which:
        out.update({"c1": _kernel_c1, "c2": _kernel_c2, "c3": _kernel_c3, "c3s": _kernel_c3s, "c4": _kernel_c4,
                    "c4g": _kernel_c4g}[name](
            torch, stream_handle, peak, flush, reps))
        torch.cuda.empty_cache()
    del flush_buf
    torch.cuda.empty_cache()
    return out


def _warm(f, k: int = 3) -> None:
    for _ in range(k):
        f()


def _kernel_c1(torch, stream_handle, peak, flush, reps) -> dict:
    """Config 1: FP8 E4M3 -> FP32, 2^26 elements (bytes uniform over all 256 codes)."""
    from manifesto_b200._abi import call
    n = 1 << 26
    src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda")
    dst = torch.empty(n, dtype=torch.float32, device="cuda")
    f = lambda: call("mf_convert", 5, 2, src.data_ptr(), dst.data_ptr(), n, 0, stream_handle)
    _warm(f)
    times = time_launches(torch, f, reps, flush)
    ceiling = probe_ceiling(torch, stream_handle, src.data_ptr(), 1, dst.data_ptr(), 4, n // 16, flush)
    return {"c1_fp8e4m3_to_f32": kernel_line("stream_kernel<ConvertOp<E4M3,F32>>", 5 * n, times, peak, n, ceiling)}


def _kernel_c2(torch, stream_handle, peak, flush, reps) -> dict:
    """Config 2: Int4 -> BF16 dequant, 4096 x 14336, group 128, BF16 scales ~ |N(0, 0.02)|."""
    from manifesto_b200._abi import call
    rows, cols, group = 4096, 14336, 128
    q = torch.randint(0, 256, (rows * cols // 2,), dtype=torch.uint8, device="cuda")
    sc = (torch.randn(rows * cols // group, device="cuda").abs() * 0.02).to(torch.bfloat16)
    o = torch.empty(rows * cols, dtype=torch.bfloat16, device="cuda")
    f = lambda: call("mf_int4_dequant_grouped", q.data_ptr(), sc.data_ptr(), 4, o.data_ptr(), 4, rows, cols, group,
                     stream_handle)
    _warm(f)
    b = rows * cols // 2 + sc.numel() * 2 + rows * cols * 2
    times = time_launches(torch, f, reps, flush)
    ceiling = probe_ceiling(torch, stream_handle, q.data_ptr(), 1, o.data_ptr(), 4, q.numel() // 16, flush)
    return {"c2_int4_to_bf16": kernel_line("int4_dequant_flat_kernel<BF16,BF16>", b, times, peak, rows * cols,
                                           ceiling)}


def _kernel_c3(torch, stream_handle, peak, flush, reps) -> dict:
    """Config 3: axpy y = 0.75 x + y, N = 2^28, in FP32 and in BF16 (FP32 arithmetic)."""
    from manifesto_b200._abi import call
    out = {}
    n = 1 << 28
    # x and y back to back in one buffer, so the ceiling probe reads both as its two input regions and
    # writes y, as axpy does
    xy = torch.randn(2 * n, device="cuda")
    x, y = xy[:n], xy[n:]
    f = lambda: call("mf_axpy", y.data_ptr(), x.data_ptr(), n, 0.75, 2, 0, stream_handle)
    _warm(f)
    times = time_launches(torch, f, reps, flush)
    xyb = xy.to(torch.bfloat16)
    ceiling = probe_ceiling(torch, stream_handle, xy.data_ptr(), 2, y.data_ptr(), 1, n // 4, flush)
    out["c3a_axpy_f32"] = kernel_line("stream_kernel<AxpyOp<F32>>", 12 * n, times, peak, n, ceiling)
    del xy, x, y
    xb, yb = xyb[:n], xyb[n:]
    f = lambda: call("mf_axpy", yb.data_ptr(), xb.data_ptr(), n, 0.75, 4, 0, stream_handle)
    _warm(f)
    times = time_launches(torch, f, reps, flush)
    ceiling = probe_ceiling(torch, stream_handle, xyb.data_ptr(), 2, yb.data_ptr(), 1, n // 8, flush)
    out["c3b_axpy_bf16"] = kernel_line("stream_kernel<AxpyOp<BF16>>", 6 * n, times, peak, n, ceiling)
    return out


def _kernel_c3s(torch, stream_handle, peak, flush, reps) -> dict:
    """The scalar loop beside axpy: out = x * 0.75 (applyScalarBroadcast, mul), N = 2^28, FP32 -> FP32 and
    BF16 -> BF16 (FP32 arithmetic)."""
    from manifesto_b200._abi import call
    out = {}
    n = 1 << 28
    for key, dt, width, name in (("c3s_scalar_mul_f32", 2, 4, "F32,F32"), ("c3s_scalar_mul_bf16", 4, 2, "BF16,BF16")):
        src = torch.randn(n, device="cuda")
        if width == 2:
            src = src.to(torch.bfloat16)
        dst = torch.empty_like(src)
        f = lambda: call("mf_scalar_broadcast", src.data_ptr(), dt, dst.data_ptr(), dt, n, 0.75, 2, stream_handle)
        _warm(f)
        times = time_launches(torch, f, reps, flush)
        ceiling = probe_ceiling(torch, stream_handle, src.data_ptr(), 1, dst.data_ptr(), 1, n * width // 16, flush)
        out[key] = kernel_line(f"stream_kernel<ScalarOp<{name},mul>>", 2 * width * n, times, peak, n, ceiling)
        del src, dst
        torch.cuda.empty_cache()
    return out


def _kernel_c4(torch, stream_handle, peak, flush, reps) -> dict:
    """Config 4: Mul(Silu(Add(Mul(x, gamma), beta)), y) on BF16 [64, 2048, 4096] -> amax -> E4M3."""
    from manifesto_b200 import fusion
    from manifesto_b200._abi import call
    from manifesto_b200.dtype import DType
    out = {}
    hidden = 4096
    n = 64 * 2048 * hidden
    xy = torch.empty(2 * n, dtype=torch.bfloat16, device="cuda")  # x, y back to back (the ceiling probe's input)
    x, y = xy[:n], xy[n:]
    fill_normal_bf16(torch, x, 41, 0.0, 1.0)
    fill_normal_bf16(torch, y, 42, 0.0, 1.0)
    g = (torch.randn(hidden, device="cuda") * 0.1 + 1.0).to(torch.bfloat16)
    be = (torch.randn(hidden, device="cuda") * 0.1).to(torch.bfloat16)
    pre = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    qo = torch.empty(n, dtype=torch.uint8, device="cuda")
    am = torch.zeros(1, dtype=torch.float32, device="cuda")
    si = torch.zeros(1, dtype=torch.float32, device="cuda")
    k = fusion.emit_cuda(fusion.swiglu_chain(), in_dtypes=[DType.BFLOAT16] * 4, in_bcast=[0, hidden, hidden, 0],
                         out_dtype=DType.BFLOAT16)
    ptrs = [x.data_ptr(), g.data_ptr(), be.data_ptr(), y.data_ptr()]
    f = lambda: k.run_fp8(ptrs, pre.data_ptr(), qo.data_ptr(), n, am.data_ptr(), si.data_ptr(), stream=stream_handle)
    _warm(f)
    t_all = time_launches(torch, f, reps, flush)
    f1 = lambda: k.run(ptrs, pre.data_ptr(), n, amax=am.data_ptr(), stream=stream_handle)
    t1 = time_launches(torch, f1, reps, flush)
    f2 = lambda: call("mf_fp8_scaled_cast", pre.data_ptr(), 4, qo.data_ptr(), 5, am.data_ptr(), si.data_ptr(), n, 0,
                      stream_handle)
    t2 = time_launches(torch, f2, reps, flush)
    # ceilings last: the probes overwrite pre and qo
    c1 = probe_ceiling(torch, stream_handle, xy.data_ptr(), 2, pre.data_ptr(), 1, n // 8, flush)
    c2 = probe_ceiling(torch, stream_handle, pre.data_ptr(), 2, qo.data_ptr(), 1, n // 16, flush)
    both = {"mix": "read 2 : write 1 (both passes)", "bytes": c1["bytes"] + c2["bytes"], "ms": c1["ms"] + c2["ms"],
            "gbs": round((c1["bytes"] + c2["bytes"]) / ((c1["ms"] + c2["ms"]) * 1e-3) / 1e9, 1),
            "kernel": "bw_probe_kernel<2,1> x 2"}
    out["c4_fused_swiglu_fp8"] = kernel_line("mf_jit_tma (SwiGLU, amax) + stream_kernel<CastOp<BF16,E4M3>>", 9 * n,
                                             t_all, peak, n, both)
    out["c4_pass1_swiglu"] = kernel_line("mf_jit_tma (generated for the SwiGLU chain) <amax>", 6 * n, t1, peak, n, c1)
    out["c4_pass2_cast"] = kernel_line("stream_kernel<CastOp<BF16,E4M3>>", 3 * n, t2, peak, n, c2)
    out["c4_fused_swiglu_fp8"]["single_pass_lower_bound_bytes"] = 5 * n
    k.close()
    return out


def _kernel_c4g(torch, stream_handle, peak, flush, reps) -> dict:
    """A chain with no specialised kernel, on config 4's shape: Gelu(Add(Mul(x, gamma), beta)) on BF16
    [64, 2048, 4096], gamma/beta broadcast over the last dimension, BF16 out (the generic fused path)."""
    from manifesto_b200 import fusion
    from manifesto_b200.dtype import DType
    hidden = 4096
    n = 64 * 2048 * hidden
    x = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    fill_normal_bf16(torch, x, 43, 0.0, 1.0)
    g = (torch.randn(hidden, device="cuda") * 0.1 + 1.0).to(torch.bfloat16)
    be = (torch.randn(hidden, device="cuda") * 0.1).to(torch.bfloat16)
    o = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    k = fusion.emit_cuda(fusion.gelu_affine_chain(), in_dtypes=[DType.BFLOAT16] * 3, in_bcast=[0, hidden, hidden],
                         out_dtype=DType.BFLOAT16)
    assert not k.specialised()
    ptrs = [x.data_ptr(), g.data_ptr(), be.data_ptr()]
    f = lambda: k.run(ptrs, o.data_ptr(), n, stream=stream_handle)
    _warm(f)
    times = time_launches(torch, f, reps, flush)
    # read x, write out: the copy-shaped 1:1 mix
    ceiling = probe_ceiling(torch, stream_handle, x.data_ptr(), 1, o.data_ptr(), 1, n * 2 // 16, flush)
    line = kernel_line("mf_jit_tma (generated for Gelu(Add(Mul(x,g),b)), BF16)", 4 * n, times, peak, n, ceiling)
    k.close()
    return {"c4g_fused_gelu_generic": line}


def run_ours(args, world: int, rank: int, local_rank: int) -> None:
    import torch

    from manifesto_b200 import CUDABackend, checkpoint
    from manifesto_b200._abi import call

    torch.cuda.set_device(local_rank)
    CUDABackend(local_rank)
    dist = Dist(world, rank, local_rank)
    dist.init(torch)
    stream = torch.cuda.current_stream().cuda_stream
    peak, peak_src = hbm_peak()

    if args.only_kernels:
        if rank == 0:
            which = tuple(args.kernels.split(","))
            print(json.dumps({"kernels": bench_kernels(torch, stream, peak, which, reps=args.steps)}), flush=True)
        dist.close()
        return

    if args.path == "auto":
        args.path = "twopass" if world == 1 else "passes"
    full = args.ckpt_layers == 32 and args.ckpt_vocab == 128256
    specs = checkpoint.llama3_8b_layout(layers=args.ckpt_layers, vocab=args.ckpt_vocab)
    total_params = sum(s.numel for s in specs)
    parts = checkpoint.partition(specs, world, rank)
    local = [rows * s.cols for (first, rows), s in zip(parts, specs)]
    local_params = sum(local)
    src = torch.empty(local_params, dtype=torch.bfloat16, device="cuda")
    dst = torch.empty(local_params, dtype=torch.uint8, device="cuda")
    amax = torch.zeros(len(specs), dtype=torch.float32, device="cuda")
    sinv = torch.zeros(len(specs), dtype=torch.float32, device="cuda")
    entries, off = [], 0
    for t, n in enumerate(local):
        if n:
            fill_normal_bf16(torch, src[off:off + n], 1000 * t + rank, 0.0, 0.02)
        entries.append((src.data_ptr() + 2 * off, dst.data_ptr() + off, n, t, BF16))
        off += n
    chunks = checkpoint.make_chunks(entries)
    comm = None
    if world > 1:
        uid = dist.broadcast_bytes(checkpoint.Communicator.unique_id() if rank == 0 else None)
        comm = checkpoint.Communicator(world, rank, uid)
    plan = None
    if args.path in ("plan", "passes"):
        plan = checkpoint.QuantPlan(chunks, len(entries), len(specs), tensor_numel=[s.numel for s in specs],
                                    group_bytes=int(args.group_mb * (1 << 20)), world=world, rank=rank)
        plan.connect(dist.all_gather_bytes(plan.ipc_handle))
        dist.barrier(torch)

    def step():
        if args.path == "plan":
            plan.run(amax.data_ptr(), sinv.data_ptr(), stream)
        elif args.path == "passes":
            plan.run_passes(amax.data_ptr(), sinv.data_ptr(), stream)
        else:
            checkpoint.quantise(chunks, len(entries), len(specs), amax.data_ptr(), sinv.data_ptr(), E4M3, 0, comm,
                                stream)

    for _ in range(args.warmup):
        step()
    dist.barrier(torch)
    gpu_id = "GPU-" + str(torch.cuda.get_device_properties(local_rank).uuid).replace("GPU-", "")
    sampler = ClockSampler(gpu_id)
    sampler.start()
    dist.barrier(torch)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    dist.barrier(torch)
    clocks = sampler.stop()
    local_ms = t0.elapsed_time(t1)
    ms = dist.max(torch, local_ms)
    value = total_params * args.steps / (ms * 1e-3)
    job_gbs = 3.0 * total_params * args.steps / (ms * 1e-3) / 1e9

    # the DRAM ceilings of the step's access mixes on this rank's buffers (the probes overwrite dst only)
    ceilings = {"read_only": probe_ceiling(torch, stream, src.data_ptr(), 1, 0, 0, 2 * local_params // 16, reps=10),
                "read2_write1": probe_ceiling(torch, stream, src.data_ptr(), 2, dst.data_ptr(), 1, local_params // 16,
                                              reps=10)}
    traffic = traffic_table()
    one_pass_bytes = 3.0 * local_params  # read BF16 once, write E4M3 once: the single-pass lower bound
    passes = None
    if args.path == "passes":
        # the step's two launches with an event between them; the cast pass's time includes its wait for
        # every rank's published maxima
        passes = passes_breakdown(torch, dist, plan, amax, sinv, stream)
        cast_x_ms = passes["cast_pass_ms"]
        achieved = one_pass_bytes / (cast_x_ms * 1e-3) / 1e9
        tr = traffic.get("ckpt_cast_pass")
        roofline = {"bound": "hbm", "kernel": "stream_kernel<CastXOp<BF16,E4M3>> (waits on the ranks' published "
                                              "amax, then reads BF16 and writes E4M3)",
                    "alg_bytes_per_launch": int(one_pass_bytes),
                    "launch_ms": round(cast_x_ms, 4), "achieved": round(achieved, 1), "peak": peak,
                    "peak_source": peak_src, "unit": "GB/s", "frac": round(achieved / peak, 4),
                    "frac_of_8tbs": round(achieved / NOMINAL_HBM_GBS, 4),
                    "traffic": int(tr * local_params) if tr else None,
                    "direction_ceiling": ceilings["read2_write1"],
                    "frac_of_direction_ceiling": round(achieved / ceilings["read2_write1"]["gbs"], 4)}
    if args.path == "plan":
        # the dominant (only) kernel: the one-launch step, events around each launch
        run_ms = statistics.mean(time_launches(torch, step, 10))
        achieved = one_pass_bytes / (run_ms * 1e-3) / 1e9
        tr = traffic.get("ckpt_plan_kernel")
        info = plan.info()
        roofline = {"bound": "hbm", "kernel": "ckpt_plan_kernel<BF16,E4M3> (amax and cast phases per tensor group, "
                                              "the cast phase re-reading its group from L2)",
                    "alg_bytes_per_launch": int(one_pass_bytes),
                    "alg_bytes_basis": "3 B/param: BF16 read once from DRAM + E4M3 written once (the single-pass "
                                       "bound); the cast phase's second read of each group is served by L2",
                    "launch_ms": round(run_ms, 4), "achieved": round(achieved, 1), "peak": peak,
                    "peak_source": peak_src, "unit": "GB/s", "frac": round(achieved / peak, 4),
                    "frac_of_8tbs": round(achieved / NOMINAL_HBM_GBS, 4),
                    "traffic": int(tr * local_params) if tr else None,
                    "direction_ceiling": ceilings["read2_write1"],
                    "frac_of_direction_ceiling": round(achieved / ceilings["read2_write1"]["gbs"], 4),
                    "groups": info["groups"], "grid": info["grid"], "group_mb": args.group_mb}
    # the two-pass path (mf_ckpt_quant_fp8: amax pass, NCCL all-reduce, cast pass) on the same buffers, for
    # comparison: its phases and each pass alone
    breakdown = step_breakdown(torch, dist, chunks, entries, specs, amax, sinv, comm, stream)

    def cast_only():
        call("mf_ckpt_cast_pass", chunks, len(entries), len(specs), amax.data_ptr(), sinv.data_ptr(), E4M3, 0,
             stream)

    def amax_only():
        call("mf_ckpt_amax_pass", chunks, len(entries), len(specs), amax.data_ptr(), stream)

    cast_ms = statistics.mean(time_launches(torch, cast_only, 10))
    amax_ms = statistics.mean(time_launches(torch, amax_only, 10))
    cast_gbs = one_pass_bytes / (cast_ms * 1e-3) / 1e9
    amax_gbs = 2.0 * local_params / (amax_ms * 1e-3) / 1e9
    tr = traffic.get("ckpt_cast_pass")
    two_pass = {"cast_pass": {"kernel": "stream_kernel<CastOp<BF16,E4M3>> (read BF16, write E4M3)",
                              "launch_ms": round(cast_ms, 4), "gbs": round(cast_gbs, 1),
                              "frac": round(cast_gbs / peak, 4),
                              "frac_of_direction_ceiling": round(cast_gbs / ceilings["read2_write1"]["gbs"], 4),
                              "traffic": int(tr * local_params) if tr else None},
                "amax_pass": {"kernel": "stream_amax_kernel<BF16> (read BF16)", "launch_ms": round(amax_ms, 4),
                              "gbs": round(amax_gbs, 1), "frac": round(amax_gbs / peak, 4),
                              "frac_of_direction_ceiling": round(amax_gbs / ceilings["read_only"]["gbs"], 4)},
                "step": breakdown}
    if plan is None:
        roofline = {"bound": "hbm", "kernel": two_pass["cast_pass"]["kernel"], "alg_bytes_per_launch": int(one_pass_bytes),
                    "launch_ms": round(cast_ms, 4), "achieved": round(cast_gbs, 1), "peak": peak,
                    "peak_source": peak_src, "unit": "GB/s", "frac": round(cast_gbs / peak, 4),
                    "frac_of_8tbs": round(cast_gbs / NOMINAL_HBM_GBS, 4),
                    "traffic": int(tr * local_params) if tr else None,
                    "direction_ceiling": ceilings["read2_write1"],
                    "frac_of_direction_ceiling": round(cast_gbs / ceilings["read2_write1"]["gbs"], 4)}

    # the sharded result of one more step, checked outside the timed region
    step()
    torch.cuda.synchronize()
    parity = check_parity(torch, dist, specs, local, src, dst, amax, sinv)

    # end to end through the C ABI with host buffers
    e2e = bench_e2e(args, torch, dist, chunks, entries, specs, src, dst, amax, sinv, comm, stream, local_params,
                    total_params)

    kernels = None
    cpu = None
    if world == 1 and not args.no_kernels:
        kernels = bench_kernels(torch, stream, peak, tuple(args.kernels.split(",")))
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        cpu = cpu_baseline(steps=2, warmup=0)
        if kernels:
            for key, c in cpu_kernel_baselines(tuple(args.kernels.split(","))).items():
                kernels[key]["cpu"] = c

    if comm is not None:
        comm.close()
    if plan is not None:
        dist.barrier(torch)  # every rank's last run has finished before any exchange buffer goes away
        plan.close()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "elems/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0, 0.02) BF16 weights)",
            "config": {"workload": "ckpt_fp8_e4m3_llama3_8b" if full else
                       f"ckpt_fp8_e4m3_reduced_layers{args.ckpt_layers}_vocab{args.ckpt_vocab} (profiling size)",
                       "description": "whole-checkpoint per-tensor amax-scaled FP8 E4M3 quantisation, Llama-3-8B "
                                      "layout (291 BF16 tensors), rows split over ranks; "
                                      + {"plan": "one launch per step, per-group amax exchanged between ranks "
                                                 "inside the kernel over NVLink peer memory",
                                         "passes": "two launches per step: the amax pass, whose last CTA "
                                                   "publishes the rank's maxima into every rank's exchange buffer "
                                                   "over NVLink peer memory, and the cast pass, which waits for "
                                                   "every rank's flag inside the kernel (no collective call, no "
                                                   "memset, no scale_inv launch)",
                                         "twopass": "amax pass, NCCL max all-reduce, cast pass"}[args.path],
                       "path": args.path,
                       "tensors": len(specs), "params": total_params, "src_dtype": "bf16", "dst_dtype": "fp8e4m3",
                       "compat": "reference", "parallelism": f"rowsplit{world}",
                       "l2": "inputs larger than L2 (BF16 shard of 16.06 GB / N per rank)"},
            "hbm_gbs_job": round(job_gbs, 1), "alg_bytes_per_param": 3,
            "roofline": roofline, "e2e": e2e, "clocks": clocks,
            "gpu_launches": {"plan": 1, "passes": 2, "twopass": 3}[args.path] * args.steps,
            "parity": parity, "two_pass": two_pass, "ceilings": ceilings,
        }
        if passes:
            line["passes"] = passes
        if kernels:
            line["kernels"] = kernels
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    dist.close()
    if not parity["ok"]:
        sys.exit(3)


def passes_breakdown(torch, dist, plan, amax, sinv, stream, reps: int = 10) -> dict:
    """The plan's two-launch step as its two launches, a CUDA event between them, median over `reps` steps,
    max over ranks per phase (every rank runs the same launches)."""
    torch.cuda.synchronize()
    dist.barrier(torch)
    rows = []
    for _ in range(reps):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record()
        plan.run_passes(amax.data_ptr(), sinv.data_ptr(), stream, passes=1)
        ev[1].record()
        plan.run_passes(amax.data_ptr(), sinv.data_ptr(), stream, passes=2)
        ev[2].record()
        rows.append(ev)
    torch.cuda.synchronize()
    out = {}
    for k, name in enumerate(["amax_pass_ms", "cast_pass_ms"]):
        out[name] = round(dist.max(torch, statistics.median(r[k].elapsed_time(r[k + 1]) for r in rows)), 4)
    out["step_ms"] = round(dist.max(torch, statistics.median(r[0].elapsed_time(r[2]) for r in rows)), 4)
    out["path"] = ("mf_ckpt_plan_run_passes: stream_amax_kernel (its last CTA publishes the rank's maxima) + "
                   "stream_kernel<CastXOp> (waits for every rank's flag, then casts; writes amax and scale_inv)")
    return out


def step_breakdown(torch, dist, chunks, entries, specs, amax, sinv, comm, stream, reps: int = 10) -> dict:
    """One step as its phases -- memset, pass 1, all-reduce, pass 2 -- with a CUDA event between each,
    median over `reps` steps, max over ranks per phase (every rank runs the same phases)."""
    from manifesto_b200._abi import call
    torch.cuda.synchronize()
    dist.barrier(torch)
    rows = []
    for _ in range(reps):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
        ev[0].record()
        amax.zero_()
        ev[1].record()
        call("mf_ckpt_amax_pass", chunks, len(entries), len(specs), amax.data_ptr(), stream)
        ev[2].record()
        if comm is not None:
            comm.allreduce_max(amax.data_ptr(), len(specs), stream)
        ev[3].record()
        call("mf_ckpt_cast_pass", chunks, len(entries), len(specs), amax.data_ptr(), sinv.data_ptr(), E4M3, 0,
             stream)
        ev[4].record()
        rows.append(ev)
    torch.cuda.synchronize()
    names = ["memset_ms", "amax_pass_ms", "allreduce_ms", "cast_pass_ms"]
    out = {}
    for k, name in enumerate(names):
        out[name] = round(dist.max(torch, statistics.median(r[k].elapsed_time(r[k + 1]) for r in rows)), 4)
    out["step_ms"] = round(dist.max(torch, statistics.median(r[0].elapsed_time(r[4]) for r in rows)), 4)
    out["outside_kernels_ms"] = round(out["step_ms"] - out["amax_pass_ms"] - out["cast_pass_ms"], 4)
    out["path"] = "mf_ckpt_amax_pass + NCCL max all-reduce (mf_comm_allreduce_max_f32) + mf_ckpt_cast_pass"
    return out


PARITY_TENSORS = ("model.layers.0.self_attn.q_proj.weight", "model.layers.0.mlp.down_proj.weight",
                  "model.layers.0.input_layernorm.weight", "lm_head.weight")


def check_parity(torch, dist, specs, local, src, dst, amax, sinv) -> dict:
    """Check the sharded result after a step, outside the timed region, on every rank:
    * the all-reduced amax vector equals, bit for bit, a torch.distributed MAX all-reduce of each
      rank's own max|v| per tensor (torch on the device);
    * every scale_inv equals the oracle's amax / 448 of that global amax;
    * this rank's FP8 codes of four tensors (a q_proj, a down_proj, a norm and lm_head) equal the
      CPU oracle's restatement of NewF8E4M3FromFloat32(v * 448 / amax) (dtype/fp8.go:77-136) on
      this rank's rows at the global amax.
    The oracle is the checker only; nothing timed runs through it."""
    import numpy as np

    from oracle import ref
    offs = [0]
    for n in local:
        offs.append(offs[-1] + n)
    want = torch.zeros(len(specs), dtype=torch.float32, device="cuda")
    for t, n in enumerate(local):
        if n:
            want[t] = src[offs[t]:offs[t] + n].abs().max().float()
    if dist.pg:
        dist.pg.all_reduce(want, op=dist.pg.ReduceOp.MAX)
    amax_ok = bool(torch.equal(amax.view(torch.int32), want.view(torch.int32)))
    want_h = want.cpu().numpy()
    si_h = sinv.cpu().numpy()
    si_bad = [t for t in range(len(specs)) if float(si_h[t]) != ref.fp8_scale_inv(float(want_h[t]), ref.E4M3)]
    threads = max(1, (os.cpu_count() or 1) // max(1, dist.world))
    names = [s.name for s in specs]
    checked, bad, elems = [], [], 0
    for name in PARITY_TENSORS:
        if name not in names:
            continue
        t = names.index(name)
        o, n = offs[t], local[t]
        checked.append(name)
        if not n:
            continue
        raw = src[o:o + n].view(torch.int16).cpu().numpy().view(np.uint16)
        got = dst[o:o + n].cpu().numpy()
        if not np.array_equal(got, ref.scaled_cast(raw, ref.BF16, ref.E4M3, float(want_h[t]), threads=threads)):
            bad.append(name)
        elems += n
    ok_local = amax_ok and not si_bad and not bad
    ok = dist.max(torch, 0.0 if ok_local else 1.0) == 0.0
    elems_all = int(dist.max(torch, float(elems))) if dist.pg else elems
    return {"ok": ok, "ranks_checked": dist.world,
            "amax_vs_torch_allreduce": "bit-exact" if amax_ok else "MISMATCH",
            "scale_inv_mismatches": len(si_bad), "tensors_checked": checked, "tensor_mismatches": bad,
            "fp8_elements_checked_on_rank0": elems, "fp8_elements_checked_max_rank": elems_all,
            "checker": "oracle/mfref.c (C restatement of dtype/fp8.go:77-136), after the timed region"}


def bench_e2e(args, torch, dist, chunks, entries, specs, src, dst, amax, sinv, comm, stream, local_params,
              total_params) -> dict:
    """Host BF16 (pinned) -> device -> quantise -> FP8 + scale_inv -> host, every step.

    Runs through checkpoint.StreamedQuantiser (the library's API for host-resident
    checkpoints): batches of whole tensors go up, through the two passes and back
    down on three streams over two device slots, so downloads overlap uploads.
    """
    from manifesto_b200 import Event, PinnedBuffer, checkpoint
    from manifesto_b200._abi import call

    h_src = PinnedBuffer(2 * local_params)
    h_dst = PinnedBuffer(local_params)
    h_si = PinnedBuffer(4 * len(specs))
    # the host copy holds the same weights the device holds
    call("mf_memcpy_d2h_async", h_src.ptr, src.data_ptr(), 2 * local_params, stream)
    torch.cuda.synchronize()
    sizes = [e[2] for e in entries]
    # batches of whole tensors cut by the global tensor sizes, identical on every rank
    q = checkpoint.StreamedQuantiser(sizes, comm=comm, batch_sizes=[s.numel for s in specs])
    steps = max(2, min(args.steps, args.e2e_steps))
    link = link_ceiling(torch, dist, q, h_src, h_dst, src, dst, local_params)
    for _ in range(2):  # warm-up: both slots once
        q.submit(h_src.ptr, h_dst.ptr, h_si.ptr)
    q.synchronize()
    dist.barrier(torch)
    t0, t1 = Event(timing=True), Event(timing=True)
    t0.record(q.up)
    q.compute.wait(t0)
    q.down.wait(t0)
    for _ in range(steps):
        q.submit(h_src.ptr, h_dst.ptr, h_si.ptr)
    t1.record(q.down)
    q.synchronize()
    t1.sync()
    ms = dist.max(torch, t0.elapsed_ms(t1))
    q.close()
    for ev in (t0, t1):
        ev.close()
    for b in (h_src, h_dst, h_si):
        b.free()
    return {"value": total_params * steps / (ms * 1e-3), "unit": "elems/s", "steps": steps,
            "ms_per_step": ms / steps, "h2d_bytes_per_step": 2 * local_params,
            "d2h_bytes_per_step": local_params + 4 * len(specs),
            "link_ceiling_gbs": link["gbs"], "link_ceiling": link,
            "frac_of_link_ceiling": round(link["ms"] / (ms / steps), 4),
            "path": "C ABI via checkpoint.StreamedQuantiser (1 GB tensor batches; upload / kernels / download "
                    "streams over 2 slots)"}


def link_ceiling(torch, dist, q, h_src, h_dst, src, dst, local_params: int, reps: int = 2) -> dict:
    """Bare pinned copies of one e2e step's bytes -- BF16 host -> device on the upload stream while the
    FP8 bytes go device -> host on the download stream -- on every rank at once (the N ranks share
    the host's links).  Best of `reps`, max over ranks: the floor under the e2e step time."""
    from manifesto_b200 import Event
    from manifesto_b200._abi import call
    best = None
    for _ in range(reps):
        q.synchronize()
        dist.barrier(torch)
        t0, tu, td = Event(timing=True), Event(timing=True), Event(timing=True)
        t0.record(q.up)
        q.down.wait(t0)
        call("mf_memcpy_h2d_async", src.data_ptr(), h_src.ptr, 2 * local_params, q.up.handle)
        call("mf_memcpy_d2h_async", h_dst.ptr, dst.data_ptr(), local_params, q.down.handle)
        tu.record(q.up)
        td.record(q.down)
        q.synchronize()
        ms = max(t0.elapsed_ms(tu), t0.elapsed_ms(td))
        for ev in (t0, tu, td):
            ev.close()
        best = ms if best is None else min(best, ms)
    ms = dist.max(torch, best)
    nbytes = 3 * local_params
    return {"ms": round(ms, 3), "h2d_bytes": 2 * local_params, "d2h_bytes": local_params,
            "gbs": round(nbytes / (ms * 1e-3) / 1e9, 2), "gbs_all_ranks": round(nbytes * dist.world / (ms * 1e-3) / 1e9, 2),
            "how": "pinned H2D and D2H of one step's bytes at once, every rank together, best of 2, max over ranks"}


# ------------------------------------------------------ CPU / reference

CPU_SAMPLE = ("the embedding matrix plus decoder layer 0 of the Llama-3-8B layout: 10 BF16 tensors, "
              "743,448,576 params, N(0, 0.02)")


def cpu_sample():
    from manifesto_b200 import checkpoint, synthetic
    specs = checkpoint.llama3_8b_layout()[0:10]
    assert specs[0].name == "model.embed_tokens.weight"
    assert all(s.name.startswith("model.layers.0.") for s in specs[1:])
    threads = os.cpu_count() or 1
    return [synthetic.normal_bf16_large(2000 + i, s.numel, 0.0, 0.02, threads=threads) for i, s in enumerate(specs)]


def cpu_step(tensors, threads: int) -> None:
    from oracle import ref
    for t in tensors:
        a = ref.amax(t, ref.BF16, threads=threads)
        ref.scaled_cast(t, ref.BF16, ref.E4M3, a, threads=threads)


def cpu_baseline(steps: int, warmup: int, tensors=None) -> dict:
    tensors = tensors if tensors is not None else cpu_sample()
    threads = os.cpu_count() or 1
    n = sum(int(t.size) for t in tensors)
    for _ in range(warmup):
        cpu_step(tensors, threads)
    t = time.perf_counter()
    for _ in range(steps):
        cpu_step(tensors, threads)
    dt = (time.perf_counter() - t) / steps
    # the Go loops are single-goroutine: one thread on one tensor of the sample (layer 0's q_proj), too
    one = tensors[1]
    t = time.perf_counter()
    cpu_step([one], 1)
    dt1 = time.perf_counter() - t
    return {"value": n / dt, "unit": "elems/s", "cores": threads, "kind": "port", "sample": CPU_SAMPLE,
            "s_per_step": dt, "cpu": cpu_model(),
            "single_thread": {"value": one.size / dt1, "unit": "elems/s", "cores": 1,
                              "sample": f"layer 0's q_proj ({one.size:,} params), one pass"}}


def _cpu_time(fn, threads: int) -> float:
    fn(threads)  # warm: page in the output, build the thread pool
    t = time.perf_counter()
    fn(threads)
    return time.perf_counter() - t


def cpu_kernel_baselines(which=KERNEL_CONFIGS) -> dict:
    """The oracle's C restatement of each config's Go loop on a bounded sample of that config, with the
    config's value distribution: on every host thread and on one (the Go loops are single-goroutine)."""
    import numpy as np

    from manifesto_b200 import fusion, synthetic
    from oracle import ref
    cores = os.cpu_count() or 1
    out = {}

    def leg(key, n, fn, sample):
        t_all, t_one = _cpu_time(fn, cores), _cpu_time(fn, 1)
        out[key] = {"elems_per_s": n / t_all, "cores": cores, "single_thread_elems_per_s": n / t_one,
                    "kind": "port", "sample": sample}

    if "c1" in which:
        n = 1 << 24
        b = synthetic.uniform_bytes(0x5EED0001, n)
        leg("c1_fp8e4m3_to_f32", n, lambda th: ref.convert(b, ref.E4M3, ref.F32, threads=th),
            "convert.BytesToFloat32 (E4M3) over 2^24 uniform bytes (a quarter of config 1)")
    if "c2" in which:
        rows, cols, group = 512, 14336, 128
        q = synthetic.uniform_bytes(0x5EED0002, rows * cols // 2)
        sc = synthetic.abs_normal_bf16(0x5EED1002, rows * cols // group, 0.02)
        leg("c2_int4_to_bf16", rows * cols,
            lambda th: ref.int4_dequant(q, sc, ref.BF16, ref.BF16, rows, cols, group, threads=th),
            "Int4 group dequant of 512 of the 4096 rows of config 2 (14336 cols, group 128)")
    if "c3" in which:
        n = 1 << 24
        x, y = synthetic.normal_f32(0x5EED0003, n), synthetic.normal_f32(0x5EED1003, n)
        leg("c3a_axpy_f32", n, lambda th: ref.axpy(y.copy(), x, 0.75, ref.F32, threads=th),
            "axpyOntoHost f32 over 2^24 elements (1/16 of config 3), copy of y included")
        xb, yb = synthetic.f32_to_bf16_bits(x), synthetic.f32_to_bf16_bits(y)
        leg("c3b_axpy_bf16", n, lambda th: ref.axpy(yb.copy(), xb, 0.75, ref.BF16, threads=th),
            "axpyOntoHost bf16 over 2^24 elements (1/16 of config 3), copy of y included")
    if "c3s" in which:
        n = 1 << 24
        x = synthetic.normal_f32(0x5EED0013, n)
        leg("c3s_scalar_mul_f32", n, lambda th: ref.scalar_broadcast(x, ref.F32, ref.F32, 0.75, 2, threads=th),
            "applyScalarBroadcast (mul) f32 over 2^24 elements (1/16 of the bench's 2^28)")
        xb = synthetic.f32_to_bf16_bits(x)
        leg("c3s_scalar_mul_bf16", n, lambda th: ref.scalar_broadcast(xb, ref.BF16, ref.BF16, 0.75, 2, threads=th),
            "applyScalarBroadcast (mul) bf16 over 2^24 elements (1/16 of the bench's 2^28)")
    if "c4" in which:
        hidden, n = 4096, 1 << 22
        ins = [synthetic.normal_bf16(0x5EED0004, n), synthetic.normal_bf16(0x5EED1004, hidden, 1.0, 0.1),
               synthetic.normal_bf16(0x5EED2004, hidden, 0.0, 0.1), synthetic.normal_bf16(0x5EED3004, n)]
        tree = fusion.node_table(fusion.swiglu_chain().root)

        def c4(th):
            pre = ref.fused_eval(tree, ins, [ref.BF16] * 4, [0, hidden, hidden, 0], ref.BF16, n, threads=th)
            ref.scaled_cast(pre, ref.BF16, ref.E4M3, ref.amax(pre, ref.BF16, threads=th), threads=th)
        leg("c4_fused_swiglu_fp8", n, c4,
            "evalCPU of Mul(Silu(Add(Mul(x,g),b)),y) to BF16, amax, scaled E4M3 cast over 2^22 elements "
            "(1/128 of config 4)")
    if "c4g" in which:
        hidden, n = 4096, 1 << 22
        ins = [synthetic.normal_bf16(0x5EED0014, n), synthetic.normal_bf16(0x5EED1014, hidden, 1.0, 0.1),
               synthetic.normal_bf16(0x5EED2014, hidden, 0.0, 0.1)]
        tree = fusion.node_table(fusion.gelu_affine_chain().root)
        leg("c4g_fused_gelu_generic", n,
            lambda th: ref.fused_eval(tree, ins, [ref.BF16] * 3, [0, hidden, hidden], ref.BF16, n, threads=th),
            "evalCPU of Gelu(Add(Mul(x,g),b)) to BF16 over 2^22 elements (1/128 of config 4's shape)")
    return out


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args, world: int, rank: int) -> None:
    if rank != 0:
        return
    from oracle import ref
    ref.lib()
    tensors = cpu_sample()
    b = cpu_baseline(steps=args.steps, warmup=args.warmup, tensors=tensors)
    line = {
        "metric": METRIC, "value": b["value"], "unit": "elems/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": b["s_per_step"] * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0, 0.02) BF16 weights)",
        "config": {"workload": "ckpt_fp8_e4m3_llama3_8b", "params": 8030261248, "src_dtype": "bf16",
                   "dst_dtype": "fp8e4m3", "compat": "reference", "sample": CPU_SAMPLE},
        "impl": "reference",
        "cpu_baseline": {"value": b["value"], "unit": "elems/s", "cores": b["cores"], "kind": "port",
                         "sample": CPU_SAMPLE, "cpu": b["cpu"], "single_thread": b["single_thread"]},
        "e2e": {"value": b["value"], "unit": "elems/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "manifesto is Go and no Go toolchain exists here; this times the C restatement of its scalar "
                "loops (oracle/mfref.c) with all host threads",
    }
    print(json.dumps(line), flush=True)


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-kernels", action="store_true", help="skip the per-config kernel lines (N=1)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kernels", default=",".join(KERNEL_CONFIGS),
                    help="comma list of per-config kernel lines to run at N=1 (c1,c2,c3,c4,c4g)")
    ap.add_argument("--only-kernels", action="store_true",
                    help="run only the per-config kernel lines (profiling); --steps sets the repetitions")
    ap.add_argument("--path", choices=["auto", "plan", "passes", "twopass"], default="auto",
                    help="checkpoint step: the plan in one launch (mf_ckpt_plan_run), the plan in two launches with "
                         "the amax exchange fused into them (mf_ckpt_plan_run_passes), or mf_ckpt_quant_fp8 (amax "
                         "pass, NCCL all-reduce, cast pass); auto: twopass on one GPU (nothing to exchange), passes "
                         "on several")
    ap.add_argument("--group-mb", type=float, default=32.0, help="plan: source MB per tensor group (L2 budget)")
    ap.add_argument("--ckpt-layers", type=int, default=32, help="decoder layers of the checkpoint (profiling only)")
    ap.add_argument("--ckpt-vocab", type=int, default=128256, help="vocabulary rows (profiling only)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and world == 1 and args.gpus > 1:
        print(f"--gpus {args.gpus} needs torchrun with {args.gpus} processes", file=sys.stderr)
        return 2
    if args.impl == "reference":
        run_reference(args, world, rank)
    else:
        run_ours(args, world, rank, local_rank)
    return 0


if __name__ == "__main__":
    sys.exit(main())
