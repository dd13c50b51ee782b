#!/usr/bin/env python
"""Benchmark of the tvarant B200 backend (one JSON line on rank 0).

Default workload, at every number of GPUs — the Llama-7B-shaped gated-SiLU
MLP stack (32 layers, d_model 4096, d_ff 11008, 8192 tokens, TF32),
tensor-parallel over the ranks (gate/up column shards, down row shards, one
all-reduce of the layer output per layer).  A step is one pass of the stack
over the 8192 tokens.

* ``value``: tokens/s of the whole job (strong scaling: the same 8192 tokens
  at every N), the step replayed from a CUDA graph, inputs resident.
* ``e2e``: the same through the same API with the activations copied in from
  pinned host memory and the result copied back every step.
* ``roofline``: the stack's dominant kernel, the SwiGLU GEMM at the stack's
  shard and chunk shape, timed back to back with events on its stream,
  against the TF32 dense peak measured with cuBLAS in this run (and against
  half the measured bf16 peak, a fixed figure).
* ``cpu_baseline``: the reference's own simulator kernels (HostKernels.cpp,
  built into oracle/_ref) running one MLP layer on a token sample, all host
  cores, with the single-thread figure beside it.

On one GPU the line also carries, under ``config``, the fused-GEMM sweep's
largest point (linear+bias+SiLU M=16384 K=N=4096 with the sub/exp/neg/abs
chain in the GEMM epilogue, TF32 and 3xTF32) and the memory-bound LLM op set
(softmax, layer norm, embedding, bmm) with each op's fraction of HBM.

``--workload gemm`` gives the fused-GEMM line alone, ``--workload sweep``
the whole sweep (M in {1, 16, 128, 1024, 4096, 16384}, TF32 and 3xTF32);
``llm-ops | bmm | gpt2 | gpt2-decode | llama-ops`` the other workloads.

``--impl reference`` times the reference's CPU implementation of the same
workload (rank 0 only) and prints the line with ``"impl": "reference"``.
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

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "fused-GEMM TFLOP/s (% peak); LLM-op GB/s (% HBM); tokens/s at 1/2/4/8 GPU"
M_DEFAULT, K_DEFAULT, N_DEFAULT = 16384, 4096, 4096
L2_FLUSH_BYTES = 256 << 20  # twice the B200's 126 MB L2


def _env_rank():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def _peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text())
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def _traffic(key: str):
    p = ROOT / "profiles" / "ncu_traffic.json"
    if p.exists():
        return json.loads(p.read_text()).get(key)
    return None


class ClockSampler:
    """Polls SM clock and throttle reasons through NVML (every ~5 ms) while
    the timed region runs; summary() keeps the samples taken inside it."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, local_rank: int):
        self.local_rank = local_rank
        self.samples: list[tuple[float, float, float, int]] = []
        self.windows: list[tuple[float, float]] = []
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None
        self._handle = None

    def _open(self):
        import pynvml

        pynvml.nvmlInit()
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        entries = [v.strip() for v in vis.split(",") if v.strip()]
        if entries and self.local_rank < len(entries):
            e = entries[self.local_rank]
            if e.isdigit():
                handle = pynvml.nvmlDeviceGetHandleByIndex(int(e))
            else:
                handle = pynvml.nvmlDeviceGetHandleByUUID(e)
        else:
            handle = pynvml.nvmlDeviceGetHandleByIndex(self.local_rank)
        self._nvml, self._handle = pynvml, handle

    def _poll(self):
        nv, h = self._nvml, self._handle
        max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        while not self._stop.is_set():
            try:
                mhz = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                try:
                    bits = int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))
                except AttributeError:
                    bits = int(nv.nvmlDeviceGetCurrentClocksThrottleReasons(h))
                self.samples.append((time.perf_counter(), mhz, max_mhz, bits))
            except Exception:
                pass
            time.sleep(0.005)

    def __enter__(self):
        try:
            self._open()
            self._thread = threading.Thread(target=self._poll, daemon=True)
            self._thread.start()
            t0 = time.perf_counter()
            while not self.samples and time.perf_counter() - t0 < 2.0:
                time.sleep(0.005)
        except Exception:
            self._nvml = None
        return self

    def mark(self, start: float, end: float):
        """Adds a timed window; summary() keeps the samples inside any window."""
        self.windows.append((start, end))

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)
        return False

    def summary(self) -> dict:
        pts = self.samples
        if self.windows:
            inside = [p for p in pts if any(a <= p[0] <= b for a, b in self.windows)]
            pts = inside or pts[-3:]
        if not pts:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                    "source": "unavailable"}
        reasons = set()
        for _, _, _, bits in pts:
            for bit, name in self.REASONS.items():
                if bits & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(p[1] for p in pts), "sm_max_mhz": max(p[2] for p in pts),
                "reasons": sorted(reasons), "samples": len(pts), "source": "NVML, 5 ms polling"}


# ------------------------------------------------------------------ CPU side

def _cpu_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def reference_gemm_chain_rows(rows: int, threads: int, seed: int = 0) -> tuple[float, float]:
    """Times the reference simulator path (HostKernels gemm_bias_act + the
    eager sub/exp/neg/abs) on `rows` rows of the workload split over
    `threads` host threads.  Returns (seconds, flops)."""
    import ctypes
    from concurrent.futures import ThreadPoolExecutor

    import numpy as np

    import oracle

    impl = "ref" if oracle.available("ref") else "port"
    lib = oracle._lib(impl)
    pre = "ref_" if impl == "ref" else "tvo_"
    gemm = getattr(lib, pre + "gemm_bias_act")
    unary = getattr(lib, pre + "unary")
    binary = getattr(lib, pre + "binary")
    rng = np.random.default_rng(seed)
    K, N = K_DEFAULT, N_DEFAULT
    x = rng.standard_normal((rows, K), dtype=np.float32)
    w = rng.uniform(-1 / 64, 1 / 64, (N, K)).astype(np.float32)
    b = rng.uniform(-1 / 64, 1 / 64, N).astype(np.float32)
    z = rng.standard_normal((rows, N), dtype=np.float32)
    y = np.empty((rows, N), np.float32)
    t1 = np.empty_like(y)
    t2 = np.empty_like(y)
    chunks = np.array_split(np.arange(rows), max(1, min(threads, rows)))

    def work(idx):
        r0, r1 = int(idx[0]), int(idx[-1]) + 1
        n = r1 - r0
        p = lambda arr: ctypes.c_void_p(arr[r0:r1].ctypes.data)  # noqa: E731
        gemm(p(x), ctypes.c_void_p(w.ctypes.data), ctypes.c_void_p(b.ctypes.data), p(y), n, N, K,
             1.0, 1.0, 2, 1)
        binary(0, p(y), p(z), p(t1), n * N, -1.0)   # sub = add with -alpha
        unary(4, p(t1), p(t2), n * N, 0.0)          # exp
        unary(2, p(t2), p(t1), n * N, 0.0)          # neg
        unary(3, p(t1), p(t2), n * N, 0.0)          # abs

    t0 = time.perf_counter()
    with ThreadPoolExecutor(max_workers=len(chunks)) as ex:
        list(ex.map(work, chunks))
    return time.perf_counter() - t0, 2.0 * rows * N * K


def cpu_baseline_gemm(budget_s: float = 12.0) -> dict:
    threads = _cpu_cores()
    rows = max(threads, 8)
    dt, fl = reference_gemm_chain_rows(rows, threads)
    # grow the sample toward the time budget
    rows2 = int(min(M_DEFAULT, max(rows, rows * budget_s / max(dt, 1e-3) * 0.5)))
    if rows2 > rows:
        dt, fl = reference_gemm_chain_rows(rows2, threads)
        rows = rows2
    dt1, fl1 = reference_gemm_chain_rows(4, 1)
    return {"value": fl / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "reference",
            "sample": f"{rows} of {M_DEFAULT} rows of the GEMM+SiLU and the sub/exp/neg/abs chain, "
                      f"reference HostKernels.cpp compiled in oracle/_ref, {threads} threads",
            "single_thread": {"value": fl1 / dt1 / 1e12, "unit": "TFLOP/s", "cores": 1,
                              "sample": "4 rows, 1 thread (the simulator has no parallel loops)"}}


D_MODEL, D_FF, MLP_LAYERS, MLP_TOKENS = 4096, 11008, 32, 8192
_MLP_REF_WEIGHTS = None


def _mlp_ref_weights():
    """One layer's gate, up and down weights ~N(0, 0.02), drawn once."""
    global _MLP_REF_WEIGHTS
    if _MLP_REF_WEIGHTS is None:
        import numpy as np

        rng = np.random.default_rng(0)
        _MLP_REF_WEIGHTS = tuple(0.02 * rng.standard_normal(shape, dtype=np.float32)
                                 for shape in ((D_FF, D_MODEL), (D_FF, D_MODEL),
                                               (D_MODEL, D_FF)))
    return _MLP_REF_WEIGHTS


def reference_mlp_rows(rows: int, threads: int, seed: int = 7) -> float:
    """Seconds for one gated-SiLU MLP layer of the reference path on ``rows``
    tokens split over ``threads`` host threads: HostKernels gemm_bias_act with
    SiLU (gate), gemm_bias_act (up), the eager elementwise product, and
    gemm_bias_act (down), as the reference runs
    ``linear(linear_act(x, Wg, None, "silu") * linear(x, Wu), Wd)``."""
    import ctypes
    from concurrent.futures import ThreadPoolExecutor

    import numpy as np

    import oracle

    impl = "ref" if oracle.available("ref") else "port"
    lib = oracle._lib(impl)
    pre = "ref_" if impl == "ref" else "tvo_"
    gemm = getattr(lib, pre + "gemm_bias_act")
    binary = getattr(lib, pre + "binary")
    wg, wu, wd = _mlp_ref_weights()
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, D_MODEL), dtype=np.float32)
    g = np.empty((rows, D_FF), np.float32)
    u = np.empty_like(g)
    h = np.empty_like(g)
    y = np.empty((rows, D_MODEL), np.float32)
    chunks = np.array_split(np.arange(rows), max(1, min(threads, rows)))
    vp = ctypes.c_void_p

    def work(idx):
        r0, r1 = int(idx[0]), int(idx[-1]) + 1
        n = r1 - r0
        p = lambda arr: vp(arr[r0:r1].ctypes.data)  # noqa: E731
        gemm(p(x), vp(wg.ctypes.data), None, p(g), n, D_FF, D_MODEL, 1.0, 0.0, 2, 1)
        gemm(p(x), vp(wu.ctypes.data), None, p(u), n, D_FF, D_MODEL, 1.0, 0.0, 0, 1)
        binary(1, p(g), p(u), p(h), n * D_FF, 1.0)
        gemm(p(h), vp(wd.ctypes.data), None, p(y), n, D_MODEL, D_FF, 1.0, 0.0, 0, 1)

    t0 = time.perf_counter()
    with ThreadPoolExecutor(max_workers=len(chunks)) as ex:
        list(ex.map(work, chunks))
    return time.perf_counter() - t0


def cpu_baseline_mlp(budget_s: float = 12.0) -> dict:
    """The reference's MLP layer on a token sample sized toward ``budget_s``,
    all host threads, as tokens/s of the whole 32-layer stack; plus the same
    on one thread (the simulator's own setting: it has no parallel loops)."""
    threads = _cpu_cores()
    rows = max(2 * threads, 16)
    dt = reference_mlp_rows(rows, threads)
    rows2 = int(min(MLP_TOKENS, max(rows, rows * budget_s / max(dt, 1e-3) * 0.5)))
    if rows2 > rows:
        dt = reference_mlp_rows(rows2, threads)
        rows = rows2
    single_rows = 4
    dt1 = reference_mlp_rows(single_rows, 1)
    return {"value": rows / (dt * MLP_LAYERS), "unit": "tokens/s", "cores": threads,
            "kind": "reference",
            "sample": f"one gated-SiLU MLP layer (4096 -> 11008 -> 4096) on {rows} of "
                      f"{MLP_TOKENS} tokens, reference HostKernels.cpp compiled in oracle/_ref, "
                      f"{threads} threads; tokens/s of the {MLP_LAYERS}-layer stack = tokens / "
                      f"({MLP_LAYERS} x layer time)",
            "single_thread": {"value": single_rows / (dt1 * MLP_LAYERS), "unit": "tokens/s",
                              "cores": 1, "sample": f"{single_rows} tokens, one layer, 1 thread"}}


# ------------------------------------------------------------------ GPU side

def _device_setup(local_rank: int):
    import torch

    import torch_tvarant  # noqa: F401

    torch.tvarant.set_device(local_rank)
    return torch


def tf32_peak_tflops(torch) -> float | None:
    """cuBLAS TF32 GEMM 8192^3 on this GPU (burst, best of 5)."""
    if not torch.cuda.is_available():
        return None
    try:
        torch.backends.cuda.matmul.allow_tf32 = True
        n = 8192
        a = torch.randn(n, n, device="cuda")
        b = torch.randn(n, n, device="cuda")
        for _ in range(3):
            torch.matmul(a, b)
        best = None
        for _ in range(5):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            torch.matmul(a, b)
            e1.record()
            torch.cuda.synchronize()
            t = e0.elapsed_time(e1) / 1e3
            best = t if best is None else min(best, t)
        del a, b
        torch.cuda.empty_cache()
        return 2 * n**3 / best / 1e12
    finally:
        torch.backends.cuda.matmul.allow_tf32 = False


class GemmChain:
    """The fused-GEMM sweep workload as a model compiled by the tvarant compiler."""

    def __init__(self, torch, m: int, mode: str):
        import torch.nn as nn
        import torch.nn.functional as F

        import torch_tvarant

        torch.set_float32_matmul_precision("high" if mode == "tf32" else "highest")
        self.m = m

        class Model(nn.Module):
            def __init__(self):
                super().__init__()
                self.lin = nn.Linear(K_DEFAULT, N_DEFAULT)

            def forward(self, x, z):
                y = F.silu(self.lin(x))
                return torch.abs(-torch.exp(y - z))

        g = torch.Generator().manual_seed(0)
        model = Model()
        with torch.no_grad():
            model.lin.weight.uniform_(-1 / 64, 1 / 64, generator=g)
            model.lin.bias.uniform_(-1 / 64, 1 / 64, generator=g)
        # When one step's own operands fit in L2 (small M), consecutive steps
        # rotate over copies of the weight in distinct buffers, more than 256 MB
        # in total, so every step streams its weight from HBM.
        step_bytes = 4 * (m * K_DEFAULT + 2 * m * N_DEFAULT + N_DEFAULT * K_DEFAULT)
        w_bytes = 4 * N_DEFAULT * K_DEFAULT
        self.copies = 1 if step_bytes >= L2_FLUSH_BYTES else -(-L2_FLUSH_BYTES // w_bytes) + 1
        import copy

        self.models = []
        for _ in range(self.copies):
            self.models.append(torch_tvarant.compiler.compile(copy.deepcopy(model).to("tvarant")))
            self.fusions = dict(torch_tvarant.compiler.last_log)
        self.model = self.models[0]
        self.i = 0
        self.x_host = torch.randn(m, K_DEFAULT, generator=g).pin_memory() if torch.cuda.is_available() else torch.randn(m, K_DEFAULT, generator=g)
        self.z_host = torch.randn(m, N_DEFAULT, generator=g).pin_memory() if torch.cuda.is_available() else torch.randn(m, N_DEFAULT, generator=g)
        self.out_host = torch.empty(m, N_DEFAULT).pin_memory() if torch.cuda.is_available() else torch.empty(m, N_DEFAULT)
        self.x = self.x_host.to("tvarant")
        self.z = self.z_host.to("tvarant")
        self.flops = 2.0 * m * N_DEFAULT * K_DEFAULT
        self.h2d_bytes = (self.x_host.numel() + self.z_host.numel()) * 4
        self.d2h_bytes = self.out_host.numel() * 4

    def next_model(self):
        self.i += 1
        return self.models[self.i % self.copies]

    def step_resident(self, torch):
        return self.next_model()(self.x, self.z)

    # End-to-end steps with host buffers.  Inputs are copied in on one stream,
    # the compiled model runs on the current stream and its output is copied
    # out on a third; the device inputs are double-buffered, so step i+1's
    # inputs cross PCIe towards the GPU while step i's output crosses back
    # (the link is full duplex) and step i computes.  Every step still moves
    # all of its inputs and its whole output inside the timed region.
    def e2e_begin(self, torch):
        """Orders the copy streams after the work queued so far (the start
        event of a timed region)."""
        if not hasattr(self, "s_in"):
            self.s_in = torch.Stream(device="tvarant")
            self.s_out = torch.Stream(device="tvarant")
            self.x_dev = [torch.empty_like(self.x) for _ in range(2)]
            self.z_dev = [torch.empty_like(self.z) for _ in range(2)]
            pin = torch.cuda.is_available()
            spare = torch.empty_like(self.out_host)
            self.out_hosts = [self.out_host, spare.pin_memory() if pin else spare]
            self.j = 0
        self.consumed = [None, None]
        start = torch.Event(device="tvarant")
        start.record(torch.tvarant.current_stream())
        self.s_in.wait_event(start)
        self.s_out.wait_event(start)

    def e2e_end(self, torch):
        """Orders the current stream after both copy streams."""
        compute = torch.tvarant.current_stream()
        for s in (self.s_in, self.s_out):
            ev = torch.Event(device="tvarant")
            ev.record(s)
            compute.wait_event(ev)

    def step_e2e(self, torch):
        k = self.j & 1
        self.j += 1
        compute = torch.tvarant.current_stream()
        if self.consumed[k] is not None:
            self.s_in.wait_event(self.consumed[k])  # step i-2 has read buffer k
        with torch.tvarant.stream(self.s_in):
            self.x_dev[k].copy_(self.x_host, non_blocking=True)
            self.z_dev[k].copy_(self.z_host, non_blocking=True)
            landed = torch.Event(device="tvarant")
            landed.record(self.s_in)
        compute.wait_event(landed)
        y = self.next_model()(self.x_dev[k], self.z_dev[k])
        done = torch.Event(device="tvarant")
        done.record(compute)
        self.consumed[k] = done
        self.s_out.wait_event(done)
        with torch.tvarant.stream(self.s_out):
            self.out_hosts[k].copy_(y, non_blocking=True)
        y.record_stream(self.s_out)
        return y


def _dist_init(world: int):
    import torch.distributed as dist

    if world > 1 and not dist.is_initialized():
        import datetime

        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    return dist


def _max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def gemm_kernel_name(m: int, mode: str, program_in_epilogue: bool = False) -> tuple[str, str]:
    """(kernel, bound) that the GEMM of the sweep runs for M rows."""
    if mode == "3xtf32" and m <= 2:
        return "tvr::gemm_skinny_kernel (fp32 FMA GEMV)", "hbm"
    if m <= 128:
        return f"tvr::ws::gemm_ws_kernel ({mode}, weight streaming)", "hbm"
    if program_in_epilogue:
        return (f"tvr::tc::gemm_tc_kernel<256, {mode}, K-major B, PROG> "
                "(abs(neg(exp(Y - Z))) in the epilogue)", "tensor")
    return f"tvr::tc::gemm_tc_kernel<256, {mode}, K-major B>", "tensor"


def program_in_epilogue(m: int, fusions: dict, sms: int = 148) -> bool:
    """Whether the compiled step is one tensor-core launch with the pointwise
    program in its epilogue: the compiler fused the program into the GEMM
    (tvarant::linear_pointwise) and the GEMM has enough 128 x 256 tiles
    (4/5 of a wave) to run without split-K."""
    tiles = -(-m // 128) * -(-N_DEFAULT // 256)
    return bool(fusions.get("gemm_pointwise")) and m > 128 and tiles >= (sms * 4) // 5


def measure_gemm_point(torch, m: int, mode: str, steps: int, warmup: int, world: int,
                       clocks=None) -> dict:
    """One point of the fused-GEMM sweep: the compiled linear+bias+SiLU +
    chain step (resident inputs), the GEMM launch alone back to back, and the
    end-to-end step with host buffers.  Times are max over ranks.

    When the compiler put the chain into the GEMM's epilogue, a step is that
    one kernel: its time is the kernel's duration (back-to-back launches on
    one stream), and the plain GEMM (linear_act alone) is timed beside it."""
    wl = GemmChain(torch, m, mode)
    Event = lambda: torch.Event(device="tvarant", enable_timing=True)  # noqa: E731
    for _ in range(warmup):
        wl.step_resident(torch)
    torch.tvarant.synchronize()
    _barrier(world)
    torch.tvarant.synchronize()
    h0 = time.perf_counter()
    e_start, e_end = Event(), Event()
    e_start.record()
    for _ in range(steps):
        wl.step_resident(torch)
    e_end.record()
    e_end.synchronize()
    if clocks is not None:
        clocks.mark(h0, time.perf_counter())
    step_ms = e_start.elapsed_time(e_end) / steps
    # The GEMM kernel alone: the same launch back to back on the same stream
    # between two events (the GPU never waits for the host).
    lins = [mdl.lin for mdl in wl.models]
    g0, g1 = Event(), Event()
    g0.record()
    for i in range(steps):
        li = lins[i % len(lins)]
        torch.ops.tvarant.linear_act(wl.x, li.weight, li.bias, "silu", True)
    g1.record()
    g1.synchronize()
    plain_gemm_ms = g0.elapsed_time(g1) / steps
    torch.tvarant.synchronize()
    _barrier(world)
    step_ms = _max_over_ranks(step_ms, world)
    plain_gemm_ms = _max_over_ranks(plain_gemm_ms, world)
    from tvarant_b200 import _C

    fused = program_in_epilogue(m, wl.fusions, _C.sm_count(torch.tvarant.current_device()))
    kernel_ms = step_ms if fused else plain_gemm_ms
    wl.e2e_begin(torch)
    for _ in range(max(1, warmup // 2)):
        wl.step_e2e(torch)
    wl.e2e_end(torch)
    torch.tvarant.synchronize()
    _barrier(world)
    t0, t1 = Event(), Event()
    t0.record()
    wl.e2e_begin(torch)
    for _ in range(steps):
        wl.step_e2e(torch)
    wl.e2e_end(torch)
    t1.record()
    t1.synchronize()
    e2e_ms = _max_over_ranks(t0.elapsed_time(t1) / steps, world)
    kernel, bound = gemm_kernel_name(m, mode, fused)
    # algorithmic bytes of the timed kernel: W, X, bias and the output, plus Z
    # when the chain runs in its epilogue
    gemm_bytes = 4.0 * (N_DEFAULT * K_DEFAULT + m * K_DEFAULT + m * N_DEFAULT + N_DEFAULT
                        + (m * N_DEFAULT if fused else 0))
    return {"wl": wl, "M": m, "mode": mode, "step_ms": step_ms, "kernel_ms": kernel_ms,
            "plain_gemm_ms": plain_gemm_ms, "program_in_epilogue": fused,
            "launches_per_step": 1 if fused else 2,
            "e2e_ms": e2e_ms, "kernel": kernel, "bound": bound, "flops": wl.flops,
            "gemm_bytes": gemm_bytes,
            "step_tflops": wl.flops / (step_ms / 1e3) / 1e12,
            "kernel_tflops": wl.flops / (kernel_ms / 1e3) / 1e12,
            "kernel_gbs": gemm_bytes / (kernel_ms / 1e3) / 1e9}


def _traffic_key(pt: dict) -> str:
    """Key of the timed kernel's ncu DRAM traffic in profiles/ncu_traffic.json."""
    prefix = "gemm_pw" if pt.get("program_in_epilogue") else "gemm"
    return f"{prefix}_{pt['mode']}_m{pt['M']}"


def _roofline(pt: dict, tf32_peak, peaks: dict) -> dict:
    if pt["bound"] == "hbm":
        hbm = peaks.get("hbm_gbs", 6650.0)
        return {"bound": "hbm", "achieved": pt["kernel_gbs"], "peak": hbm, "unit": "GB/s",
                "frac": pt["kernel_gbs"] / hbm,
                "traffic": _traffic(_traffic_key(pt)),
                "kernel": pt["kernel"], "kernel_ms": pt["kernel_ms"],
                "algorithmic_bytes": pt["gemm_bytes"],
                "peak_source": "MEASURED_PEAKS.json hbm_gbs"}
    peak = tf32_peak if tf32_peak else peaks.get("bf16_tflops", 1590.0) / 2
    if pt["mode"] == "3xtf32":
        peak = peak / 3  # three TF32 MMAs per k-step
    return {"bound": "tensor", "achieved": pt["kernel_tflops"], "peak": peak, "unit": "TFLOP/s",
            "frac": pt["kernel_tflops"] / peak,
            "traffic": _traffic(_traffic_key(pt)),
            "kernel": pt["kernel"], "kernel_ms": pt["kernel_ms"],
            "peak_source": ("cuBLAS TF32 8192^3 measured in this run" if tf32_peak
                            else "half of the bf16 peak (no cuBLAS)")
            + (" / 3 (3xTF32 issues three TF32 MMAs)" if pt["mode"] == "3xtf32" else ""),
            "frac_of_bf16_measured": pt["kernel_tflops"] / peaks.get("bf16_tflops", 1617.5)}


def run_gemm(args, rank, world, local_rank) -> dict | None:
    torch = _device_setup(local_rank)
    with ClockSampler(local_rank) as clocks:
        pt = measure_gemm_point(torch, args.m, args.mode, args.steps, args.warmup, world, clocks)
    wl = pt["wl"]
    status = torch.tvarant.get_status()
    if rank != 0:
        return None
    peaks = _peaks()
    tf32_peak = tf32_peak_tflops(torch)
    line = {
        "metric": METRIC,
        "value": world * wl.flops / (pt["step_ms"] / 1e3) / 1e12,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": pt["step_ms"],
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "tf32" if args.mode == "tf32" else "f32 (3xTF32)",
        "data": "synthetic (seeded N(0,1) activations, U(-1/64,1/64) weights)",
        "config": {
            "workload": f"linear+bias+SiLU GEMM M={args.m} K={K_DEFAULT} N={N_DEFAULT} ({args.mode}) "
                        "+ abs(neg(exp(Y - Z))) chain, compiled by torch_tvarant.compiler "
                        + ("(chain in the GEMM epilogue: one kernel per step)"
                           if pt["program_in_epilogue"] else "(chain as a second kernel)"),
            "plain_gemm_ms": pt["plain_gemm_ms"],
            "M": args.m, "K": K_DEFAULT, "N": N_DEFAULT, "mode": args.mode,
            "parallelism": f"replicas x{world}",
            "l2": ("inputs (X 268 MB + Z 268 MB + W 67 MB) exceed the 126 MB L2" if wl.copies == 1
                   else f"steps rotate over {wl.copies} weight copies ({wl.copies * 67} MB > L2), "
                        "so each step reads its weight from HBM"),
            "fusions": wl.fusions,
        },
        "e2e": {"value": world * wl.flops / (pt["e2e_ms"] / 1e3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": wl.h2d_bytes, "d2h_bytes_per_step": wl.d2h_bytes,
                "ms_per_step": pt["e2e_ms"],
                "pipeline": "pinned host X, Z in on a copy stream, compiled model on the "
                            "compute stream, Y out on another copy stream; double-buffered "
                            "device inputs, so consecutive steps overlap"},
        "roofline": _roofline(pt, tf32_peak, peaks),
        "gpu_launches": args.steps * pt["launches_per_step"],
        "clocks": clocks.summary(),
        "device_status": status,
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_gemm()
    return line


def fixed_tf32_peak(peaks: dict) -> float:
    """Half the measured dense bf16 burst peak: the TF32 tensor rate of the
    same tensor cores, a figure that does not move with the cuBLAS TF32 run of
    the day."""
    return peaks.get("bf16_tflops", 1590.0) / 2


def single_gpu_extras(torch, args, tf32_peak) -> dict:
    """The fused-GEMM sweep's largest point in both precision modes, the LLM
    op set, the memory-bound kernels, and the GPT-2-small forward with the
    fused attention kernel alone at its shapes, for the one-GPU default line."""
    from tvarant_b200 import workloads

    peaks = _peaks()
    steps = max(5, min(args.steps, 10))
    out = {}
    for mode in ("tf32", "3xtf32"):
        pt = measure_gemm_point(torch, M_DEFAULT, mode, steps, 3, 1)
        pt.pop("wl")
        torch.tvarant.empty_cache()
        rl = _roofline(pt, tf32_peak, peaks)
        fixed = fixed_tf32_peak(peaks) / (3 if mode == "3xtf32" else 1)
        out[f"gemm_m{M_DEFAULT}_{mode}"] = {
            "workload": f"linear+bias+SiLU M={M_DEFAULT} K={K_DEFAULT} N={N_DEFAULT} + "
                        "abs(neg(exp(Y - Z))) compiled into one launch",
            "step_ms": pt["step_ms"], "step_tflops": pt["step_tflops"],
            "plain_gemm_ms": pt["plain_gemm_ms"],
            "e2e_tflops": pt["flops"] / (pt["e2e_ms"] / 1e3) / 1e12,
            "kernel": pt["kernel"], "frac": rl["frac"], "peak": rl["peak"],
            "peak_source": rl["peak_source"],
            "frac_fixed": pt["kernel_tflops"] / fixed,
            "peak_fixed": fixed,
            "peak_fixed_source": "MEASURED_PEAKS.json bf16_tflops / 2 (of measured)"
                                 + (" / 3" if mode == "3xtf32" else "")}
    res = workloads.measure_llm_ops(steps, 3)
    torch.tvarant.empty_cache()
    out["llm_ops"] = {"per_op": res["per_op"], "GB/s": res["GB/s"], "frac_hbm": res["frac_hbm"],
                      "peak_gbs": res["peak_gbs"], "inputs": res["inputs"]}
    res = workloads.measure_mem_kernels(steps, 3)
    torch.tvarant.empty_cache()
    out["memory_bound_kernels"] = {k: {"GB/s": v["GB/s"], "frac_hbm": v["frac_hbm"], "ms": v["ms"]}
                                   for k, v in res["per_kernel"].items()}
    # GPT-2-small forward (fused attention, one CUDA graph per step), the gpt2
    # workload's own code path; its line carries the attention kernel alone
    import argparse

    g_args = argparse.Namespace(**vars(args))
    g_args.workload, g_args.attention, g_args.mode = "gpt2", "sdpa", "tf32"
    g_args.seq, g_args.gpt2_batch, g_args.steps, g_args.warmup = 1024, 8, steps, 3
    g_args.no_graph = False
    g_line = workloads._gpt2(g_args, 0, 1, torch.tvarant.current_device())
    torch.tvarant.empty_cache()
    out["gpt2_forward"] = {
        "workload": g_line["config"]["workload"], "tokens_per_s": g_line["value"],
        "ms_per_step": g_line["ms_per_step"], "e2e_tokens_per_s": g_line["e2e"]["value"],
        "eager_tokens_per_s": g_line["config"]["eager_tokens_per_s"],
        "tflop_per_step": g_line["config"]["tflop_per_step"],
        "last_logits_finite": g_line["config"]["last_logits_finite"]}
    out["attention"] = g_line["config"]["attention_kernel"]
    # GPT-2-small decode with a KV cache (batch 8, 512-token prompt, the step
    # replayed as one CUDA graph), the gpt2-decode workload's own code path
    d_args = argparse.Namespace(**vars(g_args))
    d_args.workload, d_args.prompt, d_args.steps, d_args.warmup = "gpt2-decode", 512, 20, 3
    d_line = workloads._gpt2_decode(d_args, 0, 1, torch.tvarant.current_device())
    torch.tvarant.empty_cache()
    out["gpt2_decode"] = {
        "workload": d_line["config"]["workload"], "tokens_per_s": d_line["value"],
        "ms_per_step": d_line["ms_per_step"],
        "eager_tokens_per_s": d_line["config"]["eager_tokens_per_s"],
        "hbm_frac_of_step_bytes": d_line["roofline"]["frac"]}
    torch.set_float32_matmul_precision("high" if args.mode == "tf32" else "highest")
    return out


SWEEP_M = (1, 16, 128, 1024, 4096, 16384)


def run_sweep(args, rank, world, local_rank) -> dict | None:
    """The whole fused-GEMM sweep: M in {1, 16, 128, 1024, 4096, 16384},
    K = N = 4096, TF32 and 3xTF32, each point the compiled GEMM + chain."""
    torch = _device_setup(local_rank)
    points = []
    with ClockSampler(local_rank) as clocks:
        for mode in ("tf32", "3xtf32"):
            for m in SWEEP_M:
                pt = measure_gemm_point(torch, m, mode, args.steps, args.warmup, world, clocks)
                pt.pop("wl")
                points.append(pt)
                torch.tvarant.empty_cache()
    status = torch.tvarant.get_status()
    if rank != 0:
        return None
    peaks = _peaks()
    tf32_peak = tf32_peak_tflops(torch)
    table = []
    for pt in points:
        rl = _roofline(pt, tf32_peak, peaks)
        table.append({"M": pt["M"], "mode": pt["mode"], "step_ms": pt["step_ms"],
                      "step_tflops": pt["step_tflops"], "kernel_ms": pt["kernel_ms"],
                      "plain_gemm_ms": pt["plain_gemm_ms"],
                      "kernel": pt["kernel"], "bound": rl["bound"], "achieved": rl["achieved"],
                      "unit": rl["unit"], "frac": rl["frac"],
                      "e2e_tflops": pt["flops"] / (pt["e2e_ms"] / 1e3) / 1e12})
    head = next(p for p in points if p["M"] == SWEEP_M[-1] and p["mode"] == "tf32")
    return {
        "metric": METRIC,
        "value": world * head["step_tflops"], "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["step_ms"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "tf32 and f32 (3xTF32)",
        "data": "synthetic (seeded N(0,1) activations, U(-1/64,1/64) weights)",
        "config": {"workload": "fused-GEMM sweep: linear+bias+SiLU M in {1,16,128,1024,4096,16384} "
                               "K=N=4096 + abs(neg(exp(Y - Z))) compiled into the GEMM epilogue "
                               "(M > 128) or a program pass (M <= 128), TF32 and 3xTF32; "
                               "value = the M=16384 TF32 point",
                   "points": table, "parallelism": f"replicas x{world}",
                   "l2": "points whose operands fit in L2 rotate over weight copies in distinct "
                         "buffers (> 256 MB in total), so each step reads its weight from HBM"},
        "roofline": _roofline(head, tf32_peak, peaks),
        "gpu_launches": sum(args.steps * p["launches_per_step"] for p in points),
        "clocks": clocks.summary(),
        "device_status": status,
    }


def run_reference(args, rank, world) -> dict | None:
    """The reference's CPU implementation of the selected workload, rank 0 only."""
    if rank != 0:
        return None
    if args.workload == "mlp":
        return run_reference_mlp(args, world)
    if args.workload in ("gemm", "sweep"):
        return run_reference_gemm(args, world)
    return {"impl": "reference",
            "unavailable": f"no CPU reference arm for --workload {args.workload}; the default "
                           "(mlp) and gemm workloads have one"}


def run_reference_mlp(args, world) -> dict:
    """The MLP stack on the reference's simulator kernels: each step one layer
    on a token sample (all host threads), reported as tokens/s of the whole
    stack."""
    threads = _cpu_cores()
    rows = args.ref_rows or 4 * threads
    for _ in range(args.warmup):
        reference_mlp_rows(rows, threads)
    times = [reference_mlp_rows(rows, threads) for _ in range(args.steps)]
    dt = sum(times) / len(times)
    value = rows / (dt * args.layers)
    # the simulator itself has no parallel loops: the same layer on one thread
    dt1 = reference_mlp_rows(4, 1)
    return {
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": dt * 1e3,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (N(0,0.02) weights, N(0,1) activations)",
        "config": {"workload": f"Llama-7B-shaped gated-SiLU MLP stack, {args.layers} layers, "
                               f"d_model {D_MODEL}, d_ff {D_FF}, {MLP_TOKENS} tokens (the "
                               "reference's eager linear_act / linear / mul / linear)",
                   "parallelism": "host threads",
                   "step": f"one layer on {rows} tokens (the timed sample); value = tokens / "
                           f"({args.layers} x step time)",
                   "single_thread_tokens_per_s": 4 / (dt1 * args.layers)},
        "impl": "reference",
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "reference",
                         "sample": f"one layer on {rows} of {MLP_TOKENS} tokens per step, "
                                   f"reference HostKernels.cpp (oracle/_ref), {threads} threads; "
                                   f"stack time = {args.layers} x layer time"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def run_reference_gemm(args, world) -> dict:
    threads = _cpu_cores()
    rows = args.ref_rows or min(args.m, 64 * threads)
    for _ in range(args.warmup):
        reference_gemm_chain_rows(rows, threads)
    times = []
    fl = 0.0
    for _ in range(args.steps):
        dt, fl = reference_gemm_chain_rows(rows, threads)
        times.append(dt)
    dt = sum(times) / len(times)
    value = fl / dt / 1e12
    return {
        "metric": METRIC,
        "value": value,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": dt * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,1) activations, U(-1/64,1/64) weights)",
        "config": {
            "workload": f"linear+bias+SiLU GEMM M={args.m} K={K_DEFAULT} N={N_DEFAULT} "
                        "+ abs(neg(exp(Y - Z))) chain (eager, as the reference runs it)",
            "M": args.m, "K": K_DEFAULT, "N": N_DEFAULT, "parallelism": "host threads",
        },
        "impl": "reference",
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "reference",
                         "sample": f"{rows} rows of {args.m} per step; reference HostKernels.cpp "
                                   f"(oracle/_ref), {threads} threads"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main() -> int:
    import torch

    with torch.no_grad():
        return _main()


def _main() -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["tvarant", "reference"], default="tvarant")
    ap.add_argument("--workload", choices=["mlp", "gemm", "sweep", "llm-ops", "mem-kernels",
                                           "llama-ops", "bmm", "gpt2", "gpt2-decode"],
                    default="mlp",
                    help="mlp (default, at every N): the tensor-parallel Llama MLP stack")
    ap.add_argument("--batch", type=int, default=256, help="bmm workload: batch size")
    ap.add_argument("--m", type=int, default=M_DEFAULT)
    ap.add_argument("--mode", choices=["tf32", "3xtf32"], default="tf32")
    ap.add_argument("--ref-rows", type=int, default=0)
    ap.add_argument("--layers", type=int, default=32, help="mlp workload: MLP layers")
    ap.add_argument("--seq", type=int, default=1024, help="gpt2 workload: sequence length")
    ap.add_argument("--prompt", type=int, default=512,
                    help="gpt2-decode workload: prompt tokens per sequence before decoding")
    ap.add_argument("--gpt2-batch", type=int, default=8, help="gpt2 workload: sequences per step (whole job)")
    ap.add_argument("--attention", choices=["bmm", "sdpa"], default="bmm",
                    help="gpt2 workload: bmm + mask + softmax + bmm (the config), or the fused "
                         "F.scaled_dot_product_attention kernel")
    ap.add_argument("--chunks", type=int, default=2, help="mlp workload: token chunks overlapped with the all-reduce")
    ap.add_argument("--comm", choices=["auto", "nccl", "nvls", "nvls-fused"], default="auto",
                    help="mlp workload at N>1: NCCL all-reduce, this library's NVLink SHARP "
                         "all-reduce over symmetric memory, or (TF32) the down projection and "
                         "that all-reduce in one kernel")
    ap.add_argument("--gemm-sms", type=int, default=0,
                    help="mlp workload at N>1: SMs the GEMMs may use while the all-reduce runs "
                         "(0: all but the collective's CTAs)")
    ap.add_argument("--nvls-blocks", type=int, default=16,
                    help="mlp workload, --comm nvls: CTAs of the all-reduce kernel")
    ap.add_argument("--nccl-ctas", type=int, default=32,
                    help="mlp workload: CTAs NCCL may use per collective (the GEMMs leave that many SMs free; 0: no limit)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="mlp workload on one GPU: skip the GEMM and LLM-op points in config")
    ap.add_argument("--no-graph", action="store_true",
                    help="mlp / gpt2 workloads: time the eager calls instead of a CUDA graph replay")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank, world, local_rank = _env_rank()
    if args.impl == "reference":
        line = run_reference(args, rank, world)
    else:
        _dist_init(world)
        if args.workload == "gemm":
            line = run_gemm(args, rank, world, local_rank)
        elif args.workload == "sweep":
            line = run_sweep(args, rank, world, local_rank)
        else:
            from tvarant_b200 import workloads

            line = workloads.run(args, rank, world, local_rank)
    if line is not None:
        print(json.dumps(line), flush=True)
    if world > 1 and args.impl != "reference":
        import torch.distributed as dist

        if dist.is_initialized():
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
