"""Benchmark workloads beyond the default fused-GEMM sweep (used by bench.py).

* ``llm-ops`` — the memory-bound LLM op set: softmax(dim=-1) on
  [8, 32, 2048, 2048], layer_norm over [16384, 4096], embedding of int64 ids
  [16, 2048] from a [32000, 4096] table, and bmm [256, 2048, 128] x
  [256, 128, 2048].  Value: algorithmic GB/s of one pass over all four.
* ``mlp`` — the Llama-7B-shaped gated-SiLU MLP stack (32 layers, d_model
  4096, d_ff 11008, 8192 tokens, TF32), tensor-parallel over the ranks with
  one NCCL all-reduce per layer.  Value: tokens/s of the whole job.
* ``gpt2`` — the GPT-2-small-shaped decoder forward (``tvarant_b200.gpt2``:
  12 layers, d_model 768, 12 heads, SiLU MLP via the fused linear, vocab
  50257, batch 8 x seq 1024), the batch split over the ranks (so every
  attention bmm / softmax is split over batch x heads).  Value: tokens/s of
  the whole job.

Inputs are seeded synthetic tensors with the shapes and distributions of
those workloads.  All work runs through the torch_tvarant device API.
"""

from __future__ import annotations

import statistics
import time

import torch

D_MODEL, D_FF, LAYERS, TOKENS = 4096, 11008, 32, 8192



def _events():
    return (torch.Event(device="tvarant", enable_timing=True),
            torch.Event(device="tvarant", enable_timing=True))


def _time_steps(fn, steps: int) -> float:
    e0, e1 = _events()
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / steps


def run(args, rank: int, world: int, local_rank: int):
    import torch_tvarant  # noqa: F401

    torch.tvarant.set_device(local_rank)
    if args.workload == "llm-ops":
        return _llm_ops(args, rank, world, local_rank)
    if args.workload == "bmm":
        return _bmm(args, rank, world, local_rank)
    if args.workload == "gpt2":
        return _gpt2(args, rank, world, local_rank)
    if args.workload == "llama-ops":
        return _llama_ops(args, rank, world, local_rank)
    if args.workload == "gpt2-decode":
        return _gpt2_decode(args, rank, world, local_rank)
    if args.workload == "mem-kernels":
        return _mem_kernels(args, rank, world, local_rank)
    return _mlp(args, rank, world, local_rank)


# ----------------------------------------------------------------------------- llama ops

def _llama_ops(args, rank, world, local_rank):
    """The row ops a Llama-style decoder adds to the LLM op set, at Llama-7B
    shapes over 8192 tokens: RMSNorm of the [8192, 4096] hidden states, and
    RoPE of the query heads [1, 32, 8192, 128] (Hugging Face layout, [T, 128]
    angle tables).  Both are HBM-bound: GB/s against the measured copy rate."""
    import bench

    g = torch.Generator().manual_seed(1)
    dev = "tvarant"
    x = torch.randn(8192, 4096, generator=g).to(dev)
    w = (1 + 0.1 * torch.randn(4096, generator=g)).to(dev)
    q = torch.randn(1, 32, 8192, 128, generator=g).to(dev)
    inv = 1.0 / (10000 ** (torch.arange(0, 128, 2, dtype=torch.float32) / 128))
    ang = torch.arange(8192, dtype=torch.float32)[:, None] * inv[None, :]
    cos = torch.cat([ang.cos(), ang.cos()], -1).to(dev)
    sin = torch.cat([ang.sin(), ang.sin()], -1).to(dev)
    F = torch.nn.functional
    ops = {
        "rms_norm": (lambda: F.rms_norm(x, (4096,), w, 1e-6), 2 * x.numel() * 4 + 4096 * 4),
        # q in and out; the half-width tables are read once per position
        "rope": (lambda: torch.ops.tvarant.rope(q, cos, sin), 2 * q.numel() * 4 + 2 * 8192 * 64 * 4),
    }
    for fn, _ in ops.values():
        for _ in range(args.warmup):
            fn()
    torch.tvarant.synchronize()
    # Each op is timed back to back on its own: at ~50 us per launch, a step
    # that alternates the two ops from Python would time the host.
    per = {}
    with bench.ClockSampler(local_rank) as clocks:
        h0 = time.perf_counter()
        for name, (fn, nbytes) in ops.items():
            ms = bench._max_over_ranks(_time_steps(fn, args.steps), world)
            per[name] = {"ms": ms, "GB/s": nbytes / (ms / 1e3) / 1e9}
        clocks.mark(h0, time.perf_counter())
    total_ms = sum(v["ms"] for v in per.values())
    total_bytes = sum(nb for _, nb in ops.values())
    if rank != 0:
        return None
    hbm = bench._peaks().get("hbm_gbs", 6650.0)
    for v in per.values():
        v["frac_hbm"] = v["GB/s"] / hbm
    value = total_bytes / (total_ms / 1e3) / 1e9
    return {
        "metric": bench.METRIC,
        "value": value * world, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total_ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) activations, Llama-7B shapes)",
        "config": {"workload": "rms_norm [8192,4096] + rope q [1,32,8192,128] (rotate-half, "
                               "[T,128] tables)",
                   "per_op": per, "parallelism": f"replicas x{world}",
                   "l2": "each operand (134 MB) exceeds the 126 MB L2"},
        "roofline": {"bound": "hbm", "achieved": value, "peak": hbm, "unit": "GB/s",
                     "frac": value / hbm, "traffic": None,
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs"},
        "gpu_launches": 2 * args.steps,
        "clocks": clocks.summary(),
        "device_status": torch.tvarant.get_status(),
    }


# ----------------------------------------------------------------------------- bmm

def _bmm(args, rank, world, local_rank):
    """bmm [batch, 2048, 128] x [batch, 128, 2048] alone (the LLM op set's bmm)."""
    import bench

    batch = args.batch
    g = torch.Generator().manual_seed(1)
    a = torch.randn(batch, 2048, 128, generator=g).to("tvarant")
    b = torch.randn(batch, 128, 2048, generator=g).to("tvarant")
    torch.set_float32_matmul_precision("high" if args.mode == "tf32" else "highest")
    for _ in range(args.warmup):
        torch.bmm(a, b)
    torch.tvarant.synchronize()
    with bench.ClockSampler(local_rank) as clocks:
        h0 = time.perf_counter()
        ms = _time_steps(lambda: torch.bmm(a, b), args.steps)
        clocks.mark(h0, time.perf_counter())
    ms = bench._max_over_ranks(ms, world)
    if rank != 0:
        return None
    nbytes = 4 * batch * (2048 * 128 * 2 + 2048 * 2048)
    hbm = bench._peaks().get("hbm_gbs", 6650.0)
    gbs = nbytes / (ms / 1e3) / 1e9
    return {
        "metric": bench.METRIC,
        "value": gbs * world, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "tf32" if args.mode == "tf32" else "f32 (3xTF32)",
        "data": "synthetic N(0,1)",
        "config": {"workload": f"bmm [{batch},2048,128] x [{batch},128,2048]",
                   "tflops": 2 * batch * 2048 * 2048 * 128 / (ms / 1e3) / 1e12,
                   "parallelism": f"replicas x{world}"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                     "frac": gbs / hbm, "traffic": None, "peak_source": "MEASURED_PEAKS.json hbm_gbs"},
        "clocks": clocks.summary(),
        "device_status": torch.tvarant.get_status(),
    }


# ----------------------------------------------------------------------------- llm-ops

def device_randn(shape, seed: int, std: float = 1.0, mean: float = 0.0) -> torch.Tensor:
    """A tvarant tensor ~N(mean, std^2) drawn on the GPU by torch's CUDA
    generator (seeded) and copied device to device: multi-GB benchmark inputs
    without a host draw and a PCIe copy."""
    import ctypes

    from . import capi

    g = torch.Generator(device="cuda").manual_seed(seed)
    src = torch.randn(*shape, device="cuda", generator=g)
    if std != 1.0:
        src.mul_(std)
    if mean != 0.0:
        src.add_(mean)
    torch.cuda.synchronize()
    out = torch.empty(*shape, device="tvarant")
    stream = torch.tvarant.stream_handle(torch.tvarant.current_stream())
    capi.call("tvr_memcpy_d2d", ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(src.data_ptr()),
              src.numel() * 4, ctypes.c_void_p(stream))
    torch.tvarant.synchronize()
    del src
    torch.cuda.empty_cache()
    return out


def measure_llm_ops(steps: int, warmup: int, mode: str = "tf32") -> dict:
    """The LLM op set, each op timed back to back on its own stream with
    events: softmax(dim=-1) on [8, 32, 2048, 2048] ~N(0, 2), layer_norm over
    [16384, 4096] (gamma ~N(1, 0.1), beta ~N(0, 0.1)), embedding of int64 ids
    [16, 2048] from a [32000, 4096] table ~N(0, 0.02), bmm [256, 2048, 128] x
    [256, 128, 2048].  Returns per-op ms, algorithmic GB/s and fraction of the
    measured copy rate, and the time of one pass over all four (the sum of
    the ops' times)."""
    import bench

    g = torch.Generator().manual_seed(1)
    dev = "tvarant"
    sm_x = device_randn((8, 32, 2048, 2048), seed=1, std=2 ** 0.5)
    ln_x = device_randn((16384, 4096), seed=2)
    ln_w = (1 + 0.1 * torch.randn(4096, generator=g)).to(dev)
    ln_b = (0.1 * torch.randn(4096, generator=g)).to(dev)
    table = device_randn((32000, 4096), seed=3, std=0.02)
    ids = torch.randint(0, 32000, (16, 2048), generator=g).to(dev)
    a = device_randn((256, 2048, 128), seed=4)
    b = device_randn((256, 128, 2048), seed=5)
    torch.set_float32_matmul_precision("high" if mode == "tf32" else "highest")
    F = torch.nn.functional
    ops = {
        "softmax": (lambda: F.softmax(sm_x, dim=-1), 2 * sm_x.numel() * 4),
        "layer_norm": (lambda: F.layer_norm(ln_x, (4096,), ln_w, ln_b, 1e-5),
                       2 * ln_x.numel() * 4 + 2 * 4096 * 4 + 2 * 16384 * 4),
        "embedding": (lambda: F.embedding(ids, table), 2 * 32768 * 4096 * 4 + 32768 * 8),
        "bmm": (lambda: torch.bmm(a, b), 4 * 256 * (2048 * 128 * 2 + 2048 * 2048)),
    }
    for fn, _ in ops.values():
        for _ in range(warmup):
            fn()
    torch.tvarant.synchronize()
    hbm = bench._peaks().get("hbm_gbs", 6650.0)
    per = {}
    for name, (fn, nbytes) in ops.items():
        ms = _time_steps(fn, steps)
        per[name] = {"ms": ms, "GB/s": nbytes / (ms / 1e3) / 1e9,
                     "frac_hbm": nbytes / (ms / 1e3) / 1e9 / hbm}
    per["bmm"]["tflops"] = 2 * 256 * 2048 * 2048 * 128 / (per["bmm"]["ms"] / 1e3) / 1e12
    # one pass over the set: each op's own back-to-back time, summed
    total_ms = sum(v["ms"] for v in per.values())
    total_bytes = sum(nb for _, nb in ops.values())
    return {"per_op": per, "total_ms": total_ms, "total_bytes": total_bytes,
            "GB/s": total_bytes / (total_ms / 1e3) / 1e9,
            "frac_hbm": total_bytes / (total_ms / 1e3) / 1e9 / hbm,
            "peak_gbs": hbm, "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)",
            "inputs": "seeded N(mean, std) drawn on the GPU (torch CUDA generator), ids on the host"}


def measure_attention(steps: int, warmup: int, batch: int = 8) -> dict:
    """The fused causal attention kernel at GPT-2's shapes (q, k, v
    [batch, 12, 1024, 64] ~N(0, 1), scale 1/8, TF32) called through the C ABI
    with preallocated buffers, timed back to back with events.  FLOPs are
    the unmasked work, 4 * B * H * 64 * (1024 * 1025 / 2) (QK^T and PV over
    the keys each query sees); the TF32 fraction is against half the measured
    bf16 peak (a fixed denominator)."""
    import ctypes

    import bench

    from . import capi

    h, s, d = 12, 1024, 64
    q = device_randn((batch, h, s, d), seed=21)
    k = device_randn((batch, h, s, d), seed=22)
    v = device_randn((batch, h, s, d), seed=23)
    out = torch.empty(batch, h, s, d, device="tvarant")
    st = capi.int64_array([h * s * d, s * d, d])
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    def launch():
        stream = ctypes.c_void_p(torch.tvarant.stream_handle(torch.tvarant.current_stream()))
        capi.call("tvr_attention_fwd", p(q), p(k), p(v), p(out), None, batch, h, s, s, d,
                  st, st, st, st, 0.125, 1, capi.GEMM_TF32, stream)

    for _ in range(warmup):
        launch()
    torch.tvarant.synchronize()
    ms = min(_time_steps(launch, steps) for _ in range(3))
    flop = 4.0 * batch * h * d * (s * (s + 1) / 2)
    peak = bench.fixed_tf32_peak(bench._peaks())
    tflops = flop / (ms / 1e3) / 1e12
    return {"workload": f"causal attention q, k, v [{batch}, {h}, {s}, {d}], TF32",
            "kernel": "tvr::attn::attn_fwd_kernel", "us": ms * 1e3, "tflops": tflops,
            "frac": tflops / peak, "peak": peak,
            "peak_source": "MEASURED_PEAKS.json bf16_tflops / 2 (of measured)",
            "flop": flop, "flop_note": "unmasked work: QK^T and PV over the keys each query sees"}


# abs(neg(exp(y - z))) as a pointwise SSA program (the fused-GEMM sweep's chain):
# Load y, Load z, Sub, Exp, Neg, Abs
_CHAIN_PROGRAM = ([0, 0, 9, 10, 6, 11], [-1, -1, 0, 2, 3, 4], [-1, -1, 1, -1, -1, -1],
                  [0, 1, -1, -1, -1, -1], [1.0] * 6, [0.0] * 6)


def measure_mem_kernels(steps: int, warmup: int) -> dict:
    """Every memory-bound kernel family on operands of 150-540 MB (above the
    126 MB L2), each timed back to back with events: softmax rows of 2048 (the
    LLM op set's row length), softmax with an additive [1024, 1024] mask,
    layer norm, embedding gather, unary exp, broadcast add, the NVRTC
    pointwise chain sub/exp/neg/abs, RMSNorm, RoPE (rotate-half) and the
    strided copy of a GPT-2 head split.  Returns per-kernel ms, algorithmic
    bytes, GB/s and fraction of the measured copy rate."""
    import bench

    g = torch.Generator().manual_seed(3)
    dev = "tvarant"
    F = torch.nn.functional
    big = (16384, 4096)
    x = device_randn(big, seed=11)
    z = device_randn(big, seed=12)
    sm = device_randn((32768, 2048), seed=13, std=2 ** 0.5)
    scores = device_randn((64, 1024, 1024), seed=14)
    mask = torch.full((1024, 1024), float("-inf")).triu(1).to(dev)
    gamma = (1 + 0.1 * torch.randn(4096, generator=g)).to(dev)
    beta = (0.1 * torch.randn(4096, generator=g)).to(dev)
    table = device_randn((32000, 4096), seed=15, std=0.02)
    ids = torch.randint(0, 32000, (16, 1024), generator=g).to(dev)
    q = device_randn((1, 32, 16384, 128), seed=16)
    inv = 1.0 / (10000 ** (torch.arange(0, 128, 2, dtype=torch.float32) / 128))
    ang = torch.arange(16384, dtype=torch.float32)[:, None] * inv[None, :]
    cos = torch.cat([ang.cos(), ang.cos()], -1).to(dev)
    sin = torch.cat([ang.sin(), ang.sin()], -1).to(dev)
    qkv = device_randn((16, 1024, 3, 12, 64), seed=17)
    n = x.numel() * 4
    cases = {
        "softmax_warp_kernel [32768, 2048]": (lambda: F.softmax(sm, dim=-1), 2 * sm.numel() * 4),
        "softmax_shared_mask_kernel [64, 1024, 1024] + [1024, 1024] mask": (
            lambda: torch.ops.tvarant.softmax_add(scores, mask), 2 * scores.numel() * 4),
        "layer_norm_kernel [16384, 4096]": (
            lambda: F.layer_norm(x, (4096,), gamma, beta, 1e-5), 2 * n + 2 * 4096 * 4 + 2 * 16384 * 4),
        "embedding_kernel [16, 1024] ids from [32000, 4096]": (
            lambda: F.embedding(ids, table), 2 * ids.numel() * 4096 * 4 + ids.numel() * 8),
        "unary exp [16384, 4096]": (lambda: torch.exp(x), 2 * n),
        "binary add [16384, 4096] + [4096]": (lambda: x + beta, 2 * n + 4096 * 4),
        "tvr_pointwise_kernel abs(neg(exp(x - z))) [16384, 4096]": (
            lambda: torch.ops.tvarant.pointwise([x, z], *_CHAIN_PROGRAM), 3 * n),
        "rms_norm_kernel [16384, 4096]": (lambda: F.rms_norm(x, (4096,), gamma, 1e-6), 2 * n + 4096 * 4),
        "rope_half_vec_kernel q [1, 32, 16384, 128]": (
            lambda: torch.ops.tvarant.rope(q, cos, sin), 2 * q.numel() * 4 + 2 * 16384 * 64 * 4),
        "copy_transpose_kernel qkv [16, 1024, 3, 12, 64] -> [3, 16, 12, 1024, 64]": (
            lambda: qkv.permute(2, 0, 3, 1, 4).contiguous(), 2 * qkv.numel() * 4),
    }
    for fn, _ in cases.values():
        for _ in range(warmup):
            fn()
    torch.tvarant.synchronize()
    hbm = bench._peaks().get("hbm_gbs", 6650.0)
    per = {}
    for name, (fn, nbytes) in cases.items():
        ms = _time_steps(fn, steps)
        per[name] = {"ms": ms, "bytes": nbytes, "GB/s": nbytes / (ms / 1e3) / 1e9,
                     "frac_hbm": nbytes / (ms / 1e3) / 1e9 / hbm}
    return {"per_kernel": per, "peak_gbs": hbm,
            "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)"}


def _mem_kernels(args, rank, world, local_rank):
    import bench

    with bench.ClockSampler(local_rank) as clocks:
        h0 = time.perf_counter()
        res = measure_mem_kernels(args.steps, args.warmup)
        clocks.mark(h0, time.perf_counter())
    per = res["per_kernel"]
    total_ms = bench._max_over_ranks(sum(v["ms"] for v in per.values()), world)
    if rank != 0:
        return None
    total_bytes = sum(v["bytes"] for v in per.values())
    value = total_bytes / (total_ms / 1e3) / 1e9
    hbm = res["peak_gbs"]
    worst = min(per, key=lambda k: per[k]["frac_hbm"])
    return {
        "metric": bench.METRIC,
        "value": value * world, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total_ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1)-family inputs drawn on the GPU)",
        "config": {"workload": "every memory-bound kernel family once per step, operands "
                               "150-540 MB", "per_kernel": per,
                   "parallelism": f"replicas x{world}",
                   "l2": "every operand exceeds the 126 MB L2"},
        "roofline": {"bound": "hbm", "achieved": value, "peak": hbm, "unit": "GB/s",
                     "frac": value / hbm, "traffic": None, "peak_source": res["peak_source"],
                     "lowest": {"kernel": worst, "frac_hbm": per[worst]["frac_hbm"]}},
        "gpu_launches": args.steps * len(per),
        "clocks": clocks.summary(),
        "device_status": torch.tvarant.get_status(),
    }


def _llm_ops(args, rank, world, local_rank):
    import bench

    with bench.ClockSampler(local_rank) as clocks:
        h0 = time.perf_counter()
        res = measure_llm_ops(args.steps, args.warmup, args.mode)
        clocks.mark(h0, time.perf_counter())
    total_ms = bench._max_over_ranks(res["total_ms"], world)
    if rank != 0:
        return None
    hbm = res["peak_gbs"]
    value = res["total_bytes"] / (total_ms / 1e3) / 1e9
    return {
        "metric": bench.METRIC,
        "value": value * world, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total_ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, shapes and distributions of the LLM op set)",
        "config": {"workload": "softmax [8,32,2048,2048] + layer_norm [16384,4096] + embedding "
                               "[16,2048] from [32000,4096] + bmm [256,2048,128]x[256,128,2048]",
                   "per_op": res["per_op"], "parallelism": f"replicas x{world}",
                   "l2": "every operand exceeds the 126 MB L2 except the LN row vectors"},
        "roofline": {"bound": "hbm", "achieved": value, "peak": hbm, "unit": "GB/s",
                     "frac": value / hbm, "traffic": None,
                     "peak_source": res["peak_source"]},
        "clocks": clocks.summary(),
        "device_status": torch.tvarant.get_status(),
    }


# ----------------------------------------------------------------------------- mlp

def build_stack(rank: int, world: int, device: str, layers: int = LAYERS, seed: int = 0):
    """This rank's shards of the MLP stack: one seeded draw of the rank's
    gate/up/down shards, scaled per layer on the device so that every layer
    has its own weights in HBM without drawing 17 GB on the host."""
    s = D_FF // world
    g = torch.Generator().manual_seed(seed * 1000 + rank)
    base_g = (0.02 * torch.randn(s, D_MODEL, generator=g)).to(device)
    base_u = (0.02 * torch.randn(s, D_MODEL, generator=g)).to(device)
    base_d = (0.02 * torch.randn(D_MODEL, s, generator=g)).to(device)
    out = []
    for layer in range(layers):
        f = 1.0 + 1e-3 * layer
        out.append((base_g * f, base_u * f, base_d * f))
    return out


class _StackIO:
    """End-to-end steps of the tensor-parallel stack with host buffers.

    Rank r owns tokens [r * T/N, (r + 1) * T/N) of the job's input and output
    (T tokens, N ranks).  Per step: its input slice is copied in from pinned
    host memory on one copy stream, one step ahead of the compute (two device
    slice buffers); on the compute stream the slices of all ranks are gathered
    (NCCL all-gather) into the stack's input — on one GPU the slice is the
    whole input and is copied device to device — the stack runs, and the
    rank's slice of the output is copied aside and sent back to pinned host
    memory on another copy stream (two buffers)."""

    def __init__(self, x, x_host, out_host, run, rank, world, comm, device):
        from tvarant_b200 import _C

        self._C = _C
        self.x, self.run, self.world, self.comm = x, run, world, comm
        self.rows = x.shape[0] // world
        self.r0 = rank * self.rows
        dev = f"tvarant:{device}"
        self.s_in = torch.Stream(device=dev)
        self.s_out = torch.Stream(device=dev)
        self.dev = dev
        self.slices = [torch.empty(self.rows, x.shape[1], device=dev) for _ in range(2)]
        self.outs = [torch.empty(self.rows, x.shape[1], device=dev) for _ in range(2)]
        self.host_in = x_host[self.r0:self.r0 + self.rows]
        spare = torch.empty(self.rows, x.shape[1])
        if torch.cuda.is_available():
            spare = spare.pin_memory()
        self.host_out = [out_host[self.r0:self.r0 + self.rows], spare]
        self.consumed = [None, None]
        self.drained = [None, None]
        self.j = 0

    def _event(self, stream):
        ev = torch.Event(device=self.dev)
        ev.record(stream)
        return ev

    def begin(self):
        """Orders both copy streams after the work queued so far."""
        start = self._event(torch.tvarant.current_stream())
        self.s_in.wait_event(start)
        self.s_out.wait_event(start)

    def end(self):
        """Orders the compute stream after both copy streams."""
        compute = torch.tvarant.current_stream()
        compute.wait_event(self._event(self.s_in))
        compute.wait_event(self._event(self.s_out))

    def step(self):
        k = self.j & 1
        self.j += 1
        compute = torch.tvarant.current_stream()
        if self.consumed[k] is not None:
            self.s_in.wait_event(self.consumed[k])  # slice k gathered two steps ago
        with torch.tvarant.stream(self.s_in):
            self.slices[k].copy_(self.host_in, non_blocking=True)
            landed = self._event(self.s_in)
        compute.wait_event(landed)
        if self.world > 1:
            self._C.all_gather(self.slices[k], self.x, self.comm.handle)
        else:
            self.x.copy_(self.slices[k])
        self.consumed[k] = self._event(compute)
        y = self.run(self.x)
        if self.drained[k] is not None:
            compute.wait_event(self.drained[k])  # out buffer k sent two steps ago
        self.outs[k].copy_(y[self.r0:self.r0 + self.rows])
        self.s_out.wait_event(self._event(compute))
        with torch.tvarant.stream(self.s_out):
            self.host_out[k].copy_(self.outs[k], non_blocking=True)
            self.drained[k] = self._event(self.s_out)


def _mlp(args, rank, world, local_rank):
    import bench
    from tvarant_b200.tp import Communicator, TPMLPStack

    torch.set_float32_matmul_precision("high" if args.mode == "tf32" else "highest")
    dev = f"tvarant:{local_rank}"
    layers = build_stack(rank, world, dev, layers=args.layers)
    comm, nvls = None, None
    kind = args.comm
    if world > 1 and kind == "auto":
        # this library's NVLS all-reduce where the switch supports it (every
        # rank must agree), else NCCL's
        from tvarant_b200.nvls import agreed_multicast

        kind = "nvls" if agreed_multicast(local_rank) else "nccl"
    use_nvls = world > 1 and kind in ("nvls", "nvls-fused")
    fused = use_nvls and kind == "nvls-fused" and args.mode == "tf32"
    if use_nvls:
        from tvarant_b200.nvls import NvlsAllReduce

        chunks = max(1, args.chunks)
        rows = -(-TOKENS // chunks)
        nvls = [NvlsAllReduce(rows * D_MODEL, local_rank, blocks=args.nvls_blocks)
                for _ in range(chunks)]
    elif world > 1:
        comm = Communicator.from_process_group(local_rank, args.nccl_ctas)
    stack = TPMLPStack(layers, comm, chunks=args.chunks if world > 1 else 1, nvls=nvls,
                       gemm_sms=args.gemm_sms if world > 1 else 0, fused=fused)
    g = torch.Generator().manual_seed(7)
    x_host = torch.randn(TOKENS, D_MODEL, generator=g)
    if torch.cuda.is_available():
        x_host = x_host.pin_memory()
    x = x_host.to(dev)
    out_host = torch.empty(TOKENS, D_MODEL)
    if torch.cuda.is_available():
        out_host = out_host.pin_memory()
    for _ in range(args.warmup):
        stack(x)
    torch.tvarant.synchronize()
    bench._barrier(world)
    eager_ms = bench._max_over_ranks(_time_steps(lambda: stack(x), args.steps), world)
    # the whole stack (GEMMs, events, all-reduces on the side stream) as one
    # CUDA graph: one launch per step instead of ~6 host-side calls per layer
    run = stack
    if not args.no_graph:
        from tvarant_b200.graphs import Graph

        graph = Graph(stack, x)
        run = lambda _x: graph.replay()  # noqa: E731
        torch.tvarant.synchronize()
        bench._barrier(world)
    with bench.ClockSampler(local_rank) as clocks:
        h0 = time.perf_counter()
        ms = _time_steps(lambda: run(x), args.steps)
        clocks.mark(h0, time.perf_counter())
    ms = bench._max_over_ranks(ms, world)
    # the per-layer GEMMs alone (one rank's share of the FLOPs)
    wg, wu, wd = layers[0]
    from tvarant_b200 import _C
    from tvarant_b200.tp import mlp_layer

    layer_ms = _time_steps(lambda: mlp_layer(x, wg, wu, wd), args.steps)
    # the dominant kernel, the SwiGLU GEMM, at the stack's chunk shape and
    # under the stack's SM limit, timed back to back on its stream
    rows = -(-TOKENS // stack.chunks)
    xc = x[:rows]
    prev_limit = _C.gemm_sm_limit(local_rank)
    sm_limit = stack.sm_limit(local_rank)
    _C.set_gemm_sm_limit(local_rank, sm_limit)
    try:
        for _ in range(3):
            torch.ops.tvarant.linear_swiglu(xc, wg, wu)
        swiglu_ms = _time_steps(lambda: torch.ops.tvarant.linear_swiglu(xc, wg, wu), args.steps)
    finally:
        _C.set_gemm_sm_limit(local_rank, prev_limit)
    swiglu_flops = 2.0 * rows * (2 * wg.shape[0]) * D_MODEL

    # End to end: each rank brings its slice of the tokens in from pinned host
    # memory and sends its slice of the output back; the slices are gathered
    # over NVLink into the stack's input.  An NCCL communicator serves that
    # gather when the stack's own exchange is NVLS.
    gather = comm
    if world > 1 and gather is None:
        gather = Communicator.from_process_group(local_rank, args.nccl_ctas)
    io = _StackIO(x, x_host, out_host, run, rank, world, gather, local_rank)
    for _ in range(2):
        io.begin()
        io.step()
        io.end()
    torch.tvarant.synchronize()
    bench._barrier(world)
    e0, e1 = _events()
    e0.record()
    io.begin()
    for _ in range(args.steps):
        io.step()
    io.end()
    e1.record()
    e1.synchronize()
    e2e_ms = bench._max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    status = torch.tvarant.get_status()
    if not args.no_graph:
        graph.close()
    if gather is not None and gather is not comm:
        bench._barrier(world)
        gather.destroy()
    if comm is not None:
        bench._barrier(world)
        comm.destroy()
    if nvls is not None:
        bench._barrier(world)
        for buf in nvls:
            buf.close()
        bench._barrier(world)
    swiglu_ms = bench._max_over_ranks(swiglu_ms, world)
    if rank != 0:
        return None
    flops_total = 3 * 2 * TOKENS * D_MODEL * D_FF * args.layers
    per_rank_flops = flops_total / world
    peak = bench.tf32_peak_tflops(torch) or 750.0
    peaks = bench._peaks()
    fixed = bench.fixed_tf32_peak(peaks)
    achieved = per_rank_flops / (ms / 1e3) / 1e12
    nvlink_bytes = (2 * (world - 1) / world) * TOKENS * D_MODEL * 4 * args.layers if world > 1 else 0
    target_s = max(per_rank_flops / (peak * 1e12), nvlink_bytes / 770e9)
    swiglu_tflops = swiglu_flops / (swiglu_ms / 1e3) / 1e12
    tf32 = args.mode == "tf32"
    kpeak = peak if tf32 else peak / 3
    line = {
        "metric": bench.METRIC,
        "value": TOKENS / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "tf32" if args.mode == "tf32" else "f32 (3xTF32)",
        "data": "synthetic (N(0,0.02) weights, N(0,1) activations)",
        "config": {"workload": f"Llama-7B-shaped gated-SiLU MLP stack, {args.layers} layers, "
                               f"d_model {D_MODEL}, d_ff {D_FF}, {TOKENS} tokens, TP x{world}",
                   "parallelism": f"tp{world}", "chunks": stack.chunks,
                   "exchange": (("down projection and NVLS all-reduce in one kernel "
                                 f"({args.nvls_blocks} reducing CTAs)") if fused
                                else ("NVLS all-reduce (multimem, this library's kernel, "
                                      f"{args.nvls_blocks} CTAs)") if use_nvls
                                else ("NCCL all-reduce" if world > 1 else None)),
                   "nccl_max_ctas": args.nccl_ctas if comm is not None else None,
                   "gemm_sms": args.gemm_sms if world > 1 else None,
                   "cuda_graph": not args.no_graph,
                   "eager_tokens_per_s": TOKENS / (eager_ms / 1e3),
                   "layer_ms_one_rank_gemms": layer_ms,
                   "l2": "weights per rank exceed L2 at tp<=4; activations 134 MB"},
        "e2e": {"value": TOKENS / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": TOKENS * D_MODEL * 4,
                "d2h_bytes_per_step": TOKENS * D_MODEL * 4, "ms_per_step": e2e_ms,
                "per_rank_bytes_each_way": io.rows * D_MODEL * 4,
                "pipeline": "each rank copies its 1/N of the tokens in from pinned host memory "
                            "on a copy stream (one step ahead), the slices are gathered into "
                            "the stack's input" + (" by an NCCL all-gather" if world > 1 else "")
                            + ", and its 1/N of the output goes back on another copy stream"},
        "roofline": {"bound": "tensor",
                     "achieved": swiglu_tflops, "peak": kpeak, "unit": "TFLOP/s",
                     "frac": swiglu_tflops / kpeak,
                     "traffic": (bench._traffic("gemm_swiglu_m8192_n11008")
                                 if world == 1 and rows == TOKENS and tf32 else None),
                     "kernel": ("tvr::tc::gemm_tc_kernel<256, tf32, K-major B, GATED> (SwiGLU: "
                                f"[{rows}, {D_MODEL}] x [2 x {wg.shape[0]}, {D_MODEL}])"
                                if tf32 else "3xTF32 SwiGLU composition"),
                     "kernel_ms": swiglu_ms,
                     "algorithmic_flops": swiglu_flops,
                     "peak_source": "cuBLAS TF32 8192^3 measured in this run"
                                    + ("" if tf32 else " / 3"),
                     "frac_fixed": swiglu_tflops / (fixed if tf32 else fixed / 3),
                     "peak_fixed": fixed if tf32 else fixed / 3,
                     "peak_fixed_source": "MEASURED_PEAKS.json bf16_tflops / 2 (of measured)",
                     "gemm_sm_limit": sm_limit,
                     "step": {"achieved_tflops_per_gpu": achieved,
                              "frac": (target_s * 1e3) / ms,
                              "target": "max(FLOPs per GPU / measured TF32 peak, all-reduce "
                                        "bytes per GPU / 770 GB/s NVLink)"}},
        # per layer and chunk: the SwiGLU GEMM and the down GEMM, plus the
        # epoch step and the all-reduce kernel with NVLS (NCCL's are not ours)
        "gpu_launches": args.steps * args.layers * stack.chunks * (3 if fused else 4 if use_nvls else 2),
        "clocks": clocks.summary(),
        "device_status": status,
    }
    if world == 1:
        if not args.no_extras:
            line["config"]["one_gpu_points"] = bench.single_gpu_extras(torch, args, peak)
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = bench.cpu_baseline_mlp()
    return line


# ----------------------------------------------------------------------------- gpt2

def _gpt2_cpu_baseline(host_model, cfg, seq: int) -> dict:
    """The reference's compiled kernels (oracle/_ref) running the same forward
    on one sequence of ``seq`` tokens, one host thread."""
    import numpy as np

    import oracle
    from oracle import gpt2 as ogpt2

    impl = "ref" if oracle.available("ref") else "port"
    n = lambda t: t.numpy()  # noqa: E731
    params = {"wte": n(host_model.wte), "wpe": n(host_model.wpe), "lnf_g": n(host_model.lnf_g),
              "lnf_b": n(host_model.lnf_b),
              "layers": [{f: n(getattr(L, f)) for f in L.__dataclass_fields__} for L in host_model.layers]}
    ids = np.random.default_rng(3).integers(0, cfg.vocab, (1, seq), dtype=np.int64)
    t0 = time.perf_counter()
    ogpt2.forward(params, ids, cfg.n_head, impl=impl)
    dt = time.perf_counter() - t0
    return {"value": seq / dt, "unit": "tokens/s", "cores": 1,
            "kind": "reference" if impl == "ref" else "port",
            "sample": f"1 sequence x {seq} tokens through all {cfg.n_layer} layers and the LM head "
                      f"({dt:.1f} s; attention per token is {seq}/1024 of the benchmark's)"}


def _gpt2_decode(args, rank, world, local_rank):
    """GPT-2-small generation with a KV cache: a prompt of ``--prompt`` tokens
    per sequence (prefill), then one token per sequence per step (decode).
    A step is one ``forward_step`` over [batch, 1] new tokens: few-row GEMMs
    (batch rows), attention of one query per head over the cached keys, and
    the LM head; the decode tokens are the model's greedy choices, so nothing
    of a step is precomputed.  ``value`` = batch / step time, for the step
    captured as a CUDA graph (TF32: ``gpt2.decode_step``, position and key
    count on the device) unless ``--no-graph``; the eager step (the cache
    views grow by one position a step) is timed beside it."""
    import bench
    from tvarant_b200 import gpt2

    torch.set_float32_matmul_precision("high" if args.mode == "tf32" else "highest")
    dev = f"tvarant:{local_rank}"
    cfg = gpt2.GPT2Config()
    batch, prompt = args.gpt2_batch, args.prompt
    steps = args.steps
    if prompt + args.warmup + 2 * steps + 3 > cfg.n_ctx:
        raise ValueError(f"prompt {prompt} + {args.warmup + 2 * steps + 3} steps exceed "
                         f"{cfg.n_ctx} positions")
    model = gpt2.init_gpt2(cfg, seed=0).to(dev)
    g = torch.Generator().manual_seed(12)
    ids = torch.randint(0, cfg.vocab, (batch, prompt), generator=g).to(dev)
    cache = gpt2.new_cache(model, batch, cfg.n_ctx, dev)
    t0, t1 = _events()
    t0.record()
    logits = gpt2.forward_step(model, ids, cache)
    t1.record()
    t1.synchronize()
    prefill_ms = t0.elapsed_time(t1)
    nxt = logits[:, -1:].argmax(-1)
    first = nxt.clone()
    for _ in range(args.warmup):
        nxt = gpt2.forward_step(model, nxt, cache)[:, -1:].argmax(-1)
    torch.tvarant.synchronize()
    bench._barrier(world)

    def step():
        nonlocal nxt
        nxt = gpt2.forward_step(model, nxt, cache)[:, -1:].argmax(-1)

    eager_ms = bench._max_over_ranks(_time_steps(step, steps), world)
    run, graph = step, None
    if not args.no_graph and args.mode == "tf32":
        # the fixed-shape step (cache position and key count on the device)
        # captured once; each replay decodes one token per sequence
        from tvarant_b200.graphs import Graph

        ids = first.clone()
        pos = torch.full((1,), prompt, dtype=torch.int64).to(dev)
        graph = Graph(gpt2.decode_step, model, ids, cache, pos, warmup=1)
        pos.copy_(torch.full((1,), prompt, dtype=torch.int64))
        ids.copy_(first)
        run = graph.replay
        torch.tvarant.synchronize()
        bench._barrier(world)
    with bench.ClockSampler(local_rank) as clocks:
        h0 = time.perf_counter()
        ms = _time_steps(run, steps)
        clocks.mark(h0, time.perf_counter())
    ms = bench._max_over_ranks(ms, world)
    if graph is not None:
        graph.close()
    status = torch.tvarant.get_status()
    if rank != 0:
        return None
    weight_bytes = 4 * (cfg.n_layer * (4 * cfg.d_model ** 2 + 2 * cfg.d_model * cfg.d_ff)
                        + cfg.vocab * cfg.d_model)
    # the timed steps attend over prompt + 1 .. prompt + steps cached
    # positions (the graph's position restarts at the prompt; the eager
    # steps' were further on): keys and values of every layer, head and
    # sequence, read once per step
    mean_keys = prompt + (steps + 1) / 2
    kv_bytes = 2 * 4 * cfg.n_layer * batch * cfg.d_model * mean_keys
    step_bytes = weight_bytes + kv_bytes
    peak_gbs = bench._peaks().get("hbm_gbs", 6650.0)
    return {
        "metric": bench.METRIC,
        "value": world * batch / (ms / 1e3), "unit": "tokens/s (decode)", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "tf32" if args.mode == "tf32" else "f32 (3xTF32)",
        "data": "synthetic (N(0,0.02) weights, uniform prompt ids, greedy decode tokens)",
        "config": {"workload": f"GPT-2-small decode with a KV cache: batch {batch}, prompt {prompt}, "
                               f"{steps} timed single-token steps "
                               + ("(CUDA graph of the fixed-shape step)" if graph is not None
                                  else "(eager)"),
                   "eager_ms_per_step": eager_ms,
                   "eager_tokens_per_s": world * batch / (eager_ms / 1e3),
                   "prefill_ms": prefill_ms, "parallelism": f"replicas x{world}",
                   "weights_mb": weight_bytes / 1e6,
                   "kv_cache_read_mb_per_step": kv_bytes / 1e6,
                   "l2": "the 0.5 GB of weights exceed L2; every step streams them"},
        "roofline": {"bound": "hbm", "achieved": step_bytes / (ms / 1e3) / 1e9,
                     "peak": peak_gbs, "unit": "GB/s",
                     "frac": step_bytes / (ms / 1e3) / 1e9 / peak_gbs,
                     "traffic": None,
                     "note": "algorithmic bytes per step (every weight once, plus the cached keys "
                             "and values each layer attends over) over the step time; the step is "
                             "bound by ~150 small kernels, not by HBM"},
        "gpu_launches": None,
        "clocks": clocks.summary(),
        "device_status": status,
    }


def _gpt2(args, rank, world, local_rank):
    import bench
    from tvarant_b200 import gpt2

    torch.set_float32_matmul_precision("high" if args.mode == "tf32" else "highest")
    dev = f"tvarant:{local_rank}"
    cfg = gpt2.GPT2Config()
    seq, batch = args.seq, args.gpt2_batch
    host_model = gpt2.init_gpt2(cfg, seed=0)
    model = host_model.to(dev)
    b0, b1 = gpt2.shard_batch(batch, rank, world)
    g = torch.Generator().manual_seed(11)
    ids_all = torch.randint(0, cfg.vocab, (batch, seq), generator=g)
    ids_host = ids_all[b0:b1].contiguous()
    last_host = torch.empty(b1 - b0, cfg.vocab)
    if torch.cuda.is_available():
        ids_host = ids_host.pin_memory()
        last_host = last_host.pin_memory()
    ids = ids_host.to(dev)
    mask = gpt2.causal_mask(seq, dev)
    att = args.attention
    for _ in range(args.warmup):
        gpt2.forward(model, ids, mask, att)
    torch.tvarant.synchronize()
    bench._barrier(world)
    eager_ms = bench._max_over_ranks(
        _time_steps(lambda: gpt2.forward(model, ids, mask, att), args.steps), world)
    run = lambda: gpt2.forward(model, ids, mask, att)  # noqa: E731
    graph = None
    if not args.no_graph:
        from tvarant_b200.graphs import Graph

        graph = Graph(gpt2.forward, model, ids, mask, att)
        run = graph.replay
        torch.tvarant.synchronize()
        bench._barrier(world)
    with bench.ClockSampler(local_rank) as clocks:
        h0 = time.perf_counter()
        ms = _time_steps(run, args.steps)
        clocks.mark(h0, time.perf_counter())
    ms = bench._max_over_ranks(ms, world)

    def e2e_step():
        ids.copy_(ids_host, non_blocking=True)
        logits = run()
        last_host.copy_(logits[:, -1, :], non_blocking=True)

    e2e_step()
    torch.tvarant.synchronize()
    bench._barrier(world)
    e2e_ms = bench._max_over_ranks(_time_steps(e2e_step, args.steps), world)
    status = torch.tvarant.get_status()
    # parity on the device-resident result: the last position of every local
    # sequence is a proper distribution after softmax (finite logits)
    logits = run()
    finite = bool(torch.isfinite(logits[:, -1, :].cpu()).all())
    if graph is not None:
        del logits
        graph.close()
    attention_point = (measure_attention(max(5, min(args.steps, 20)), 3, batch=b1 - b0)
                       if att == "sdpa" and seq == 1024 else None)
    if rank != 0:
        return None
    tokens = batch * seq
    flops_rank = cfg.flops_per_token(seq) * tokens / world
    peak = bench.tf32_peak_tflops(torch) or 750.0
    achieved = flops_rank / (ms / 1e3) / 1e12
    line = {
        "metric": bench.METRIC,
        "value": tokens / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "tf32" if args.mode == "tf32" else "f32 (3xTF32)",
        "data": "synthetic (N(0,0.02) weights, uniform token ids)",
        "config": {"workload": f"GPT-2-small-shaped forward, {cfg.n_layer} layers, d_model {cfg.d_model}, "
                               f"{cfg.n_head} heads, d_ff {cfg.d_ff} SiLU, vocab {cfg.vocab}, "
                               f"batch {batch} x seq {seq}, causal attention as "
                               + ("bmm + mask add + softmax + bmm" if att == "bmm"
                                  else "fused scaled_dot_product_attention (TF32 kernel)")
                               + ", tied LM head",
                   "attention": att,
                   "cuda_graph": not args.no_graph,
                   "eager_tokens_per_s": batch * seq / (eager_ms / 1e3),
                   "parallelism": f"batch split over {world} rank(s) (attention split over batch x heads)",
                   "tflop_per_step": cfg.flops_per_token(seq) * tokens / 1e12,
                   "last_logits_finite": finite,
                   "attention_kernel": attention_point,
                   "l2": "attention scores 403 MB per layer, weights 497 MB, logits 1.6 GB"},
        "e2e": {"value": tokens / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": batch * seq * 8, "d2h_bytes_per_step": batch * cfg.vocab * 4,
                "ms_per_step": e2e_ms},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s per GPU",
                     "frac": achieved / peak, "traffic": None,
                     "peak_source": "cuBLAS TF32 8192^3 measured in this run"},
        "gpu_launches": args.steps * (cfg.n_layer * (17 if att == "bmm" else 10) + 4),
        "clocks": clocks.summary(),
        "device_status": status,
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = _gpt2_cpu_baseline(host_model, cfg, 128)
    return line
