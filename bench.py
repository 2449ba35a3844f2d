#!/usr/bin/env python
"""Benchmark of the B200 W4G64 QuantLinear forward (decode GEMV headline).

Workload (the seven-shape sweep at M=1, i.e. one decode token through every
quantised linear of Qwen2-1.5B): the seven linear shapes q 1536->1536,
k/v 1536->256, o 1536->1536, gate/up 1536->8960, down 8960->1536, for each
of the 28 layers, symmetric W4G64 RTN of bf16 weights ~N(0, 0.02), bf16
activations ~N(0, 1), q/k/v with bf16 bias. A step is one pass over all 196
linears; the 655 MB of packed weights per step are far larger than L2, so no
flush is needed. Synthetic, seeded data (no checkpoint is used).

  value  = algorithmic bytes per step (N*K/2 + 2*N*K/64 + 2*M*K + 2*M*N per linear, + 2*N with bias) / device time,
           step captured once in a CUDA graph of C-ABI launches, replayed K times
  e2e    = same metric through the public Python API (b200_w4g64_linear) with
           the step's activations copied host->device and outputs device->host
           inside the timed region
  gemm   = the seven shapes at M=2048 (TFLOP/s), tensor-core kernel
  roofline, cpu_baseline, clocks: see the JSON keys.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
Multi-GPU (torchrun): independent replicas, one per rank, weak scaling.
"""

from __future__ import annotations

import argparse
import ctypes
import importlib
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
PACKAGE = "qwen2-int4-systems_b200"

METRIC = "W4G64 GEMV HBM GB/s (M=1), GEMM TFLOP/s (M=2048); Qwen2-1.5B decode tok/s"
UNIT = "GB/s"
LAYERS = 28
# (name, in_features K, out_features N, has_bias) - model.py:56-59,129-131
SHAPES = [("q", 1536, 1536, True), ("k", 1536, 256, True), ("v", 1536, 256, True),
          ("o", 1536, 1536, False), ("gate", 1536, 8960, False), ("up", 1536, 8960, False),
          ("down", 8960, 1536, False)]
WORKLOAD = "qwen2-1.5b-7-linears-x28-layers-w4g64-rtn-m1"


def alg_bytes(m: int, n: int, k: int, bias: bool, asym: bool = False) -> int:
    """Algorithmic bytes of one linear: packed weights + fp16 scales + x + out (+zeros, +bias)."""
    b = n * k // 2 + n * (k // 64) * 2 + m * k * 2 + m * n * 2
    if asym:
        b += (n * (k // 64) + 1) // 2
    if bias:
        b += 2 * n
    return b


# ---------------------------------------------------------------------------
# clocks during the timed region (NVML, sampled from a thread)
# ---------------------------------------------------------------------------

class ClockSampler:
    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
        "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
        "display_clock_setting": 0x100,
    }

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.samples: list[tuple[int, int]] = []
        self.period = period_s
        self.handle = None
        self.max_mhz = None
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            props = torch.cuda.get_device_properties(device_index)
            uuid = str(getattr(props, "uuid", ""))
            try:
                self.handle = pynvml.nvmlDeviceGetHandleByUUID(
                    uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
                idx = int(visible.split(",")[device_index]) if visible else device_index
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.handle = None
        self._thread = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                sm = self.nvml.nvmlDeviceGetClockInfo(self.handle, self.nvml.NVML_CLOCK_SM)
                reasons = self.nvml.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                self.samples.append((sm, reasons))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.handle is not None:
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self.handle is not None:
            self._thread.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        mhz = [s for s, _ in self.samples]
        mask = 0
        for _, r in self.samples:
            mask |= r
        reasons = [name for name, bit in self.REASONS.items() if mask & bit and name != "gpu_idle"]
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(mhz)}


# ---------------------------------------------------------------------------
# synthetic weights (symmetric RTN of quantization.py:87-111, on the GPU)
# ---------------------------------------------------------------------------

def quantize_symmetric_rtn_gpu(n: int, k: int, gen: torch.Generator, device) -> tuple:
    q2 = importlib.import_module(PACKAGE + ".qwen2")
    w = (torch.randn(n, k, device=device, generator=gen) * 0.02).to(torch.bfloat16).float()
    packed, scales = q2.quantize_symmetric_rtn_torch(w)
    zeros = torch.zeros((n * (k // 64) + 1) // 2, 1, dtype=torch.uint8, device=device)
    return packed, scales, zeros


def build_model_weights(device, seed: int = 0) -> list[list[dict]]:
    gen = torch.Generator(device=device).manual_seed(seed)
    layers = []
    for _ in range(LAYERS):
        layer = []
        for name, k, n, has_bias in SHAPES:
            qw, sc, z = quantize_symmetric_rtn_gpu(n, k, gen, device)
            bias = (torch.randn(n, device=device, generator=gen) * 0.02).to(torch.bfloat16) if has_bias else None
            layer.append({"name": name, "k": k, "n": n, "qweight": qw, "scales": sc, "zeros": z, "bias": bias})
        layers.append(layer)
    return layers


# ---------------------------------------------------------------------------
# device-side measurement through the C ABI
# ---------------------------------------------------------------------------

class Chain:
    """A list of C-ABI launches with preallocated activations and outputs."""

    def __init__(self, lib, entries: list[dict], m: int, device, gen: torch.Generator, algo: int = 0):
        self.lib, self.entries, self.m, self.algo = lib, entries, m, algo
        self.x = [torch.randn(m, e["k"], device=device, generator=gen).to(torch.bfloat16) for e in entries]
        self.out = [torch.empty(m, e["n"], device=device, dtype=torch.bfloat16) for e in entries]

    def launch(self):
        stream = torch.cuda.current_stream().cuda_stream
        for e, x, o in zip(self.entries, self.x, self.out):
            b = e["bias"]
            rc = self.lib.qi4_w4g64_linear_ex(
                x.data_ptr(), 1, self.m, e["k"], e["qweight"].data_ptr(), e["scales"].data_ptr(),
                e["zeros"].data_ptr(), None if b is None else b.data_ptr(), -1 if b is None else 1,
                o.data_ptr(), e["n"], stream, self.algo, 1)
            if rc:
                raise RuntimeError(f"launch failed: {rc}")

    def graph(self) -> torch.cuda.CUDAGraph:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            self.launch()
            self.launch()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.launch()
        return g

    def bytes(self) -> int:
        return sum(alg_bytes(self.m, e["n"], e["k"], e["bias"] is not None) for e in self.entries)

    def flops(self) -> int:
        return sum(2 * self.m * e["n"] * e["k"] for e in self.entries)


class GroupedChain:
    """The decode step with the linears that share an input grouped into one
    C-ABI launch (qi4_w4g64_linear_multi): per layer q/k/v, o, gate/up, down
    (4 launches instead of 7). Same weights, same bytes, same outputs."""

    GROUPS = (("q", "k", "v"), ("o",), ("gate", "up"), ("down",))

    def __init__(self, lib, layers: list[list[dict]], device, gen: torch.Generator):
        self.lib = lib
        self.launches = []
        for layer in layers:
            by_name = {e["name"]: e for e in layer}
            for group in self.GROUPS:
                ents = [by_name[n] for n in group]
                k = ents[0]["k"]
                x = torch.randn(1, k, device=device, generator=gen).to(torch.bfloat16)
                outs = [torch.empty(1, e["n"], device=device, dtype=torch.bfloat16) for e in ents]
                c = len(ents)
                arr = lambda vals: (ctypes.c_void_p * c)(*vals)
                bias = [e["bias"] for e in ents]
                self.launches.append((x, outs, c, k, arr([e["qweight"].data_ptr() for e in ents]),
                                      arr([e["scales"].data_ptr() for e in ents]),
                                      arr([e["zeros"].data_ptr() for e in ents]),
                                      arr([None if b is None else b.data_ptr() for b in bias]),
                                      1 if any(b is not None for b in bias) else -1,
                                      arr([o.data_ptr() for o in outs]),
                                      (ctypes.c_int64 * c)(*[e["n"] for e in ents])))

    def launch(self):
        stream = torch.cuda.current_stream().cuda_stream
        for x, outs, c, k, qw, sc, z, b, bd, o, ns in self.launches:
            rc = self.lib.qi4_w4g64_linear_multi(x.data_ptr(), 1, 1, k, c, qw, sc, z, b, bd, o, ns, stream)
            if rc:
                raise RuntimeError(f"grouped launch failed: {rc}")

    graph = Chain.graph


def time_graph(g: torch.cuda.CUDAGraph, reps: int, warmup: int) -> float:
    """Average ms per replay (CUDA events on the replay stream)."""
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(reps):
        g.replay()
    end.record()
    end.synchronize()
    return start.elapsed_time(end) / reps


# ---------------------------------------------------------------------------
# CPU baseline: the reference's torch backend restated (oracle/torch_port.py)
# ---------------------------------------------------------------------------

def cpu_linear_sample(reps: int = 3, sample: str = "layer") -> dict:
    from oracle import torch_port

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    gen = torch.Generator().manual_seed(1)
    shapes = SHAPES if sample == "layer" else [s for s in SHAPES if s[0] == "gate"]
    data = []
    for name, k, n, has_bias in shapes:
        w = (torch.randn(n, k, generator=gen) * 0.02).to(torch.bfloat16).float().view(n, k // 64, 64)
        s = w.abs().amax(-1) / 7.0
        s = torch.where(s == 0, torch.ones_like(s), s)
        codes = torch.round(w / s.unsqueeze(-1)).clamp_(-7, 7).to(torch.int16).view(n, k)
        qw = ((codes[:, 0::2] & 0xF) | ((codes[:, 1::2] & 0xF) << 4)).to(torch.uint8).reshape(-1, 1)
        z = torch.zeros((n * (k // 64) + 1) // 2, 1, dtype=torch.uint8)
        bias = (torch.randn(n, generator=gen) * 0.02).to(torch.bfloat16) if has_bias else None
        x = torch.randn(1, k, generator=gen).to(torch.bfloat16)
        data.append((x, qw, s.to(torch.float16), z, bias, n, k))

    def run():
        for x, qw, sc, z, bias, n, k in data:
            torch_port.linear(x, qw, sc, z, bias, out_features=n, in_features=k)

    run()
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    nbytes = sum(alg_bytes(1, n, k, bias is not None) for _, _, _, _, bias, n, k in data)
    t = statistics.median(times)
    return {"value": nbytes / t / 1e9, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{len(data)} linear(s) of one layer at M=1 ({sample}), median of {reps}, "
                      f"oracle/torch_port.py (reference torch backend restated) on {threads} threads",
            "seconds_per_sample": t}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import torch_port  # noqa: F401  (fails loudly if the oracle is missing)

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    gen = torch.Generator().manual_seed(1)
    per_step = []
    for name, k, n, has_bias in SHAPES:
        w = (torch.randn(n, k, generator=gen) * 0.02).to(torch.bfloat16).float().view(n, k // 64, 64)
        s = w.abs().amax(-1) / 7.0
        s = torch.where(s == 0, torch.ones_like(s), s)
        codes = torch.round(w / s.unsqueeze(-1)).clamp_(-7, 7).to(torch.int16).view(n, k)
        qw = ((codes[:, 0::2] & 0xF) | ((codes[:, 1::2] & 0xF) << 4)).to(torch.uint8).reshape(-1, 1)
        z = torch.zeros((n * (k // 64) + 1) // 2, 1, dtype=torch.uint8)
        bias = (torch.randn(n, generator=gen) * 0.02).to(torch.bfloat16) if has_bias else None
        per_step.append((torch.randn(1, k, generator=gen).to(torch.bfloat16), qw, s.to(torch.float16), z,
                         bias, n, k))
    from oracle import torch_port as tp

    def step():
        for x, qw, sc, z, bias, n, k in per_step:
            tp.linear(x, qw, sc, z, bias, out_features=n, in_features=k)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    elapsed = time.perf_counter() - t0
    nbytes = sum(alg_bytes(1, n, k, bias is not None) for _, _, _, _, bias, n, k in per_step)
    value = nbytes * args.steps / elapsed / 1e9
    sample = (f"one layer's 7 linears at M=1 per step (1/28 of the GPU step), "
              f"oracle/torch_port.py on {threads} host threads")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed * 1e3 / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": {"workload": WORKLOAD, "m": 1, "sample": "1 of 28 layers"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


# ---------------------------------------------------------------------------
# main (our arm)
# ---------------------------------------------------------------------------

def e2e_decode(device, prompt_len: int = 512, new_tokens: int = 128) -> dict:
    """Batch-1 decode: the reference's Qwen2-1.5B (random init, W4G64 RTN) on
    the b200 backend, batch 1, greedy decode through the reference's own
    ``greedy_generate_cached``; the same model on the reference's ``torch``
    backend on this GPU for comparison (fewer steps). The ``b200_fused_mlp``
    leg also routes the MLP through the fused gate/up SwiGLU call
    (``register_with_reference(fuse_mlp=True)``)."""
    q2 = importlib.import_module(PACKAGE + ".qwen2")
    try:
        q2.reference_package()
    except ImportError as exc:
        return {"unavailable": f"reference package not installed: {exc}"}
    gen_mod = importlib.import_module("qwen_int4.generation")
    model = q2.build_random_qwen2(device=device, seed=0)
    prompt = torch.randint(0, model.config.vocab_size, (1, prompt_len),
                           generator=torch.Generator().manual_seed(20260831)).to(device)

    def timed(fn):
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        out = fn()
        b.record()
        b.synchronize()
        return a.elapsed_time(b), out

    result = {"model": "Qwen2-1.5B random-init W4G64 RTN (reference model.py)", "batch": 1,
              "prompt_tokens": prompt_len,
              "harness": "cuDNN SDPA backend disabled (per-call graph builds as the KV cache grows)"}
    cudnn_sdp = torch.backends.cuda.cudnn_sdp_enabled()
    torch.backends.cuda.enable_cudnn_sdp(False)
    with torch.inference_mode():
        for leg, backend, fuse, steps in (("b200", "b200", False, new_tokens),
                                          ("b200_fused_mlp", "b200", True, new_tokens),
                                          ("torch", "torch", False, 8)):
            q2.register_with_reference(q2.reference_package().__name__, fuse_mlp=fuse)
            model.set_backend(backend)
            gen_mod.greedy_generate_cached(model, prompt, max_new_tokens=3)  # warm-up at full length
            prefill_ms, _ = timed(lambda: model(prompt, use_cache=True))
            total_ms, _ = timed(lambda: gen_mod.greedy_generate_cached(model, prompt, max_new_tokens=steps))
            decode_ms = max(total_ms - prefill_ms, 1e-6)
            result[leg] = {"prefill_ms": prefill_ms, "new_tokens": steps,
                               "generate_ms": total_ms, "decode_tok_s": steps / (decode_ms / 1e3)}
    torch.backends.cuda.enable_cudnn_sdp(cudnn_sdp)
    result["decode_tok_s"] = result["b200"]["decode_tok_s"]
    result["decode_tok_s_fused_mlp"] = result["b200_fused_mlp"]["decode_tok_s"]
    del model
    torch.cuda.empty_cache()
    return result


def split_prefill(device, dist, world: int, m: int = 4096, reps: int = 10) -> dict:
    """Column-split prefill: one Qwen2-1.5B MLP (gate/up/down) at M tokens with
    gate/up/down column-split over the ranks and NCCL all-gathers (two per
    MLP). Time is the max over ranks of CUDA-event time per forward."""
    par = importlib.import_module(PACKAGE + ".parallel")
    from types import SimpleNamespace

    gen = torch.Generator(device=device).manual_seed(5)

    def qlinear(n, k):
        qw, sc, z = quantize_symmetric_rtn_gpu(n, k, gen, device)
        return SimpleNamespace(qweight=qw, scales=sc, zeros=z, bias=None, in_features=k, out_features=n)

    mlp = SimpleNamespace(gate_proj=qlinear(8960, 1536), up_proj=qlinear(8960, 1536), down_proj=qlinear(1536, 8960))
    split = par.ColumnParallelMLP(mlp)
    x = torch.randn(m, 1536, device=device, generator=gen).to(torch.bfloat16)
    for _ in range(3):
        split(x)
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        split(x)
    b.record()
    b.synchronize()
    ms = torch.tensor([a.elapsed_time(b) / reps], device=device)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    flops = 2 * m * 1536 * 8960 * 3
    return {"m": m, "ms_per_mlp": float(ms.item()), "TFLOPs": flops / (float(ms.item()) / 1e3) / 1e12,
            "collectives": "2 x all_gather_into_tensor (NCCL) per MLP", "ranks": world}


def config_sweep(lib, layers, device, gen, tensor_peak: float) -> dict:
    """Secondary figures for the workloads the headline does not cover:
    config 0 (gate, symmetric, M = 1/4/16), config 1's remaining M points
    (8/32/128/512, seven shapes of four layers), config 2 (AWQ-style
    asymmetric down_proj, M = 1/16/2048) and config 4's batch-64 decode step
    (196 linears at M = 64). Library-chosen kernels (GEMV up to M = 16,
    tensor cores above), CUDA graphs of C-ABI launches."""
    q2 = importlib.import_module(PACKAGE + ".qwen2")
    out = {}

    def run(chain, reps=10):
        t = time_graph(chain.graph(), reps=reps, warmup=3)
        return t, chain.bytes() / (t / 1e3) / 1e9, chain.flops() / (t / 1e3) / 1e12

    gates = [layer[4] for layer in layers]
    out["cfg0_gate_sym_GBps"] = {f"m{m}": round(run(Chain(lib, gates, m, device, gen))[1], 1) for m in (1, 4, 16)}
    sweep = {}
    for m in (8, 32, 128, 512):
        t, gbps, tf = run(Chain(lib, [e for layer in layers[:4] for e in layer], m, device, gen))
        sweep[f"m{m}"] = {"GBps": round(gbps, 1), "TFLOPs": round(tf, 2), "ms_4_layers": round(t, 4)}
    out["cfg1_seven_shapes"] = sweep
    # Config 2: per-input-channel scaled weights, asymmetric RTN, activations divided by the channel scale.
    chan = torch.exp(torch.empty(8960, device=device).uniform_(float(np.log(0.5)), float(np.log(2.0)), generator=gen))
    downs = []
    for _ in range(4):
        w = torch.randn(1536, 8960, device=device, generator=gen) * 0.02 * chan
        qw, sc, z = q2.quantize_asymmetric_rtn_torch(w.to(torch.bfloat16).float())
        downs.append({"name": "down_awq", "k": 8960, "n": 1536, "qweight": qw, "scales": sc, "zeros": z, "bias": None})
    cfg2 = {}
    for m in (1, 16, 2048):
        chain = Chain(lib, downs, m, device, gen)
        chain.x = [(x.float() / chan).to(torch.bfloat16) for x in chain.x]
        t, _, tf = run(chain)
        nbytes = sum(alg_bytes(m, 1536, 8960, False, asym=True) for _ in downs)
        cfg2[f"m{m}"] = {"GBps": round(nbytes / (t / 1e3) / 1e9, 1)} if m <= 16 else \
            {"TFLOPs": round(tf, 1), "frac_of_bf16_peak": round(tf / tensor_peak, 3)}
    out["cfg2_awq_down"] = cfg2
    t, _, tf = run(Chain(lib, [e for layer in layers for e in layer], 64, device, gen), reps=5)
    out["cfg4_decode_m64"] = {"ms_per_step": round(t, 3), "tokens_per_s": round(64 / (t / 1e3), 1),
                              "TFLOPs": round(tf, 1), "note": "196 linears at M = 64 (tensor-core path), one GPU"}
    return out


def profile_case(kind: str) -> None:
    """Small, ncu-sized run of the dominant kernel (see --profile-case)."""
    device = torch.device("cuda", 0)
    lib = importlib.import_module(PACKAGE + "._lib").load()
    gen = torch.Generator(device=device).manual_seed(0)
    ents = []
    for _ in range(8):
        qw, sc, z = quantize_symmetric_rtn_gpu(8960, 1536, gen, device)
        ents.append({"name": "gate", "k": 1536, "n": 8960, "qweight": qw, "scales": sc, "zeros": z, "bias": None})
    m, algo = (1, 1) if kind == "gemv" else (2048, 2)
    chain = Chain(lib, ents if kind == "gemv" else ents[:2], m, device, gen, algo=algo)
    for _ in range(3):
        chain.launch()
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": kind, "launches": 3 * len(chain.entries), "m": m}))


def load_traffic() -> dict:
    path = ROOT / "profiles" / "traffic.json"
    if path.exists():
        return json.loads(path.read_text())
    return {}


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=200)
    parser.add_argument("--warmup", type=int, default=10)
    parser.add_argument("--impl", choices=["b200", "reference"], default="b200")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-gemm", action="store_true")
    parser.add_argument("--no-model", action="store_true", help="skip the Qwen2-1.5B decode tok/s section")
    parser.add_argument("--no-configs", action="store_true",
                        help="skip the secondary workload figures (gate M=1/4/16, seven shapes M=8..512, AWQ down, batch-64 linears)")
    parser.add_argument("--profile-case", choices=["gemv", "gemm"],
                        help="run only a small case of one kernel for an ncu capture: 8 gate-shaped "
                             "weights (1536->8960, 59 MB), 3 chained launches at M=1 (gemv) or M=2048 (gemm)")
    args = parser.parse_args()
    if args.warmup < 3:
        parser.error("--warmup must be at least 3")
    if args.impl == "reference":
        run_reference(args)
        return
    if args.profile_case:
        profile_case(args.profile_case)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=device)

    pkg = importlib.import_module(PACKAGE)
    lib = importlib.import_module(PACKAGE + "._lib").load()
    layers = build_model_weights(device, seed=1234 + rank)
    gen = torch.Generator(device=device).manual_seed(99 + rank)
    entries = [e for layer in layers for e in layer]
    step_chain = Chain(lib, entries, 1, device, gen)
    step_graph = step_chain.graph()
    step_bytes = step_chain.bytes()
    launches_per_step = len(entries)

    # Timed region: K replays of the step graph, barrier + sync on both sides.
    for _ in range(args.warmup):
        step_graph.replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        start.record()
        for _ in range(args.steps):
            step_graph.replay()
        end.record()
        end.synchronize()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    ms = start.elapsed_time(end)
    if dist:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    value = step_bytes * world * args.steps / (ms / 1e3) / 1e9

    # Dominant kernel: the gate GEMV at M=1, chained over the 28 layers.
    per_shape = {}
    for idx, (name, k, n, has_bias) in enumerate(SHAPES):
        chain = Chain(lib, [layer[idx] for layer in layers], 1, device, gen)
        g = chain.graph()
        t = time_graph(g, reps=20, warmup=3)
        per_shape[name] = {"m": 1, "us_per_launch": t * 1e3 / LAYERS,
                           "GBps": chain.bytes() / (t / 1e3) / 1e9}
    gate = per_shape["gate"]

    # The same step with the input-sharing linears grouped per launch.
    grouped = GroupedChain(lib, layers, device, gen)
    t = time_graph(grouped.graph(), reps=20, warmup=3)
    decode_grouped = {"launches_per_step": len(grouped.launches), "ms_per_step": t,
                      "GBps": step_bytes / (t / 1e3) / 1e9,
                      "api": "qi4_w4g64_linear_multi (q/k/v and gate/up grouped), CUDA graph"}
    peaks_path = ROOT / "MEASURED_PEAKS.json"
    if peaks_path.exists():
        peaks = json.loads(peaks_path.read_text())
        hbm_peak, peak_src = float(peaks["hbm_gbs"]), "measured"
        tensor_peak = float(peaks.get("bf16_tflops", 1590.0))
    else:
        hbm_peak, peak_src, tensor_peak = 6650.0, "fallback", 1590.0
    traffic = load_traffic().get("gemv_gate_m1_bytes_per_launch")
    roofline = {"bound": "hbm", "kernel": "gemv_mma_kernel (gate 1536->8960, M=1)",
                "achieved": gate["GBps"], "peak": hbm_peak, "unit": "GB/s",
                "frac": gate["GBps"] / hbm_peak, "peak_source": peak_src,
                "traffic": traffic, "algorithmic_bytes_per_launch": alg_bytes(1, 8960, 1536, False)}

    configs = None
    if not args.no_configs and world == 1:
        configs = config_sweep(lib, layers, device, gen, tensor_peak)

    # GEMM at M=2048 (tensor-core kernel) over one layer's seven shapes.
    gemm = None
    if not args.no_gemm and world == 1:
        gemm = {"m": 2048, "per_shape": {}}
        total_flops, total_ms = 0, 0.0
        for idx, (name, k, n, has_bias) in enumerate(SHAPES):
            chain = Chain(lib, [layers[i][idx] for i in range(4)], 2048, device, gen, algo=2)
            try:
                g = chain.graph()
            except RuntimeError:
                gemm = None
                break
            t = time_graph(g, reps=10, warmup=3)
            tf = chain.flops() / (t / 1e3) / 1e12
            gemm["per_shape"][name] = {"TFLOPs": tf, "us_per_launch": t * 1e3 / 4}
            total_flops += chain.flops()
            total_ms += t
        if gemm is not None:
            gemm["TFLOPs_all_shapes"] = total_flops / (total_ms / 1e3) / 1e12
            gemm["frac_of_bf16_peak"] = gemm["TFLOPs_all_shapes"] / tensor_peak

    # End to end through the public API with host buffers.
    x_host = torch.cat([x.view(-1) for x in step_chain.x]).cpu().pin_memory()
    out_host = torch.empty(sum(e["n"] for e in entries), dtype=torch.bfloat16).pin_memory()
    offsets, off = [], 0
    for e in entries:
        offsets.append(off)
        off += e["k"]

    def e2e_step():
        xd = x_host.to(device, non_blocking=True)
        outs = []
        for e, o in zip(entries, offsets):
            outs.append(pkg.b200_w4g64_linear(
                xd[o:o + e["k"]].view(1, e["k"]), e["qweight"], e["scales"], e["zeros"], e["bias"],
                out_features=e["n"], in_features=e["k"], group_size=64, packing="canonical"))
        out_host.copy_(torch.cat([t.view(-1) for t in outs]), non_blocking=True)

    e2e_steps = max(3, min(args.steps, 20))
    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    es.record()
    for _ in range(e2e_steps):
        e2e_step()
    ee.record()
    ee.synchronize()
    e2e_ms = es.elapsed_time(ee) / e2e_steps
    if dist:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e = {"value": step_bytes * world / (e2e_ms / 1e3) / 1e9, "unit": UNIT,
           "h2d_bytes_per_step": x_host.numel() * 2, "d2h_bytes_per_step": out_host.numel() * 2,
           "ms_per_step": e2e_ms, "api": "b200_w4g64_linear per linear (Python call; C++ binding of the C ABI)"}

    split = split_prefill(device, dist, world) if dist else None

    decode = None
    if not args.no_model and world == 1:
        del layers, entries, step_chain, step_graph
        torch.cuda.empty_cache()
        decode = e2e_decode(device)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_linear_sample()

    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    print(json.dumps({
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random-init W4G64 RTN weights)",
        "config": {"workload": WORKLOAD, "m": 1, "layers": LAYERS, "linears_per_step": launches_per_step,
                   "bytes_per_step": step_bytes, "parallelism": f"replicas x{world}",
                   "l2": "inputs larger than L2 (655 MB packed weights per step); no flush"},
        "gpu_launches": launches_per_step * args.steps,
        "roofline": roofline, "per_shape_m1": per_shape, "decode_step_grouped": decode_grouped,
        "gemm_m2048": gemm, "configs": configs, "qwen2_decode": decode,
        "split_prefill_mlp": split,
        "e2e": e2e, "cpu_baseline": cpu, "clocks": clocks.summary(),
    }))


if __name__ == "__main__":
    main()
