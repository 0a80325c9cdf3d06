#!/usr/bin/env python
"""Benchmark of the MoE training step's hot path on B200.

Workload ("config 2"): one isolated ScatterMoE
GLUMLP layer, forward + backward, bf16, including the aux-loss-free routing:
  16384 tokens x d_model 1024 (N(0,1)), 64 routed SwiGLU experts of ffn 512,
  top-8, router logits N(0,1) + per-expert bias N(0,0.1) (skewed loads),
  expert weights N(0,0.02), upstream gradient N(0,1).
A step = sigmoid(logits) -> biased top-k (libzs) -> GLUMLP forward (libzs
grouped GEMMs) -> backward to x, routing weights (and logits) and both expert
weight stacks.  With --gpus N > 1 every rank runs its own 16384 tokens (data
parallel, weak scaling) and the expert-weight gradients are all-reduced over
NCCL each step, as a data-parallel training step does.

Prints one JSON line (rank 0).  --impl reference times the reference
algorithm's CPU restatement (oracle/) on the host cores instead.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "architecture-zarelga-superposition_b200"
for _p in (str(PKG), str(ROOT)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

CFG = dict(T=16384, d=1024, E=64, k=8, f=512)
METRIC = "training tokens/sec (whole box)"
UNIT = "tokens/s"
WORKLOAD = ("config2: isolated ScatterMoE GLUMLP layer fwd+bwd with aux-loss-free routing, "
            "T=16384 d=1024 E=64 ffn=512 top-8, bf16")


def flops_per_step(T, d, E, k, f):
    """Algorithmic tensor-core FLOPs of one step: 6 grouped GEMMs of
    2*n*d*f*{2,1} (fwd up/down), x2 for backward (dX and dW), n = T*k."""
    n = T * k
    return 18 * n * d * f


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            j = json.loads(p.read_text())
            return float(j["bf16_tflops"]), float(j["bf16_tflops_sustained"]), float(j["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 1590.0, 1400.0, 6650.0, "fallback"


# ---------------------------------------------------------------- CPU oracle

def _np_inputs(T, d, E, k, f, seed):
    import numpy as np

    from oracle.routing import round_bf16

    rng = np.random.default_rng(seed)
    logits = round_bf16(rng.standard_normal((T, E), dtype=np.float32))
    bias = (rng.standard_normal(E, dtype=np.float32) * 0.1).astype(np.float32)
    x = round_bf16(rng.standard_normal((T, d), dtype=np.float32))
    W1 = round_bf16(rng.standard_normal((E, 2 * f, d), dtype=np.float32) * 0.02)
    W2 = round_bf16(rng.standard_normal((E, d, f), dtype=np.float32) * 0.02)
    dy = round_bf16(rng.standard_normal((T, d), dtype=np.float32))
    return logits, bias, x, W1, W2, dy


def cpu_oracle_step(inp, k):
    import numpy as np

    from oracle import routing as R
    from oracle import scattermoe as S

    logits, bias, x, W1, W2, dy = inp
    probs = R.round_bf16(1.0 / (1.0 + np.exp(-logits)))
    idx, w = R.gate_topk(probs, bias, k, dtype="bf16")
    _, saved = S.glu_mlp_forward(x, w, idx, W1, W2, dtype="bf16")
    S.glu_mlp_backward(dy, x, w, W1, W2, saved, dtype="bf16")


def blas_threads():
    try:
        from threadpoolctl import threadpool_info

        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        return max(n) if n else 1
    except Exception:
        return os.cpu_count() or 1


def cpu_baseline(target_s=10.0, max_tokens=1024):
    """Tokens/s of the oracle on a bounded sample of the config-2 workload."""
    c = CFG
    T = 64
    while True:
        inp = _np_inputs(T, c["d"], c["E"], c["k"], c["f"], seed=7)
        t0 = time.perf_counter()
        cpu_oracle_step(inp, c["k"])
        dt = time.perf_counter() - t0
        if dt * 2 > target_s or T * 2 > max_tokens:
            break
        T *= 2
    return {"value": T / dt, "unit": UNIT, "cores": blas_threads(), "kind": "port",
            "sample": f"{T} of 16384 tokens of config 2 (same d/E/ffn/top-k), one fwd+bwd in {dt:.2f} s, "
                      "oracle/ numpy float64 on f32/bf16-exact inputs"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    c = CFG
    # calibrate the per-step sample so the whole run stays within minutes
    T = 64
    while True:
        inp = _np_inputs(T, c["d"], c["E"], c["k"], c["f"], seed=11)
        t0 = time.perf_counter()
        cpu_oracle_step(inp, c["k"])
        dt = time.perf_counter() - t0
        if dt * 2 * (args.steps + args.warmup) > 150 or T >= 1024:
            break
        T *= 2
    for _ in range(args.warmup):
        cpu_oracle_step(inp, c["k"])
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        cpu_oracle_step(inp, c["k"])
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = T * args.steps / total
    cores = blas_threads()
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": WORKLOAD, "sample_tokens_per_step": T},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": f"{T} tokens of config 2 per step through oracle/ (numpy)"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU arm

class ClockSampler:
    FIELDS = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self, t0=None, t1=None):
        """Summarise the samples taken between host times t0 and t1."""
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path).read().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                clk, cmax = float(parts[1]), float(parts[2])
            except ValueError:
                continue
            if t0 is not None and not (t0 <= ts <= t1):
                continue
            sm.append(clk)
            mx = max(mx, cmax)
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def run_gpu(args):
    import torch
    import torch.distributed as dist

    from modeling.moe_gate import GateTopK
    from scattermoe.mlp import GLUMLP
    from zs_b200 import _lib as Z

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)

    c = dict(CFG)
    if args.tokens:
        c["T"] = args.tokens
    T, d, E, k, f = c["T"], c["d"], c["E"], c["k"], c["f"]
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    bf = torch.bfloat16
    logits = torch.randn(T, E, device=dev, generator=g).to(bf)
    bias = torch.randn(E, device=dev, generator=g) * 0.1
    x = torch.randn(T, d, device=dev, generator=g).to(bf)
    dy = torch.randn(T, d, device=dev, generator=g).to(bf)
    wg = torch.Generator(device=dev).manual_seed(99)  # identical weights on every rank
    m = GLUMLP(d, f, E, k).to(dev)
    with torch.no_grad():
        m.experts.weight.copy_(torch.randn(E, 2 * f, d, device=dev, generator=wg) * 0.02)
        m.output_experts.weight.copy_(torch.randn(E, d, f, device=dev, generator=wg) * 0.02)
    m = m.to(bf)
    # weight gradients straight from the GEMM epilogues into .grad; with N > 1 each one's
    # all-reduce starts as soon as it is written and overlaps the rest of the backward
    m.fuse_weight_grad = True
    params = [m.experts.weight, m.output_experts.weight]
    reducer = None
    if world > 1:
        from zs_b200.dp import GradAllReducer

        reducer = GradAllReducer(params, bucket_mb=1.0, engine=args.dp_engine)

    def step(xs, ls, dys):
        for p_ in params:
            p_.grad = None
        xs.requires_grad_(True)
        ls.requires_grad_(True)
        probs = torch.sigmoid(ls)
        idx, w = GateTopK.apply(probs, bias, k)
        y = m(xs, w, idx)
        y.backward(dys)
        if reducer is not None:
            reducer.finish()
        return xs.grad

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(max(args.warmup, 1)):
        step(x.detach(), logits.detach(), dy)
    torch.cuda.synchronize()
    barrier()

    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.5)  # let nvidia-smi start sampling
    Z.INSTR.events = {}
    Z.INSTR.timing = True
    launches0 = Z.INSTR.launches
    stream = torch.cuda.current_stream()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    barrier()
    host_t0 = time.time()
    t_start.record(stream)
    for _ in range(args.steps):
        step(x.detach(), logits.detach(), dy)
    t_end.record(stream)
    torch.cuda.synchronize()
    barrier()
    host_t1 = time.time()
    Z.INSTR.timing = False
    launches = Z.INSTR.launches - launches0
    clocks = sampler.stop(host_t0, host_t1)
    ms = t_start.elapsed_time(t_end)
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())

    # per-kernel durations of the grouped GEMM launches (same stream, same region)
    kern = {}
    for name, evs in Z.INSTR.events.items():
        durs = [s.elapsed_time(e) for s, e, *_ in evs]
        kern[name] = {"launches": len(durs), "avg_ms": sum(durs) / len(durs), "total_ms": sum(durs)}
    gemm_ms = sum(v["total_ms"] for v in kern.values())

    # End-to-end through the public API with host buffers: every step copies its
    # inputs from pinned host memory and reads dX back.  The copies run on their own
    # streams into double-buffered device inputs (a prefetching loader), so step i+1's
    # upload and step i-1's download overlap step i's compute; the timed region spans
    # the first upload to the last download.
    xh = x.detach().cpu().pin_memory()
    lh = logits.detach().cpu().pin_memory()
    dyh = dy.detach().cpu().pin_memory()
    dxh = [torch.empty((T, d), dtype=bf).pin_memory() for _ in range(2)]
    slots = [(torch.empty_like(x), torch.empty_like(logits), torch.empty_like(dy)) for _ in range(2)]
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    e_steps = 0 if args.no_e2e else max(1, args.steps)
    torch.cuda.synchronize()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    uploaded = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    downloaded = torch.cuda.Event()

    def upload(i):
        xd, ld, dyd = slots[i % 2]
        with torch.cuda.stream(h2d):
            if i >= 2:
                h2d.wait_event(consumed[i % 2])
            xd.copy_(xh, non_blocking=True)
            ld.copy_(lh, non_blocking=True)
            dyd.copy_(dyh, non_blocking=True)
            uploaded[i % 2].record(h2d)

    e0.record(stream)
    h2d.wait_event(e0)
    if e_steps:
        upload(0)
    for i in range(e_steps):
        if i + 1 < e_steps:
            upload(i + 1)
        xd, ld, dyd = slots[i % 2]
        stream.wait_event(uploaded[i % 2])
        dx = step(xd.detach(), ld.detach(), dyd)
        consumed[i % 2].record(stream)
        with torch.cuda.stream(d2h):
            d2h.wait_event(consumed[i % 2])
            dx.record_stream(d2h)
            dxh[i % 2].copy_(dx, non_blocking=True)
            downloaded.record(d2h)
    stream.wait_event(downloaded)
    e1.record(stream)
    torch.cuda.synchronize()
    e_ms = max(e0.elapsed_time(e1), 1e-9)
    if world > 1:
        tt = torch.tensor([e_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e_ms = float(tt.item())
        dist.barrier()
    err = Z.device_error()

    if rank == 0:
        burst, sustained, hbm, src = measured_peaks()
        fl = flops_per_step(T, d, E, k, f)
        achieved = fl * args.steps / (gemm_ms * 1e-3) / 1e12 if gemm_ms > 0 else None
        traffic = None
        tf = ROOT / "profiles" / "grouped_gemm_traffic.json"
        if tf.exists():
            try:
                traffic = json.loads(tf.read_text()).get("bytes_per_launch_avg")
            except Exception:
                traffic = None
        value = world * T * args.steps / (ms * 1e-3)
        mfu = value * (fl / T) / (world * sustained * 1e12)
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "tokens_per_gpu": T, "d_model": d, "experts": E, "ffn": f, "top_k": k,
                       "parallelism": f"dp{world}", "l2": "working set ~3 GB per step, larger than the 126 MB L2",
                       "grad_allreduce": (None if world == 1 else
                                          "copy engines over NVLink peer memory (zs_ce_allreduce)"
                                          if args.dp_engine == "ce" else "NCCL"),
                       "mfu_sustained_peak": mfu, "flops_per_step_per_gpu": fl},
            "roofline": {"bound": "tensor", "kernel": "grouped_gemm_kernel (6 launches per step: up+SwiGLU, down, "
                                                      "2 input-gradient, 2 weight-gradient)",
                         "achieved": achieved, "peak": sustained, "unit": "TFLOP/s",
                         "frac": (achieved / sustained) if achieved else None, "traffic": traffic,
                         "peak_source": f"{src} bf16_tflops_sustained (kernel timed inside the step loop)",
                         "kernels": kern},
            "cpu_baseline": None,
            "e2e": None if not e_steps else {"value": world * T * e_steps / (e_ms * 1e-3), "unit": UNIT,
                    "h2d_bytes_per_step": xh.numel() * 2 + lh.numel() * 2 + dyh.numel() * 2,
                    "d2h_bytes_per_step": dxh[0].numel() * 2,
                    "overlap": "uploads and downloads on separate streams, double-buffered inputs"},
            "gpu_launches": launches,
            "clocks": clocks,
            "device_error": err,
        }
        if args.tokens and args.tokens != CFG["T"]:
            line["config"]["workload"] = WORKLOAD.replace("T=16384", f"T={T} (reduced)")
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_config3(args):
    """cut cross entropy forward + backward, bf16, hidden
    16384 x 2048 N(0,1), classifier 131072 x 2048 N(0,0.02), uniform targets
    with 5 % ignore_index (CCE) or 4 targets per position (--mcce)."""
    import torch

    from zs_b200 import _lib as Z
    from zs_b200.xent import fused_linear_cross_entropy

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    T, D, V = (args.tokens or 16384), 2048, 131072
    g = torch.Generator(device=dev).manual_seed(3)
    h = torch.randn(T, D, device=dev, generator=g).to(torch.bfloat16)
    c = (torch.randn(V, D, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    if args.mcce:
        labels = torch.randint(0, V, (T, 4), device=dev, generator=g)
        s = torch.full((T,), 4, dtype=torch.int32, device=dev)
    else:
        labels = torch.randint(0, V, (T, 1), device=dev, generator=g)
        s = (torch.rand(T, device=dev, generator=g) >= 0.05).to(torch.int32)

    def step():
        hh = h.detach().requires_grad_(True)
        cc = c.detach().requires_grad_(True)
        loss = fused_linear_cross_entropy(hh, cc, labels, s)
        loss.backward()
        return loss

    for _ in range(max(args.warmup, 1)):
        step()
    torch.cuda.synchronize()
    Z.INSTR.events = {}
    Z.INSTR.timing = True
    l0 = Z.INSTR.launches
    sampler = ClockSampler(0)
    sampler.start()
    time.sleep(0.5)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ht0 = time.time()
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    ht1 = time.time()
    Z.INSTR.timing = False
    clocks = sampler.stop(ht0, ht1)
    ms = t0.elapsed_time(t1)
    kern = {}
    for name, evs in Z.INSTR.events.items():
        durs = [a.elapsed_time(b) for a, b, *_ in evs]
        kern[name] = {"launches": len(durs), "avg_ms": sum(durs) / len(durs)}
    _, sustained, _, src = measured_peaks()
    fl = 3 * 2 * T * V * D  # algorithmic: forward logits, dH, dW (the backward's logit recompute excluded)
    executed = 4 * 2 * T * V * D
    value = T * args.steps / (ms * 1e-3)
    achieved = executed * args.steps / (ms * 1e-3) / 1e12
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": ("config3: MCCE 4 targets" if args.mcce else "config3: CCE 5% ignored")
                       + f", fwd+bwd, T={T} D={D} V={V}, bf16",
                       "algorithmic_tflop_per_step": fl / 1e12, "executed_tflop_per_step": executed / 1e12,
                       "useful_tflops": fl * args.steps / (ms * 1e-3) / 1e12},
            "roofline": {"bound": "tensor", "kernel": "grouped_gemm_kernel (classifier GEMMs: LSE forward, "
                                                      "logit-gradient recompute, dH, dW)",
                         "achieved": achieved, "peak": sustained, "unit": "TFLOP/s", "frac": achieved / sustained,
                         "traffic": None, "peak_source": f"{src} bf16_tflops_sustained", "kernels": kern},
            "gpu_launches": Z.INSTR.launches - l0, "clocks": clocks, "device_error": Z.device_error()}
    print(json.dumps(line), flush=True)


KERNEL_FAMILIES = {
    # grouped_gemm_kernel (csrc/zs_gemm.cu): every tcgen05 GEMM launch of the step
    "grouped_gemm_kernel": ("newton_schulz5", "up_swiglu", "down_dx", "down_fwd", "down_dw", "up_dw", "up_dx",
                            "xent_fwd", "xent_bwd", "scatter2scatter", "groupXtY", "proj_", "shared_expert"),
    # attn_fwd_kernel / attn_bwd_* (csrc/zs_attn.cu)
    "attention": ("attention_fwd", "attention_bwd"),
}


def _family(name):
    for fam, keys in KERNEL_FAMILIES.items():
        if any(name.startswith(k) for k in keys):
            return fam
    return None


def kernel_table(steps):
    """Per instrumented region: launches per step, ms per step and achieved TFLOP/s, from the
    CUDA events recorded in the timed region (eager launches: every step; launches inside
    the recorded optimizer graph: the last replay, which is one step)."""
    from zs_b200 import _lib as Z

    out = {}
    for name, evs in Z.INSTR.events.items():
        durs = [s.elapsed_time(e) for s, e, _ in evs]
        fl = sum(f for _, _, f in evs)
        out[name] = {"launches_per_step": len(durs) / steps, "ms_per_step": sum(durs) / steps,
                     "tflop_per_step": fl / steps / 1e12, "graph": False}
    for name, evs in Z.INSTR.graph_events.items():
        durs = [s.elapsed_time(e) for s, e, _ in evs]
        fl = sum(f for _, _, f in evs)
        row = {"launches_per_step": len(durs), "ms_per_step": sum(durs), "tflop_per_step": fl / 1e12, "graph": True}
        prev = out.get(name)
        if prev is not None:  # both eager and recorded launches of one region
            row = {k: (prev[k] + row[k]) if k != "graph" else True for k in row}
        out[name] = row
    for r in out.values():
        r["achieved_tflops"] = (r["tflop_per_step"] / (r["ms_per_step"] * 1e-3)) if r["ms_per_step"] > 0 else None
    return out


def roofline_from_table(table, clocks):
    """Roofline of the dominant kernel family (largest share of the instrumented time):
    achieved = its algorithmic FLOPs / its summed CUDA-event time.  The peak is the burst
    cuBLAS figure when the timed region ran at the maximum SM clock, else the sustained one
    (the power-capped clock the sustained figure was measured at)."""
    burst, sustained, _, src = measured_peaks()
    fams = {}
    for name, r in table.items():
        fam = _family(name)
        if fam is None:
            continue
        f = fams.setdefault(fam, {"ms_per_step": 0.0, "tflop_per_step": 0.0, "regions": []})
        f["ms_per_step"] += r["ms_per_step"]
        f["tflop_per_step"] += r["tflop_per_step"]
        f["regions"].append(name)
    if not fams:
        return None
    for f in fams.values():
        f["achieved_tflops"] = f["tflop_per_step"] / (f["ms_per_step"] * 1e-3) if f["ms_per_step"] > 0 else None
    dom = max(fams, key=lambda k: fams[k]["ms_per_step"])
    at_max = bool(clocks and clocks.get("sm_max_mhz") and clocks["sm_mhz"] >= 0.95 * clocks["sm_max_mhz"])
    peak = burst if at_max else sustained
    ach = fams[dom]["achieved_tflops"]
    return {"bound": "tensor", "kernel": dom, "achieved": ach, "peak": peak, "unit": "TFLOP/s",
            "frac": (ach / peak) if ach else None, "traffic": None,
            "peak_source": (f"{src} bf16_tflops (burst: the timed region ran at the maximum SM clock)" if at_max else
                            f"{src} bf16_tflops_sustained (the timed region ran below the maximum SM clock)"),
            "families": fams}


def config4_model_config(layers=16):
    from modeling.model_config import ModelConfig

    return ModelConfig(vocab_size=65536, embed_size=1536, hidden_size=1536, transformer_depth=layers,
                       intermediate_size=768, n_experts=65, n_shared_experts=1, n_experts_per_token=6,
                       n_attention_heads=12, n_key_value_heads=4, attention_window_pattern=(None,) * layers,
                       max_position_embeddings=4096, sequence_length=4096, attention_sink=True)


def model_flops_per_token(cfg, seq_len):
    """6 * active matmul parameters (incl. the LM head) + 6 * L * H * hd * S
    (causal attention), the MFU numerator the metric is defined on."""
    d, hd = cfg.hidden_size, cfg.hidden_size // cfg.n_attention_heads
    kv = cfg.n_key_value_heads * hd
    attn = 2 * d * d + 2 * d * kv + d * cfg.n_attention_heads
    router = cfg.n_routed_experts * d
    shared = 3 * d * cfg.intermediate_size * cfg.n_shared_experts
    routed = cfg.n_experts_per_token * 3 * d * cfg.intermediate_size
    active = cfg.transformer_depth * (attn + router + shared + routed) + cfg.vocab_size * d
    return 6 * active + 6 * cfg.transformer_depth * cfg.n_attention_heads * hd * seq_len


WORKLOAD4 = ("config4: full MoE LM training step (forward, cut cross entropy, backward, MuonMD + AdamW + "
             "sparse-embedding optimizer, aux-loss-free bias update); L={L} d=1536 H=12/4 hd=128 gated sink "
             "attention, E=64+1 shared ffn=768 top-6, V=65536, seq 4096 x micro-batch {B} per GPU, bf16")


def run_config4(args):
    """BASELINE configs[3], the headline: the full MoE LM training step (forward, CCE loss,
    backward, MuonMD + AdamW + sparse embedding optimizer step, aux-loss-free bias update),
    micro-batch 8 x 4096 tokens per GPU, data parallel over N GPUs (weak scaling).  Every
    step draws fresh uniform token ids.  `value` times the step with the ids already in HBM;
    `e2e` times the same step with the ids and attention mask uploaded from pinned host
    memory every step and the loss read back to the host every step."""
    import torch
    import torch.distributed as dist

    from cut_cross_entropy import linear_cross_entropy
    from zs_b200 import _lib as Z
    from zs_b200.lm import MoELM
    from zs_b200.train import (auxillary_loss_free_update, build_muonmd_optimizer, build_next_token_loss_inputs,
                               enable_fused_weight_grad)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    pg = dist.group.WORLD if world > 1 else None
    cfg = config4_model_config(args.layers)
    torch.manual_seed(1234)
    model = MoELM(cfg).to(dev)
    enable_fused_weight_grad(model)
    # with N ranks the Newton-Schulz batches are split over the ranks (all-gathered)
    opt = build_muonmd_optimizer(model, dev, capture_warmup_steps=3, process_group=pg)
    reducer = None
    if world > 1:
        from zs_b200.dp import GradAllReducer

        # gradients averaged over ranks: each rank's loss is the mean over its own
        # batch, so the average is the gradient of the global batch mean
        reducer = GradAllReducer(list(model.parameters()), bucket_mb=64.0, average=True)
    B, S = args.micro_batch, 4096
    warmup = max(args.warmup, 5)
    g = torch.Generator(device=dev).manual_seed(77 + rank)
    nb = 4
    # fresh uniform token ids every step: a ring of device batches, each refilled after use
    batches = torch.randint(0, cfg.vocab_size, (nb, B, S), device=dev, generator=g)
    mask = torch.ones(B, S, dtype=torch.long, device=dev)
    it = [0]

    def train_step(ids, am):
        opt.zero_grad(set_to_none=False)
        with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
            emb, all_topk = model.headless_forward(ids)
            le, labels = build_next_token_loss_inputs(emb, ids, am)
            loss = linear_cross_entropy(le, model.get_classifier_weights(), labels, ignore_index=-100)
        loss.backward()
        if reducer is not None:
            reducer.finish()
        opt.step()
        auxillary_loss_free_update(model, all_topk, 1e-3, am, process_group=pg)
        return loss

    def step():
        i = it[0] % nb
        it[0] += 1
        loss = train_step(batches[i], mask)
        batches[i].random_(0, cfg.vocab_size, generator=g)
        return loss

    Z.INSTR.timing = True  # the optimizer graph recorded in warm-up carries its event nodes
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.5)
    Z.INSTR.events = {}
    l0 = Z.INSTR.launches
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ht0 = time.time()
    if args.profile_timed:
        torch.cuda.profiler.start()   # a profiler started with --profile-from-start off records from here
    t0.record()
    for _ in range(args.steps):
        loss = step()
    t1.record()
    torch.cuda.synchronize()
    if args.profile_timed:
        torch.cuda.profiler.stop()
    if world > 1:
        dist.barrier()
    ht1 = time.time()
    Z.INSTR.timing = False
    clocks = sampler.stop(ht0, ht1)
    launches = Z.INSTR.launches - l0
    ms = t0.elapsed_time(t1)
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    table = kernel_table(args.steps)
    loss_v = float(loss.item())

    # End to end through the public API with host buffers: every step uploads its ids and
    # attention mask from pinned host memory and reads the loss back into pinned memory.
    e_steps = 0 if args.no_e2e else max(1, min(args.steps, args.e2e_steps))
    ids_h = torch.randint(0, cfg.vocab_size, (nb, B, S), generator=torch.Generator().manual_seed(5 + rank))
    ids_h = ids_h.pin_memory()
    mask_h = torch.ones(B, S, dtype=torch.long).pin_memory()
    loss_h = torch.empty(max(e_steps, 1), dtype=torch.float32).pin_memory()
    ids_d = torch.empty(B, S, dtype=torch.long, device=dev)
    mask_d = torch.empty(B, S, dtype=torch.long, device=dev)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(e_steps):
        ids_d.copy_(ids_h[i % nb], non_blocking=True)
        mask_d.copy_(mask_h, non_blocking=True)
        lo = train_step(ids_d, mask_d)
        loss_h[i:i + 1].copy_(lo.detach().reshape(1), non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e_ms = max(e0.elapsed_time(e1), 1e-9)
    if world > 1:
        tt = torch.tensor([e_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e_ms = float(tt.item())
    err = Z.device_error()
    if rank == 0:
        burst, sustained, _, src = measured_peaks()
        fpt = model_flops_per_token(cfg, S)
        value = world * B * S * args.steps / (ms * 1e-3)
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": WORKLOAD4.format(L=cfg.transformer_depth, B=B),
                           "model": "config4 MoE LM (3.98 B total / 0.60 B active matmul parameters)",
                           "global_batch": world * B, "seq_len": S, "tokens_per_gpu_step": B * S,
                           "parallelism": f"dp{world}", "model_gflop_per_token": fpt / 1e9,
                           "mfu_of_sustained_peak": value * fpt / (world * sustained * 1e12),
                           "mfu_of_burst_peak": value * fpt / (world * burst * 1e12),
                           "l2": "working set per step tens of GB (weights alone 16 GB), far larger than the 126 MB L2",
                           "ids": "fresh uniform token ids every step", "loss": loss_v},
                "roofline": roofline_from_table(table, clocks),
                "kernels": table,
                "cpu_baseline": None,
                "e2e": None if not e_steps else {
                    "value": world * B * S * e_steps / (e_ms * 1e-3), "unit": UNIT,
                    "h2d_bytes_per_step": ids_d.numel() * 8 + mask_d.numel() * 8, "d2h_bytes_per_step": 4,
                    "steps": e_steps,
                    "path": "MoELM.headless_forward + cut_cross_entropy.linear_cross_entropy + backward + "
                            "optimizer.step + auxillary_loss_free_update; ids/mask H2D and loss D2H every step",
                    "last_loss": float(loss_h[e_steps - 1])},
                "gpu_launches": launches,
                "gpu_launches_note": "libzs kernels launched by eager calls in the timed region; the kernels of "
                                     "the replayed optimizer graphs are not counted",
                "clocks": clocks, "device_error": err}
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_config4(cfg)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def cpu_baseline_config4(cfg):
    """The reference's step restated on the CPU (oracle/model_step.py), on the box's host cores."""
    try:
        from oracle.model_step import time_config4_sample
    except ImportError as exc:
        return {"value": None, "unit": UNIT, "cores": None, "kind": "port", "sample": f"unavailable: {exc}"}
    return time_config4_sample(cfg_fields(cfg), budget_s=25.0)


def run_reference_config4(args):
    """--impl reference for config 4: the CPU restatement of the reference's step, timed on a
    bounded sample on the host cores (rank 0 only)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    try:
        from oracle.model_step import reference_arm
    except ImportError as exc:
        print(json.dumps({"impl": "reference", "unavailable": f"oracle/model_step.py missing: {exc}"}), flush=True)
        return
    line = reference_arm(cfg_fields(config4_model_config(args.layers)), args.steps, args.warmup,
                         micro_batch=args.micro_batch)
    line.update({"impl": "reference", "metric": METRIC, "unit": UNIT, "n_gpus": args.gpus,
                 "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "data": "synthetic"})
    print(json.dumps(line), flush=True)


def cfg_fields(cfg):
    keys = ("vocab_size", "hidden_size", "transformer_depth", "intermediate_size", "n_routed_experts",
            "n_shared_experts", "n_experts_per_token", "n_attention_heads", "n_key_value_heads", "rms_norm_eps",
            "rope_theta", "pos_rope_dims", "max_position_embeddings", "initializer_range")
    return {k: getattr(cfg, k) for k in keys}


def run_config5(args):
    """BASELINE configs[4]'s MoE layer, expert parallel: 128 routed SwiGLU experts of
    ffn 1024 at d_model 2048, top-8, split evenly over the N ranks (16 per GPU at N=8),
    32768 latent positions per GPU; a step = sigmoid + biased top-k routing ->
    dispatch all-to-all -> local grouped GEMMs -> combine all-to-all, forward and
    backward (ExpertParallelGLUMLP).  Router logits N(0,1) + bias N(0,0.1), expert
    weights N(0,0.02), upstream gradient N(0,1), as config 2."""
    import torch
    import torch.distributed as dist

    from modeling.moe_gate import GateTopK
    from scattermoe.expert_parallel import ExpertParallelGLUMLP
    from zs_b200 import _lib as Z

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl" if torch.cuda.is_available() else "gloo", timeout=datetime.timedelta(seconds=180),
                            device_id=dev, init_method=None if world > 1 else f"tcp://127.0.0.1:{_free_port()}",
                            world_size=world, rank=rank)
    T = args.tokens or 32768
    d, E, k, f = 2048, 128, 8, 1024
    g = torch.Generator(device=dev).manual_seed(2000 + rank)
    bf = torch.bfloat16
    logits = torch.randn(T, E, device=dev, generator=g).to(bf)
    bias = torch.randn(E, device=dev, generator=torch.Generator(device=dev).manual_seed(7)) * 0.1
    x = torch.randn(T, d, device=dev, generator=g).to(bf)
    dy = torch.randn(T, d, device=dev, generator=g).to(bf)
    m = ExpertParallelGLUMLP(d, f, E, k).to(dev)
    wg = torch.Generator(device=dev).manual_seed(99 + rank)
    with torch.no_grad():
        m.experts.weight.copy_(torch.randn(m.experts.weight.shape, device=dev, generator=wg) * 0.02)
        m.output_experts.weight.copy_(torch.randn(m.output_experts.weight.shape, device=dev, generator=wg) * 0.02)
    m = m.to(bf)
    m.fuse_weight_grad = True
    params = [m.experts.weight, m.output_experts.weight]

    def step(xs, ls, dys):
        for p_ in params:
            p_.grad = None
        xs.requires_grad_(True)
        ls.requires_grad_(True)
        idx, w = GateTopK.apply(torch.sigmoid(ls), bias, k)
        y = m(xs, w, idx)
        y.backward(dys)
        return xs.grad

    for _ in range(max(args.warmup, 3)):
        step(x.detach(), logits.detach(), dy)
    torch.cuda.synchronize()
    dist.barrier()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.5)
    Z.INSTR.events = {}
    Z.INSTR.timing = True
    l0 = Z.INSTR.launches
    stream = torch.cuda.current_stream()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    dist.barrier()
    ht0 = time.time()
    t0.record(stream)
    for _ in range(args.steps):
        step(x.detach(), logits.detach(), dy)
    t1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    ht1 = time.time()
    Z.INSTR.timing = False
    clocks = sampler.stop(ht0, ht1)
    ms = t0.elapsed_time(t1)
    tt = torch.tensor([ms], device=dev)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms = float(tt.item())
    kern = {}
    for name, evs in Z.INSTR.events.items():
        durs = [s.elapsed_time(e) for s, e, *_ in evs]
        kern[name] = {"launches": len(durs), "avg_ms": sum(durs) / len(durs), "total_ms": sum(durs)}
    gemm_ms = sum(v["total_ms"] for v in kern.values())
    err = Z.device_error()
    if rank == 0:
        burst, sustained, hbm, src = measured_peaks()
        fl = flops_per_step(T, d, E, k, f)  # per GPU: every rank's experts see T*k rows on average
        value = world * T * args.steps / (ms * 1e-3)
        achieved = fl * world * args.steps / (gemm_ms * 1e-3 * world) / 1e12 if gemm_ms > 0 else None
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": max(args.warmup, 3), "ms_per_step": ms / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": f"config5 MoE layer, expert parallel: T={T} latent positions per GPU, "
                                       f"d=2048, E=128 ({E // world} per GPU), ffn=1024, top-8, fwd+bwd with "
                                       "dispatch/combine all-to-all",
                           "parallelism": f"ep{world}", "mfu_sustained_peak": value * (fl / T) / (world * sustained * 1e12)},
                "roofline": {"bound": "tensor", "kernel": "grouped_gemm_kernel (rank 0's launches)",
                             "achieved": achieved, "peak": sustained, "unit": "TFLOP/s",
                             "frac": (achieved / sustained) if achieved else None, "traffic": None,
                             "peak_source": f"{src} bf16_tflops_sustained", "kernels": kern},
                "gpu_launches": Z.INSTR.launches - l0, "clocks": clocks, "device_error": err}
        print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def config5_model_config(layers):
    from modeling.model_config import ModelConfig

    return ModelConfig(vocab_size=65536, embed_size=2048, hidden_size=2048, transformer_depth=layers,
                       intermediate_size=1024, n_experts=129, n_shared_experts=1, n_experts_per_token=8,
                       n_attention_heads=16, n_key_value_heads=4, attention_window_pattern=(None,) * layers,
                       max_position_embeddings=8192, sequence_length=8192)


def run_config5_model(args):
    """BASELINE configs[4] as a whole training step: the 2048-wide MoE LM (16 heads of 128, 128
    routed experts of ffn 1024 + 1 shared, top-8, V 65536) on token-superposition batches: 8192
    latent positions per sequence, each a bag of 4 raw token ids (the bag-mean embedding), the
    next position's 4 ids as the multi-target MCCE labels (s = 4 everywhere), micro-batch 4 per
    GPU, uniform synthetic ids drawn fresh every step; forward, MCCE loss, backward, MuonMD +
    AdamW + sparse-embedding optimizer, aux-loss-free bias update.  With N > 1 the routed
    experts are split over the ranks (expert parallel, all-to-all dispatch/combine) and the
    other parameters are data parallel.  Depth: --layers (default 4 per GPU up to 24: the
    24-layer model holds 19 B expert parameters and needs several GPUs' memory)."""
    import torch
    import torch.distributed as dist

    from modeling.mcce_fast_v2 import mcce_raw_token_mean_v2
    from zs_b200 import _lib as Z
    from zs_b200.data import bag_label_entropy_floor, ce_equivalent_reducible_loss
    from zs_b200.lm import MoELM
    from zs_b200.train import auxillary_loss_free_update, build_muonmd_optimizer, enable_fused_weight_grad

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    pg = dist.group.WORLD if world > 1 else None
    layers = args.layers_c5 or min(24, 4 * world)
    cfg = config5_model_config(layers)
    torch.manual_seed(4321)
    model = MoELM(cfg).to(dev)
    enable_fused_weight_grad(model)
    expert_params = set()
    if world > 1:
        from scattermoe.expert_parallel import shard_experts

        for m in shard_experts(model, pg):
            expert_params.update(id(p) for p in m.parameters())
    # expert weights differ between ranks, so Newton-Schulz is not split over them
    opt = build_muonmd_optimizer(model, dev, capture_warmup_steps=3, process_group=None)
    reducer = None
    if world > 1:
        from zs_b200.dp import GradAllReducer

        reducer = GradAllReducer([p for p in model.parameters() if id(p) not in expert_params], bucket_mb=64.0,
                                 average=True)
    B, S, bag = args.micro_batch_c5, 8192, 4
    V = cfg.vocab_size
    warmup = max(args.warmup, 5)
    g = torch.Generator(device=dev).manual_seed(500 + rank)
    nb = 3
    batches = torch.randint(0, V, (nb, B, S, bag), device=dev, generator=g)
    mask = torch.ones(B, S, dtype=torch.long, device=dev)
    s_full = torch.full((B * (S - 1),), bag, dtype=torch.long, device=dev)
    it = [0]

    def train_step(ids):
        opt.zero_grad(set_to_none=False)
        with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
            emb, all_topk = model.headless_forward(ids)
            hidden = emb[:, :-1].reshape(-1, emb.size(-1))
            labels = ids[:, 1:].reshape(-1, bag)
            raw = mcce_raw_token_mean_v2(hidden, model.get_classifier_weights(), labels, s_full)
        floor = bag_label_entropy_floor(labels, s_full)
        loss, _ = ce_equivalent_reducible_loss(raw, V, floor)
        loss.backward()
        if reducer is not None:
            reducer.finish()
        opt.step()
        auxillary_loss_free_update(model, all_topk, 1e-3, mask, process_group=pg)
        return loss

    def step():
        i = it[0] % nb
        it[0] += 1
        loss = train_step(batches[i])
        batches[i].random_(0, V, generator=g)
        return loss

    Z.INSTR.timing = True
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.5)
    Z.INSTR.events = {}
    l0 = Z.INSTR.launches
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ht0 = time.time()
    t0.record()
    for _ in range(args.steps):
        loss = step()
    t1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ht1 = time.time()
    Z.INSTR.timing = False
    clocks = sampler.stop(ht0, ht1)
    launches = Z.INSTR.launches - l0
    ms = t0.elapsed_time(t1)
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    table = kernel_table(args.steps)
    loss_v = float(loss.item())
    # end to end: the bags uploaded from pinned host memory and the loss read back every step
    e_steps = 0 if args.no_e2e else max(1, min(args.steps, args.e2e_steps))
    ids_h = torch.randint(0, V, (2, B, S, bag), generator=torch.Generator().manual_seed(6 + rank)).pin_memory()
    loss_h = torch.empty(max(e_steps, 1), dtype=torch.float32).pin_memory()
    ids_d = torch.empty(B, S, bag, dtype=torch.long, device=dev)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(e_steps):
        ids_d.copy_(ids_h[i % 2], non_blocking=True)
        lo = train_step(ids_d)
        loss_h[i:i + 1].copy_(lo.detach().reshape(1), non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e_ms = max(e0.elapsed_time(e1), 1e-9)
    if world > 1:
        tt = torch.tensor([e_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e_ms = float(tt.item())
    err = Z.device_error()
    if rank == 0:
        burst, sustained, _, src = measured_peaks()
        fpt = model_flops_per_token(cfg, S)
        value = world * B * S * args.steps / (ms * 1e-3)
        line = {"metric": METRIC, "value": value, "unit": "latent tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": f"config5 full training step at L={layers}: d=2048 H=16/4 hd=128, E=128+1 "
                                       f"shared ffn=1024 top-8 ({128 // world} experts per GPU), V=65536, 8192 "
                                       f"latent positions x micro-batch {B} per GPU, bags of 4 raw ids (bag-mean "
                                       "embedding), MCCE with 4 targets, bf16",
                           "model": "config5 MoE LM", "layers": layers, "global_batch": world * B, "seq_len": S,
                           "bag": bag, "raw_tokens_per_s": value * bag,
                           "parallelism": f"ep{world}+dp{world}" if world > 1 else "single GPU",
                           "model_gflop_per_latent_token": fpt / 1e9,
                           "mfu_of_sustained_peak": value * fpt / (world * sustained * 1e12),
                           "l2": "working set per step tens of GB, far larger than the 126 MB L2",
                           "ids": "fresh uniform token ids every step", "loss": loss_v},
                "roofline": roofline_from_table(table, clocks), "kernels": table, "cpu_baseline": None,
                "e2e": None if not e_steps else {
                    "value": world * B * S * e_steps / (e_ms * 1e-3), "unit": "latent tokens/s",
                    "h2d_bytes_per_step": ids_d.numel() * 8, "d2h_bytes_per_step": 4, "steps": e_steps,
                    "last_loss": float(loss_h[e_steps - 1])},
                "gpu_launches": launches, "clocks": clocks, "device_error": err}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------ kernel workloads
# Fixed single-kernel workloads at the configs' shapes, for timing with CUDA events and for
# capturing one kernel under a profiler (one process, one GPU):  bench.py --kernel NAME
# [--batch B].  Each runs `--warmup` passes, then `--steps` timed passes, and prints one JSON
# line of mean milliseconds per pass (forward and backward separately where both exist).

def _kernel_attention(args, g):
    """config 4 attention: B x 4096, H=12, Hkv=4, hd=128, causal, sink key; forward and backward."""
    import torch

    from zs_b200.attn import attention, attention_flops

    B, S, H, Hkv, hd = args.batch or 8, 4096, 12, 4, 128
    q = torch.randn(B, S, H, hd, device="cuda", generator=g).bfloat16().requires_grad_(True)
    k = torch.randn(B, S, Hkv, hd, device="cuda", generator=g).bfloat16().requires_grad_(True)
    v = torch.randn(B, S, Hkv, hd, device="cuda", generator=g).bfloat16().requires_grad_(True)
    ks = (torch.randn(H, hd, device="cuda", generator=g) * 0.5).requires_grad_(True)
    do = torch.randn(B, S, H, hd, device="cuda", generator=g).bfloat16()
    holder = {}

    def fwd():
        holder["o"] = attention(q, k, v, k_sink=ks)

    def bwd():
        torch.autograd.grad(holder["o"], (q, k, v, ks), do, retain_graph=True)

    fl = attention_flops(B, S, H, hd)
    return {"shape": [B, S, H, Hkv, hd]}, [("fwd", fwd, fl), ("bwd", bwd, 2.5 * fl)]


def _kernel_newton_schulz(args, g):
    """zeropower_via_newtonschulz5 on config 4's expert stacks [64, 1536, 1536] and [64, 1536, 768]."""
    import torch

    from optimizer.muon import newton_schulz_flops, zeropower_via_newtonschulz5

    a = torch.randn(64, 1536, 1536, device="cuda", generator=g).bfloat16()
    b = torch.randn(64, 1536, 768, device="cuda", generator=g).bfloat16()
    return {"shapes": [[64, 1536, 1536], [64, 1536, 768]]}, [
        ("w1_stack", lambda: zeropower_via_newtonschulz5(a, 5), newton_schulz_flops(64, 1536, 1536, 5)),
        ("w2_stack", lambda: zeropower_via_newtonschulz5(b, 5), newton_schulz_flops(64, 768, 1536, 5))]


def _kernel_xent(args, g):
    """config 3 cut cross entropy: hidden [16384, 2048], classifier [131072, 2048], 5 % ignored."""
    import torch

    from cut_cross_entropy import linear_cross_entropy

    T, D, V = args.tokens or 16384, 2048, 131072
    h = torch.randn(T, D, device="cuda", generator=g).bfloat16().requires_grad_(True)
    c = (torch.randn(V, D, device="cuda", generator=g) * 0.02).bfloat16().requires_grad_(True)
    t = torch.randint(0, V, (T,), device="cuda", generator=g)
    t[torch.rand(T, device="cuda", generator=g) < 0.05] = -100
    holder = {}

    def fwd():
        holder["l"] = linear_cross_entropy(h, c, t, ignore_index=-100)

    def bwd():
        torch.autograd.grad(holder["l"], (h, c), retain_graph=True)

    return {"shape": [T, D, V]}, [("fwd", fwd, 2.0 * T * V * D), ("bwd", bwd, 6.0 * T * V * D)]


def _kernel_muonmd(args, g):
    """md_decoupled_step on config 4's expert stacks, f32, gains "both": W1 [64, 1536, 1536]
    (square) and W2 [64, 1536, 768] (tall: Newton-Schulz runs on the transpose); for W1 also
    its element-wise passes alone (md_pre: momentum + Newton-Schulz input + gain reductions;
    md_post: the projection reduction, gain Adam and the weight write)."""
    import torch

    from optimizer.muon import _md_post, _md_pre, md_decoupled_step, zeropower_via_newtonschulz5

    hp = dict(momentum=0.95, gain_mode="both", norm_axis="frobenius", capturable=True)
    post = dict(gain_lr=1e-3, gain_betas=(0.9, 0.95), gain_eps=1e-10, rescale_mode="balanced")
    lr = torch.tensor(0.02, device="cuda")
    parts = []
    for name, shape in (("w1", (64, 1536, 1536)), ("w2", (64, 1536, 768))):
        p = torch.randn(*shape, device="cuda", generator=g) * 0.02
        grad = torch.randn(*shape, device="cuda", generator=g) * 1e-3
        state = {}

        def step(p=p, grad=grad, state=state):
            md_decoupled_step(p, grad, state, lr=lr, ns_steps=5, **hp, **post)

        parts.append((f"{name}_step", step, 0.0))
        if name == "w1":
            step()
            W, red, X = _md_pre(p, grad, state, **hp)
            U = zeropower_via_newtonschulz5(X, steps=5)

            def pre(p=p, grad=grad, state=state):
                _md_pre(p, grad, state, **hp)

            def post_(p=p, W=W, red=red, U=U, state=state):
                _md_post(p, W, red, U, state, lr=lr, norm_axis="frobenius", **post)

            parts += [("w1_md_pre", pre, 0.0), ("w1_md_post", post_, 0.0)]
    return {"shapes": [[64, 1536, 1536], [64, 1536, 768]]}, parts


def _kernel_norm_rope(args, g):
    """zRMSNorm and the fused residual add + zRMSNorm on [32768, 1536], partial RoPE on config 4's q/k."""
    import torch

    from modeling.liger_rope import PartialRopeFunction
    from modeling.zRMSNorm import AddZRMSNormFunction, ZRMSNormFunction

    x = torch.randn(32768, 1536, device="cuda", generator=g).requires_grad_(True)
    w = (torch.randn(1536, device="cuda", generator=g) * 0.1).requires_grad_(True)
    dy = torch.randn(32768, 1536, device="cuda", generator=g)
    br = torch.randn(32768, 1536, device="cuda", generator=g).bfloat16().requires_grad_(True)
    q = torch.randn(8, 4096, 12, 128, device="cuda", generator=g).bfloat16()
    k = torch.randn(8, 4096, 4, 128, device="cuda", generator=g).bfloat16()
    ang = torch.arange(4096, device="cuda", dtype=torch.float32)[:, None] * torch.logspace(0, -4, 8, device="cuda")
    cos, sin = ang.cos().expand(8, 4096, 8).contiguous(), ang.sin().expand(8, 4096, 8).contiguous()

    def norm():
        y = ZRMSNormFunction.apply(x, w, 1e-6)
        torch.autograd.grad(y, (x, w), dy)

    def add_norm():
        h, yb = AddZRMSNormFunction.apply(x, br, w, 1e-6)
        torch.autograd.grad((h, yb), (x, br, w), (dy, dy.bfloat16()))

    def rope():
        qq, kk = q.clone().requires_grad_(True), k.clone().requires_grad_(True)
        qo, ko = PartialRopeFunction.apply(qq * 1, kk * 1, cos, sin, 8)
        torch.autograd.grad((qo, ko), (qq, kk), (torch.ones_like(qo), torch.ones_like(ko)))

    return {"rows": [32768, 1536]}, [("zrmsnorm", norm, 0.0), ("add_zrmsnorm", add_norm, 0.0), ("rope", rope, 0.0)]


def _kernel_routing(args, g):
    """config 2 routing: sigmoid + biased top-8 of [16384, 64] bf16, flatten_sort_count, gate backward."""
    import torch

    from modeling.moe_gate import GateTopK
    from scattermoe.parallel_experts import flatten_sort_count

    logits = torch.randn(16384, 64, device="cuda", generator=g).bfloat16().requires_grad_(True)
    bias = torch.randn(64, device="cuda", generator=g) * 0.1

    def route():
        idx, w = GateTopK.apply(torch.sigmoid(logits), bias, 8)
        flatten_sort_count(idx, 64)
        torch.autograd.grad(w, logits, torch.ones_like(w))

    return {"shape": [16384, 64, 8]}, [("route", route, 0.0)]


KERNEL_WORKLOADS = {"attention": _kernel_attention, "newton_schulz": _kernel_newton_schulz, "xent": _kernel_xent,
                    "muonmd": _kernel_muonmd, "norm_rope": _kernel_norm_rope, "routing": _kernel_routing}


def run_kernel(args):
    import torch

    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(0)
    meta, parts = KERNEL_WORKLOADS[args.kernel](args, g)
    out = {"kernel_workload": args.kernel, **meta, "passes": args.steps}
    for name, fn, fl in parts:
        for _ in range(max(args.warmup, 1)):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            fn()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / args.steps
        out[name] = {"ms": ms, **({"tflops": fl / ms / 1e9} if fl else {})}
    print(json.dumps(out), flush=True)


def _free_port():
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=0, help="timed steps (default: 20 for config 4, 200 otherwise)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="zs", choices=["zs", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end (host buffer) loop")
    ap.add_argument("--e2e-steps", type=int, default=10, help="config 4: steps of the end-to-end loop")
    ap.add_argument("--profile-timed", action="store_true",
                    help="config 4: bracket the timed steps with cudaProfilerStart/Stop (for ncu --profile-from-start off)")
    ap.add_argument("--tokens", type=int, default=0, help="config 2/3/5: tokens per GPU")
    ap.add_argument("--config", type=int, default=4, choices=[2, 3, 4, 5],
                    help="BASELINE config (default 4, the full training step the metric is quoted on)")
    ap.add_argument("--layers", type=int, default=16, help="config 4: transformer depth")
    ap.add_argument("--micro-batch", type=int, default=8, help="config 4: sequences of 4096 per GPU")
    ap.add_argument("--mcce", action="store_true", help="config 3: the 4-target MCCE variant")
    ap.add_argument("--full-model", action="store_true",
                    help="config 5: the whole training step of the model instead of its MoE layer")
    ap.add_argument("--layers-c5", type=int, default=0,
                    help="config 5 --full-model: transformer depth (default 4 per GPU, at most 24)")
    ap.add_argument("--micro-batch-c5", type=int, default=4,
                    help="config 5 --full-model: sequences of 8192 latent positions per GPU")
    ap.add_argument("--kernel", default=None, choices=sorted(KERNEL_WORKLOADS),
                    help="time one fixed kernel workload instead of a config (for profiling)")
    ap.add_argument("--batch", type=int, default=0, help="--kernel attention: sequences of 4096 (default 8)")
    ap.add_argument("--dp-engine", default="nccl", choices=["nccl", "ce"],
                    help="config 2 with N > 1: gradient all-reduce on the copy engines (ce) or NCCL")
    args = ap.parse_args()
    if not args.steps:
        args.steps = 10 if args.kernel else (20 if args.config == 4 else (10 if args.full_model else 200))
    if args.kernel:
        run_kernel(args)
        return
    if args.impl == "reference":
        if args.config == 4:
            run_reference_config4(args)
        else:
            run_reference(args)
    elif args.config == 3:
        run_config3(args)
    elif args.config == 4:
        run_config4(args)
    elif args.config == 5:
        run_config5_model(args) if args.full_model else run_config5(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
