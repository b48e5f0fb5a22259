#!/usr/bin/env python
"""Decode throughput of the paged fused-MoE stack.

Workload (``config.workload``): the full 48-layer Qwen3-30B-A3B expert stack
(H 2048, I 768, E 128, top-8), bf16 random-init weights N(0, 0.02) in pinned
host memory, synthetic routing with per-layer Zipf(1.1) popularity and 0.6
temporal reuse, decode at batch B with a fixed cap of C slots per layer
(default B 16, C 32).  One step = one decode token for the batch through all
48 MoE layers (pager, page-in, expert compute, combine).

Arms:
  --impl wisp       (default) this package's CUDA path;
  --impl reference  the CPU restatement of the reference's path (the pager of
                    fused_moe.py:264-358 with first-fit sub-batching, and the
                    expert math of vLLM fused_experts in torch on CPU), timed
                    on the host cores on a bounded sample.

Prints one JSON line (rank 0).
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

from wisp_b200 import workloads as wl  # noqa: E402

METRIC = "decode tok/s at fixed expert-cache cap"
SHAPE = wl.QWEN3_30B


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=24)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="wisp", choices=["wisp", "reference"])
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--cap", type=int, default=32)
    ap.add_argument("--layers", type=int, default=SHAPE.layers)
    ap.add_argument("--no-resident", action="store_true", help="skip the resident-decode phase")
    ap.add_argument("--phase", default="all", choices=["all", "resident", "prefill"],
                    help="'resident' runs only the resident-decode region (profiling: the paged "
                         "forward waits on page-ins a host thread issues during the launch, which "
                         "a kernel-serialising profiler would stall)")
    ap.add_argument("--cpu-sample-s", type=float, default=15.0)
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """SM clocks and throttle reasons of the given GPUs, sampled every 0.2 s
    during the timed region by in-process NVML queries (read-only; no
    subprocess is started while the GPUs run).  Falls back to nvidia-smi when
    NVML cannot be loaded.  Under torchrun only rank 0 samples (every rank's
    GPU), so N processes do not contend for the host during the timed region."""
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, indices, enabled: bool = True):
        self.indices = [int(i) for i in (indices if isinstance(indices, (list, tuple)) else [indices])]
        self.enabled = enabled
        self.rows = []          # (sm_mhz, sm_max_mhz, [reason names])
        self._stop = threading.Event()
        self._t = None
        self._nvml = None
        self._handles = []

    def _open_nvml(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self._handles = [pynvml.nvmlDeviceGetHandleByIndex(i) for i in self.indices]
            self._nvml = pynvml
        except Exception:
            self._nvml = None

    def _sample_nvml(self):
        nv = self._nvml
        bits = (nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap)
        for h in self._handles:
            sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
            mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
            self.rows.append((float(sm), float(mx), [n for n, b in zip(self.NAMES, bits) if r & b]))

    def _sample_smi(self):
        for i in self.indices:
            out = subprocess.run(["nvidia-smi", "-i", str(i), f"--query-gpu={self.Q}",
                                  "--format=csv,noheader,nounits"], capture_output=True,
                                 text=True, timeout=5).stdout.strip()
            if not out:
                continue
            c = [x.strip() for x in out.split(",")]
            num = [float(v) if v.replace(".", "").isdigit() else None for v in c[1:3]]
            reasons = [n for k, n in enumerate(self.NAMES) if len(c) > 5 + k
                       and c[5 + k].lower().startswith("active")]
            if num[0] is not None and num[1] is not None:
                self.rows.append((num[0], num[1], reasons))

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample_nvml() if self._nvml is not None else self._sample_smi()
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        if self.enabled:
            self._open_nvml()
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        if self._t is not None:
            self._stop.set()
            self._t.join(timeout=10)

    def summary(self):
        if not self.enabled:
            return None
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(r[0] for r in self.rows),
                "sm_max_mhz": max(r[1] for r in self.rows),
                "reasons": sorted({n for r in self.rows for n in r[2]}),
                "samples": len(self.rows), "gpus": self.indices,
                "via": "nvml" if self._nvml is not None else "nvidia-smi"}


def h2d_peak_gbs(dev, nbytes=1 << 30, reps=6):
    """Pinned host -> HBM copy bandwidth (decimal GB/s), best of reps; the
    page-in link's measured peak (method of the reference's bandwidth probe)."""
    src = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    dst = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    best = 0.0
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dst.copy_(src, non_blocking=True)
        b.record()
        torch.cuda.synchronize()
        best = max(best, nbytes / (a.elapsed_time(b) * 1e-3) / 1e9)
    del src, dst
    return best


def make_masters(layers, dev):
    """Pinned bf16 host masters per layer, N(0, 0.02) drawn on the GPU from a
    per-layer seed (fast) and copied to pinned host memory."""
    E, H, I = SHAPE.experts, SHAPE.hidden, SHAPE.inter
    out = []
    for layer in range(layers):
        g = torch.Generator(device=dev).manual_seed(1000 + layer)
        h13 = torch.empty(E, 2 * I, H, dtype=torch.bfloat16, pin_memory=True)
        h2 = torch.empty(E, H, I, dtype=torch.bfloat16, pin_memory=True)
        t = torch.randn(E, 2 * I, H, device=dev, generator=g, dtype=torch.float32).mul_(0.02)
        h13.copy_(t.to(torch.bfloat16))
        del t
        t = torch.randn(E, H, I, device=dev, generator=g, dtype=torch.float32).mul_(0.02)
        h2.copy_(t.to(torch.bfloat16))
        del t
        out.append((h13, h2))
    torch.cuda.synchronize()
    return out


def routing(steps, layers, batch):
    ids, w = wl.zipf_trace(steps, layers, batch, SHAPE.experts, SHAPE.top_k, 1.1, 0.6, seed=0)
    return ids, w


def profile_traffic(name: str):
    """DRAM bytes per launch of the dominant kernel from a committed ncu summary
    (a line ``traffic_bytes_per_launch: N``), or None."""
    path = os.path.join(ROOT, "profiles", name)
    try:
        with open(path) as f:
            for line in f:
                if line.strip().startswith("traffic_bytes_per_launch:"):
                    return float(line.split(":", 1)[1].strip().split()[0])
    except OSError:
        pass
    return None


def dominant_kernel(batch: int, tc_min_pairs: int) -> str:
    """The kernel that streams the expert weights in a resident forward of
    ``batch`` tokens: the one-launch CUDA-core forward below the layer's
    tensor-core threshold, the weight-stationary tcgen05 kernel from it to 256
    pairs, the token-major GEMMs above."""
    from wisp_b200 import _lib
    pairs = batch * SHAPE.top_k
    if pairs >= _lib.PREFILL_MIN_PAIRS:
        return "gateup_gemm_kernel+down_gemm_kernel"
    return "batch_moe_kernel" if pairs >= tc_min_pairs else "forward_kernel"


def algorithmic_bytes(unique_experts: int, tokens: int, launches: int) -> int:
    """Bytes a layer forward must move (expert weights read once per group,
    activations in and out, routing ids and weights)."""
    return (unique_experts * SHAPE.expert_bytes + tokens * SHAPE.hidden * 2 * 2
            + tokens * SHAPE.top_k * (4 + 4)) if launches else 0


def run_wisp(args):
    from wisp_b200.integrations.vllm.fused_moe import WispMoEState
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    hbm_peak, peak_src = peaks()
    L, B, C = args.layers, args.batch, args.cap
    total = args.warmup + args.steps
    if args.phase == "resident":
        return resident_only(args, dev, hbm_peak, peak_src)
    if args.phase == "prefill":
        return prefill_only(args, dev, hbm_peak, peak_src)
    t0 = time.time()
    masters = make_masters(L, dev)
    states = [WispMoEState(h13, h2, C, "paged", dev, i) for i, (h13, h2) in enumerate(masters)]
    ids_np, w_np = routing(total, L, B)
    ids_d = torch.from_numpy(ids_np).to(dev)
    w_d = torch.from_numpy(w_np).to(dev)
    x_d = wl.hidden_states(B, SHAPE.hidden, seed=0).to(dev)
    out_d = torch.empty_like(x_d)
    setup_s = time.time() - t0

    def step(s, x, ids, w, out):
        for layer in range(L):
            states[layer].forward(x, w[s, layer], ids[s, layer], out=out)

    for s in range(args.warmup):
        step(s, x_d, ids_d, w_d, out_d)
    torch.cuda.synchronize()
    for st in states:
        st.synchronize()
    before = [st.stats() for st in states]
    tel0 = [st.telemetry() for st in states]
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clk:
        torch.cuda.synchronize()
        ev0.record()
        for s in range(args.warmup, total):
            step(s, x_d, ids_d, w_d, out_d)
        ev1.record()
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    for st in states:
        st.synchronize()
    tel1 = [st.telemetry() for st in states]

    def delta(key):
        return sum(b[key] - a[key] for a, b in zip(tel0, tel1))

    pagein_bytes = delta("pagein_bytes")
    launches = delta("kernel_launches")
    unique = delta("unique_experts")
    after = [st.stats() for st in states]
    misses = sum(a[1] - b[1] for a, b in zip(after, before))
    hits = sum(a[2] - b[2] for a, b in zip(after, before))
    tok_s = B * args.steps / (ms * 1e-3)

    # end to end through the public API: routing + hidden states copied in from
    # pinned host memory and the output copied back, every step
    ids_h = torch.from_numpy(ids_np).pin_memory()
    w_h = torch.from_numpy(w_np).pin_memory()
    x_h = wl.hidden_states(B, SHAPE.hidden, seed=0).pin_memory()
    out_h = torch.empty_like(x_h).pin_memory()
    ids_s = torch.empty((L, B, SHAPE.top_k), dtype=ids_d.dtype, device=dev)
    w_s = torch.empty((L, B, SHAPE.top_k), dtype=w_d.dtype, device=dev)
    e2e_steps = min(args.steps, 8)
    torch.cuda.synchronize()
    ev2, ev3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev2.record()
    for j in range(e2e_steps):
        s = args.warmup + (j % args.steps)
        ids_s.copy_(ids_h[s], non_blocking=True)
        w_s.copy_(w_h[s], non_blocking=True)
        x_d.copy_(x_h, non_blocking=True)
        for layer in range(L):
            states[layer].forward(x_d, w_s[layer], ids_s[layer], out=out_d)
        out_h.copy_(out_d, non_blocking=True)
    ev3.record()
    torch.cuda.synchronize()
    e2e_ms = ev2.elapsed_time(ev3)
    e2e = {"value": B * e2e_steps / (e2e_ms * 1e-3), "unit": "tok/s",
           "h2d_bytes_per_step": int(ids_s.numel() * ids_s.element_size()
                                     + w_s.numel() * w_s.element_size()
                                     + x_h.numel() * x_h.element_size()),
           "d2h_bytes_per_step": int(out_h.numel() * out_h.element_size()),
           "steps": e2e_steps}

    h2d = h2d_peak_gbs(dev)
    pagein_gbs = pagein_bytes / (ms * 1e-3) / 1e9
    # step roofline: the slower of the HBM bytes at the HBM peak and the page-in
    # bytes at the measured pinned-H2D peak, divided by the measured time
    hbm_bytes = algorithmic_bytes(unique, B * L * args.steps, launches)
    hbm_s = hbm_bytes / (hbm_peak * 1e9)
    link_s = pagein_bytes / (h2d * 1e9)
    step_roof = {"hbm_bytes": hbm_bytes, "pagein_bytes": pagein_bytes, "hbm_s": hbm_s,
                 "link_s": link_s, "measured_s": ms * 1e-3,
                 "bound": "h2d" if link_s >= hbm_s else "hbm",
                 "frac": max(hbm_s, link_s) / (ms * 1e-3)}
    for st in states:
        st.close()
    del states
    torch.cuda.empty_cache()
    res = {}
    if not args.no_resident:
        for rb in sorted({B, 1}, reverse=True):
            res[f"batch{rb}"] = resident_phase(args, masters, dev, hbm_peak, rb)
    del masters

    roofline = None
    if res:
        r = res[f"batch{B}"]
        roofline = {"bound": "hbm", "kernel": r["kernel"],
                    "region": f"resident decode (cap = E), batch {B}, {r['layers']} layers: whole "
                              f"forward ({r['launches_per_forward']:.0f} launches) timed with CUDA events",
                    "achieved": r["hbm_gbs"], "peak": hbm_peak, "unit": "GB/s",
                    "frac": r["frac"], "peak_src": peak_src,
                    "traffic": profile_traffic(f"{r['kernel']}_resident_decode_b{B}.md"),
                    "bytes_per_forward": r["bytes_per_forward"], "us_per_forward": r["us_per_forward"]}

    line = {
        "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded Zipf routing trace; random-init N(0,0.02) weights)",
        "config": {"workload": f"qwen3-30b-a3b {L}-layer expert stack, decode batch {B}, cap {C}",
                   "layers": L, "batch": B, "cap": C, "experts": SHAPE.experts,
                   "top_k": SHAPE.top_k, "hidden": SHAPE.hidden, "inter": SHAPE.inter,
                   "routing": "zipf1.1 reuse0.6", "l2": "inputs larger than L2 (each step reads "
                   "every layer's routed experts, >= 48 x 8 x 9.4 MB, from HBM)"},
        "gpu_launches": launches,
        "roofline": roofline,
        "step_roofline": step_roof,
        "pagein": {"gbs": pagein_gbs, "h2d_peak_gbs": h2d, "frac": pagein_gbs / h2d,
                   "misses": misses, "hits": hits, "bytes": pagein_bytes},
        "resident_decode": res,
        "e2e": e2e,
        "clocks": clk.summary(),
        "setup_s": setup_s,
    }
    return line


def resident_only(args, dev, hbm_peak, peak_src):
    """The resident-decode region alone, at the given batch (profiling runs)."""
    masters = make_masters(min(args.layers, 24), dev)
    r = resident_phase(args, masters, dev, hbm_peak, args.batch)
    return {"metric": "resident decode tok/s (cap = E)", "value": r["tok_s_per_layer_stack"],
            "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": r["us_per_forward"] * r["layers"] / 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"qwen3-30b-a3b {r['layers']}-layer expert stack, resident decode "
                                   f"batch {args.batch}"},
            "gpu_launches": r["launches"],
            "roofline": {"bound": "hbm", "kernel": r["kernel"], "achieved": r["hbm_gbs"],
                         "peak": hbm_peak, "unit": "GB/s", "frac": r["frac"], "peak_src": peak_src,
                         "bytes_per_forward": r["bytes_per_forward"], "us_per_forward": r["us_per_forward"]},
            "resident_decode": r}


def prefill_only(args, dev, hbm_peak, peak_src):
    """Config 3's prefill chunk on resident layers (cap = E): T = 2048 tokens,
    uniform top-8 of 128 (every expert touched), one forward per layer on the
    tcgen05 tensor-core path; reports tensor TFLOP/s (2 T k 3 H I per layer)
    and the expert-weight HBM GB/s against the measured peaks."""
    from wisp_b200.integrations.vllm.fused_moe import WispMoEState
    tflops_peak = 1680.6
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            tflops_peak = float(json.load(f)["bf16_tflops"])
    except Exception:
        pass
    L = min(args.layers, 8)
    T = 2048
    masters = make_masters(L, dev)
    states = []
    for i in range(L):
        st = WispMoEState(masters[i][0], masters[i][1], SHAPE.experts, "resident", dev, i)
        st.prime_identity()
        states.append(st)
    x = wl.hidden_states(T, SHAPE.hidden, seed=3).to(dev)
    out = torch.empty_like(x)
    routes = []
    for s in range(args.warmup + args.steps):
        ids, w = wl.uniform_topk(T, SHAPE.experts, SHAPE.top_k, seed=100 + s)
        routes.append((torch.from_numpy(ids).to(dev), torch.from_numpy(w).to(dev)))
    for s in range(args.warmup):
        for layer in range(L):
            states[layer].forward(x, routes[s][1], routes[s][0], out=out)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for s in range(args.warmup, args.warmup + args.steps):
        for layer in range(L):
            states[layer].forward(x, routes[s][1], routes[s][0], out=out)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    n = args.steps * L
    us = ms * 1e3 / n
    flop = 2.0 * T * SHAPE.top_k * 3 * SHAPE.hidden * SHAPE.inter
    wbytes = SHAPE.experts * SHAPE.expert_bytes
    for st in states:
        st.close()
    tf = flop / (us * 1e-6) / 1e12
    gbs = wbytes / (us * 1e-6) / 1e9
    roof_us = max(flop / (tflops_peak * 1e12), wbytes / (hbm_peak * 1e9)) * 1e6
    return {"metric": "prefill tok/s (resident, 2048-token chunk)", "value": T * args.steps / (ms * 1e-3 / L) / L,
            "unit": "tok/s per layer stack of %d" % L, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "dtype": "bf16", "data": "synthetic (uniform top-8 routing)",
            "config": {"workload": f"qwen3-30b-a3b prefill, {L} resident layers, T {T}, uniform top-8"},
            "prefill": {"us_per_layer": us, "tflops": tf, "tflops_peak": tflops_peak,
                        "tensor_frac": tf / tflops_peak, "weight_gbs": gbs, "hbm_peak_gbs": hbm_peak,
                        "hbm_frac": gbs / hbm_peak, "roofline_us": roof_us, "roofline_frac": roof_us / us,
                        "peak_src": peak_src}}


def resident_phase(args, masters, dev, hbm_peak, batch):
    """Resident-expert decode (cap = E, prime_identity), HBM-bound: below the
    tensor-core threshold one forward-kernel launch per layer, from it the
    pager, gather, weight-stationary tcgen05 kernel and combine, queued with
    no host round trip.  A forward's duration is the CUDA-event time of
    back-to-back forwards divided by their number (the host issues faster
    than the kernels run)."""
    from wisp_b200.integrations.vllm.fused_moe import WispMoEState
    L = min(args.layers, 24)
    B = batch
    states = []
    for i in range(L):
        st = WispMoEState(masters[i][0], masters[i][1], SHAPE.experts, "resident", dev, i)
        st.prime_identity()
        states.append(st)
    ids_np, w_np = routing(args.warmup + args.steps, L, B)
    ids_d = torch.from_numpy(ids_np).to(dev)
    w_d = torch.from_numpy(w_np).to(dev)
    x = wl.hidden_states(B, SHAPE.hidden, seed=1).to(dev)
    out = torch.empty_like(x)
    for s in range(args.warmup):
        for layer in range(L):
            states[layer].forward(x, w_d[s, layer], ids_d[s, layer], out=out)
    torch.cuda.synchronize()
    tel0 = [st.telemetry() for st in states]
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for s in range(args.warmup, args.warmup + args.steps):
        for layer in range(L):
            states[layer].forward(x, w_d[s, layer], ids_d[s, layer], out=out)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    tel1 = [st.telemetry() for st in states]
    unique = sum(t1["unique_experts"] - t0["unique_experts"] for t0, t1 in zip(tel0, tel1))
    launches = sum(t1["kernel_launches"] - t0["kernel_launches"] for t0, t1 in zip(tel0, tel1))
    nbytes = algorithmic_bytes(unique, B * L * args.steps, launches)
    gbs = nbytes / (ms * 1e-3) / 1e9
    tc_min_pairs = states[0].tc_min_pairs
    for st in states:
        st.close()
    torch.cuda.empty_cache()
    forwards = args.steps * L
    return {"layers": L, "batch": B, "kernel": dominant_kernel(B, tc_min_pairs),
            "tc_min_pairs": tc_min_pairs,
            "tok_s_per_layer_stack": B * args.steps / (ms * 1e-3),
            "us_per_forward": ms * 1e3 / forwards, "launches": launches,
            "launches_per_forward": launches / forwards,
            "bytes_per_forward": nbytes / forwards, "unique_experts_per_forward": unique / forwards,
            "hbm_gbs": gbs, "hbm_peak_gbs": hbm_peak, "frac": gbs / hbm_peak}


def make_shard_masters(layers, dev, rank, world):
    """Pinned bf16 host masters of this rank's experts per layer: the same
    N(0, 0.02) weights as make_masters (same per-layer seeds), sliced to the
    shard, so the whole model is identical at every rank count."""
    E = SHAPE.experts
    lo, hi = rank * E // world, (rank + 1) * E // world
    out = []
    for layer in range(layers):
        g = torch.Generator(device=dev).manual_seed(1000 + layer)
        t = torch.randn(E, 2 * SHAPE.inter, SHAPE.hidden, device=dev, generator=g, dtype=torch.float32)
        h13 = t[lo:hi].mul_(0.02).to(torch.bfloat16).cpu().pin_memory()
        del t
        t = torch.randn(E, SHAPE.hidden, SHAPE.inter, device=dev, generator=g, dtype=torch.float32)
        h2 = t[lo:hi].mul_(0.02).to(torch.bfloat16).cpu().pin_memory()
        del t
        out.append((h13, h2))
    torch.cuda.synchronize()
    return out


def run_wisp_ep(args):
    """Expert-parallel stack over the torchrun ranks (one GPU each): rank r owns
    experts [r E/P, (r+1) E/P) of every layer in its own pinned memory and
    pages them into cap = min(--cap, E/P) slots per layer; each rank decodes its
    own batch of --batch tokens (weak scaling: global batch = P x batch),
    tokens exchanged by NCCL all-to-all.  Times are CUDA events, max over ranks."""
    import datetime

    import torch.distributed as dist
    from wisp_b200.expert_parallel import EPMoELayer
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    L, B = args.layers, args.batch
    E = SHAPE.experts
    per = E // world
    C = min(args.cap, per)
    total = args.warmup + args.steps
    t0 = time.time()
    masters = make_shard_masters(L, dev, rank, world)
    # a cap that holds the whole shard makes it resident (primed once; the
    # one-launch forward), otherwise the shard pages
    mode = "resident" if C == per else "paged"
    layers = [EPMoELayer(h13, h2, E, C, mode, dev, i) for i, (h13, h2) in enumerate(masters)]
    ids_all, w_all = routing(total, L, B * world)
    ids_d = torch.from_numpy(np.ascontiguousarray(ids_all[:, :, rank * B:(rank + 1) * B])).to(dev)
    w_d = torch.from_numpy(np.ascontiguousarray(w_all[:, :, rank * B:(rank + 1) * B])).to(dev)
    x_d = wl.hidden_states(B * world, SHAPE.hidden, seed=0)[rank * B:(rank + 1) * B].contiguous().to(dev)
    out_d = torch.empty_like(x_d)
    setup_s = time.time() - t0

    def step(s, x, w, ids, out):
        for layer in range(L):
            layers[layer].forward(x, w[s, layer], ids[s, layer], out=out)

    for s in range(args.warmup):
        step(s, x_d, w_d, ids_d, out_d)
    torch.cuda.synchronize()
    for lay in layers:
        lay.local.synchronize()
    tel0 = [lay.local.telemetry() for lay in layers]
    dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(list(range(world)), enabled=rank == 0)
    with clk:
        torch.cuda.synchronize()
        ev0.record()
        for s in range(args.warmup, total):
            step(s, x_d, w_d, ids_d, out_d)
        ev1.record()
        torch.cuda.synchronize()
    dist.barrier()
    for lay in layers:
        lay.local.synchronize()
    tel1 = [lay.local.telemetry() for lay in layers]

    def delta(key):
        return sum(b[key] - a[key] for a, b in zip(tel0, tel1))

    # per forward: route + pack + combine kernels of the exchange, plus the shard's own launches
    stats = torch.tensor([ev0.elapsed_time(ev1), float(delta("pagein_bytes")),
                          float(delta("kernel_launches") + 3 * L * args.steps),
                          float(delta("unique_experts"))], dtype=torch.float64, device=dev)
    mx = stats.clone()
    dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    dist.all_reduce(stats, op=dist.ReduceOp.SUM)
    ms = float(mx[0])

    # end to end: this rank's routing + hidden states in from pinned host, output back, every step
    ids_h = torch.from_numpy(np.ascontiguousarray(ids_all[:, :, rank * B:(rank + 1) * B])).pin_memory()
    w_h = torch.from_numpy(np.ascontiguousarray(w_all[:, :, rank * B:(rank + 1) * B])).pin_memory()
    x_h = x_d.cpu().pin_memory()
    out_h = torch.empty_like(x_h).pin_memory()
    ids_s = torch.empty((L, B, SHAPE.top_k), dtype=ids_d.dtype, device=dev)
    w_s = torch.empty((L, B, SHAPE.top_k), dtype=w_d.dtype, device=dev)
    e2e_steps = min(args.steps, 8)
    torch.cuda.synchronize()
    dist.barrier()
    ev2, ev3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev2.record()
    for j in range(e2e_steps):
        s = args.warmup + (j % args.steps)
        ids_s.copy_(ids_h[s], non_blocking=True)
        w_s.copy_(w_h[s], non_blocking=True)
        x_d.copy_(x_h, non_blocking=True)
        for layer in range(L):
            layers[layer].forward(x_d, w_s[layer], ids_s[layer], out=out_d)
        out_h.copy_(out_d, non_blocking=True)
    ev3.record()
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([ev2.elapsed_time(ev3)], dtype=torch.float64, device=dev)
    dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    for lay in layers:
        lay.close()
    dist.barrier()
    dist.destroy_process_group()
    h2d = h2d_peak_gbs(dev) if rank == 0 else 0.0
    pagein_gbs = float(stats[1]) / (ms * 1e-3) / 1e9
    return {
        "metric": METRIC, "value": world * B * args.steps / (ms * 1e-3), "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded Zipf routing trace; random-init N(0,0.02) weights)",
        "config": {"workload": f"qwen3-30b-a3b {L}-layer expert stack, expert-parallel over {world} GPUs, "
                               f"decode batch {B} per GPU, cap {C} per GPU",
                   "layers": L, "batch_per_gpu": B, "global_batch": B * world, "cap_per_gpu": C,
                   "experts_per_gpu": per, "shard_mode": mode, "parallelism": f"ep{world}",
                   "routing": "zipf1.1 reuse0.6",
                   "l2": "inputs larger than L2 (each step reads every layer's routed experts from HBM)"},
        "gpu_launches": int(stats[2]),
        "roofline": None,
        "pagein": {"gbs_all_ranks": pagein_gbs, "h2d_peak_gbs_per_gpu": h2d,
                   "frac_of_per_gpu_peak_x_gpus": pagein_gbs / (h2d * world) if h2d else None,
                   "bytes": float(stats[1])},
        "e2e": {"value": world * B * e2e_steps / (float(e2e_ms[0]) * 1e-3), "unit": "tok/s",
                "h2d_bytes_per_step": int(ids_s.numel() * ids_s.element_size() + w_s.numel()
                                          * w_s.element_size() + x_h.numel() * x_h.element_size()) * world,
                "d2h_bytes_per_step": int(out_h.numel() * out_h.element_size()) * world,
                "steps": e2e_steps},
        "clocks": clk.summary(),
        "setup_s": setup_s,
    }


def run_reference(args):
    """CPU restatement of the reference path on the host cores (bounded sample)."""
    from oracle.moe import moe_reference  # noqa: F401
    from oracle.pager import PagerOracle, first_fit_groups
    n = len(os.sched_getaffinity(0))
    torch.set_num_threads(n)
    L, B, C = args.layers, args.batch, args.cap
    E, H, I = SHAPE.experts, SHAPE.hidden, SHAPE.inter
    sample_layers = 2
    g = torch.Generator().manual_seed(0)
    masters = [((torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16),
                (torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16))
               for _ in range(sample_layers)]
    scratch = [(torch.empty(C, 2 * I, H, dtype=torch.bfloat16), torch.empty(C, H, I, dtype=torch.bfloat16))
               for _ in range(sample_layers)]
    pagers = [PagerOracle(E, C) for _ in range(sample_layers)]
    # a trace long enough for the time-bounded sample (config 2 decodes 512 tokens)
    n_trace = args.warmup + max(args.steps, 512)
    ids_np, w_np = routing(n_trace, sample_layers, B)
    x = wl.hidden_states(B, H, seed=0).float()

    def layer_fwd(li, s):
        ids = ids_np[s, li]
        w = torch.from_numpy(w_np[s, li])
        p = pagers[li]
        p.stats_forward += 1
        out = torch.zeros(B, H)
        for t0, t1 in first_fit_groups(ids, C):
            rec = p.ensure_resident(ids[t0:t1])
            for e, slot in rec.placed:
                scratch[li][0][slot].copy_(masters[li][0][e])
                scratch[li][1][slot].copy_(masters[li][1][e])
            for t in range(t0, t1):
                acc = torch.zeros(H)
                for k in range(ids.shape[1]):
                    slot = p.expert_to_slot[int(ids[t, k])]
                    h = (scratch[li][0][slot].float() @ x[t]).to(torch.bfloat16).float()
                    a = (torch.nn.functional.silu(h[:I]) * h[I:]).to(torch.bfloat16).float()
                    y = ((scratch[li][1][slot].float() @ a) * w[t, k]).to(torch.bfloat16).float()
                    acc += y
                out[t] = acc
        return out

    for s in range(min(args.warmup, 2)):
        for li in range(sample_layers):
            layer_fwd(li, s)
    t0 = time.perf_counter()
    done = 0
    s = args.warmup
    while True:
        for li in range(sample_layers):
            layer_fwd(li, s)
        done += 1
        s += 1
        if time.perf_counter() - t0 > args.cpu_sample_s or s >= n_trace:
            break
    dt = time.perf_counter() - t0
    per_layer = dt / (done * sample_layers)
    tok_s = B / (per_layer * L)
    return {"value": tok_s, "unit": "tok/s", "cores": n, "kind": "port",
            "sample": f"{done} decode steps x {sample_layers} layers (of {L}) at batch {B}, cap {C}; "
                      f"tok/s extrapolated to {L} layers ({dt:.1f} s of CPU work)"}


def main():
    args = parse()
    rank = int(os.environ.get("RANK", 0))
    if args.impl == "reference":
        if rank != 0:
            return
        cpu = run_reference(args)
        line = {"metric": METRIC, "value": cpu["value"], "unit": "tok/s", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "impl": "reference",
                "data": "synthetic", "config": {"workload": f"qwen3-30b-a3b {args.layers}-layer "
                                                f"expert stack, decode batch {args.batch}, cap {args.cap}"},
                "cpu_baseline": cpu,
                "e2e": {"value": cpu["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return
    world = int(os.environ.get("WORLD_SIZE", 1))
    if world > 1:
        line = run_wisp_ep(args)
        if rank == 0:
            print(json.dumps(line))
        return
    line = run_wisp(args)
    if rank == 0:
        if args.gpus == 1 and args.cpu_sample_s > 0 and args.phase == "all":
            line["cpu_baseline"] = run_reference(args)
        print(json.dumps(line))


if __name__ == "__main__":
    main()
