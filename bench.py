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

# Benchmark workloads: model shape, decode batch per GPU,
# expert-cache cap, layers, routing (Zipf exponent, temporal reuse).
WORKLOADS = {
    # one GPU; under expert parallelism `cap` stays the layer's
    # total cache, split evenly over the GPUs (every shard pages at every N)
    "qwen3-30b": dict(shape=wl.QWEN3_30B, batch=16, cap=32, layers=48, zipf=1.1, reuse=0.6, cap_split=True),
    # the expert-parallel configuration, `cap` slots per GPU
    "qwen3-235b": dict(shape=wl.QWEN3_235B, batch=64, cap=16, layers=16, zipf=1.1, reuse=0.5, cap_split=False),
}
SHAPE = wl.QWEN3_30B
ZIPF, REUSE = 1.1, 0.6


def parse():
    global SHAPE, ZIPF, REUSE
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=24)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="wisp", choices=["wisp", "reference"])
    ap.add_argument("--workload", default="qwen3-30b", choices=sorted(WORKLOADS))
    ap.add_argument("--batch", type=int, default=None, help="decode tokens per GPU (default: the workload's)")
    ap.add_argument("--cap", type=int, default=None, help="expert-cache slots per layer (default: the workload's)")
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--no-resident", action="store_true", help="skip the resident-decode phase")
    ap.add_argument("--no-sweep", dest="sweep", action="store_false",
                    help="skip the other BASELINE configurations (extra keys of the line)")
    ap.add_argument("--phase", default="all", choices=["all", "resident", "prefill"],
                    help="'resident' runs only the resident-decode region (profiling: the paged "
                         "forward waits on page-ins a host thread issues during the launch, which "
                         "a kernel-serialising profiler would stall)")
    ap.add_argument("--cpu-sample-s", type=float, default=15.0)
    args = ap.parse_args()
    w = WORKLOADS[args.workload]
    SHAPE, ZIPF, REUSE = w["shape"], w["zipf"], w["reuse"]
    for k in ("batch", "cap", "layers"):
        if getattr(args, k) is None:
            setattr(args, k, w[k])
    args.cap_split = w["cap_split"]
    return args


def release_pinned() -> None:
    """Hand torch's cached pinned host blocks back to the OS (expert masters
    of a finished phase), so the next phase's masters fit the host."""
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    if hasattr(torch._C, "_host_emptyCache"):
        torch._C._host_emptyCache()


def use_workload(name: str) -> None:
    global SHAPE, ZIPF, REUSE
    w = WORKLOADS[name]
    SHAPE, ZIPF, REUSE = w["shape"], w["zipf"], w["reuse"]


def workload_args(args, name: str, **over):
    """A copy of ``args`` for another workload (its batch, cap and layers),
    made current."""
    a = argparse.Namespace(**vars(args))
    w = WORKLOADS[name]
    a.workload = name
    a.batch, a.cap, a.layers, a.cap_split = w["batch"], w["cap"], w["layers"], w["cap_split"]
    for k, v in over.items():
        setattr(a, k, v)
    use_workload(name)
    return a


def host_memory_check(nbytes: int, world: int) -> None:
    """Refuse a run whose pinned expert masters (all ranks of this host)
    would take more than half of the host's available memory."""
    try:
        with open("/proc/meminfo") as f:
            avail = next(int(l.split()[1]) * 1024 for l in f if l.startswith("MemAvailable:"))
    except Exception:
        return
    if nbytes * world > avail // 2:
        raise SystemExit(f"bench: {nbytes * world / 1e9:.1f} GB of pinned expert masters would exceed half "
                         f"of the host's {avail / 1e9:.1f} GB available; pass fewer --layers")


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

    def __init__(self, indices, enabled: bool = True, interval: float = 0.2):
        self.indices = [int(i) for i in (indices if isinstance(indices, (list, tuple)) else [indices])]
        self.enabled = enabled
        self.interval = interval
        self._max = {}
        self.rows = []          # (sm_mhz, sm_max_mhz, [reason names])
        self._stop = threading.Event()
        self._t = None
        self._nvml = None
        self._handles = []

    def _open_nvml(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            # NVML numbers the machine's GPUs; map the CUDA device indices through
            # CUDA_VISIBLE_DEVICES (indices or UUIDs) when it is set
            vis = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
            hs = []
            for i in self.indices:
                v = vis[i] if i < len(vis) else str(i)
                hs.append(pynvml.nvmlDeviceGetHandleByIndex(int(v)) if v.isdigit()
                          else pynvml.nvmlDeviceGetHandleByUUID(v))
            self._handles = hs
            self._nvml = pynvml
        except Exception:
            self._nvml = None

    def _sample_nvml(self):
        nv = self._nvml
        bits = (nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap)
        for i, h in enumerate(self._handles):
            sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
            if i not in self._max:
                self._max[i] = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            mx = self._max[i]
            r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
            self.rows.append((float(sm), float(mx), [n for n, b in zip(self.NAMES, bits) if r & b]))

    def _sample_smi(self):
        vis = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
        for i in self.indices:
            out = subprocess.run(["nvidia-smi", "-i", vis[i] if i < len(vis) else str(i), f"--query-gpu={self.Q}",
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
            self._stop.wait(self.interval)

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
        """Median SM clock, max clock and throttle reasons seen."""
        if not self.enabled:
            return None
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(r[0] for r in self.rows),
                "sm_max_mhz": max(r[1] for r in self.rows),
                "reasons": sorted({n for r in self.rows for n in r[2]}),
                "samples": len(self.rows), "gpus": self.indices,
                "via": "nvml" if self._nvml is not None else "nvidia-smi"}


class SmiSampler(ClockSampler):
    """Clocks of several GPUs from one separate ``nvidia-smi -lms`` process
    (the expert-parallel runs: queries from inside the ranks' processes slowed
    the ranks' waits on one another), started before the timed region and
    stopped after it."""

    def __init__(self, indices, enabled: bool = True, interval_ms: int = 1000):
        super().__init__(indices, enabled)
        self.interval_ms = interval_ms
        self._p = None
        self._path = None

    def __enter__(self):
        if self.enabled:
            import tempfile
            fd, self._path = tempfile.mkstemp(prefix="wisp_clocks_", suffix=".csv")
            os.close(fd)
            self._f = open(self._path, "w")
            try:
                # nvidia-smi numbers the machine's GPUs; map the ranks' device
                # indices through CUDA_VISIBLE_DEVICES when it is set
                vis = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
                ids = [vis[i] if i < len(vis) else str(i) for i in self.indices]
                self._p = subprocess.Popen(
                    ["nvidia-smi", "-i", ",".join(ids), f"--query-gpu={self.Q}",
                     "--format=csv,noheader,nounits", "-lms", str(self.interval_ms)],
                    stdout=self._f, stderr=subprocess.DEVNULL)
            except OSError:
                self._p = None
        return self

    def __exit__(self, *a):
        if self._p is not None:
            self._p.terminate()
            try:
                self._p.wait(timeout=10)
            except subprocess.TimeoutExpired:
                self._p.kill()
        if self._path:
            self._f.close()
            with open(self._path) as f:
                for line in f:
                    c = [x.strip() for x in line.split(",")]
                    if len(c) < 9:
                        continue
                    try:
                        sm, mx = float(c[1]), float(c[2])
                    except ValueError:
                        continue
                    reasons = [n for k, n in enumerate(self.NAMES) if c[5 + k].lower().startswith("active")]
                    self.rows.append((sm, mx, reasons))
            os.unlink(self._path)

    def summary(self):
        r = super().summary()
        if r is not None and self.rows:
            r["via"] = f"nvidia-smi -lms {self.interval_ms} (one process, rank 0)"
        return r


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


def make_masters(layers, dev, lo=0, hi=None, shape=None):
    """Pinned bf16 host masters of experts [lo, hi) per layer, N(0, 0.02)
    drawn on the GPU from a per-layer seed over all E experts (so a shard is
    the same slice of the same model at every rank count) and copied to
    pinned host memory."""
    shape = shape or SHAPE
    E, H, I = shape.experts, shape.hidden, shape.inter
    hi = E if hi is None else hi
    out = []
    for layer in range(layers):
        g = torch.Generator(device=dev).manual_seed(1000 + layer)
        h13 = torch.empty(hi - lo, 2 * I, H, dtype=torch.bfloat16, pin_memory=True)
        h2 = torch.empty(hi - lo, H, I, dtype=torch.bfloat16, pin_memory=True)
        for e0 in range(lo, hi, 8):   # a few experts at a time: bounded device memory for large experts
            e1 = min(hi, e0 + 8)
            g.manual_seed(1000 + layer * 4099 + e0)
            t = torch.randn(e1 - e0, 2 * I, H, device=dev, generator=g, dtype=torch.float32)
            h13[e0 - lo:e1 - lo].copy_(t.mul_(0.02).to(torch.bfloat16))
            t = torch.randn(e1 - e0, H, I, device=dev, generator=g, dtype=torch.float32)
            h2[e0 - lo:e1 - lo].copy_(t.mul_(0.02).to(torch.bfloat16))
            del t
        out.append((h13, h2))
    # one host-to-device read of every master before anything is timed: the
    # first page-in of a host page ran slower than later ones (expert-parallel
    # runs with 3 warm-up steps timed at half their end-to-end rate, with 12 at
    # the same rate), so the warm-up steps should not have to cover all of them
    n = max(1, min(8, hi - lo))
    b13 = torch.empty(n, 2 * I, H, dtype=torch.bfloat16, device=dev)
    b2 = torch.empty(n, H, I, dtype=torch.bfloat16, device=dev)
    for h13, h2 in out:
        for e0 in range(0, hi - lo, n):
            e1 = min(hi - lo, e0 + n)
            b13[:e1 - e0].copy_(h13[e0:e1], non_blocking=True)
            b2[:e1 - e0].copy_(h2[e0:e1], non_blocking=True)
    torch.cuda.synchronize()
    del b13, b2
    return out


def routing(steps, layers, batch):
    ids, w = wl.zipf_trace(steps, layers, batch, SHAPE.experts, SHAPE.top_k, ZIPF, REUSE, seed=0)
    return ids, w


def workload_name(args, world: int = 1) -> str:
    s = f"{SHAPE.name} {args.layers}-layer expert stack, decode batch {args.batch}"
    if world == 1:
        return s + f", cap {args.cap}"
    cap = args.cap // world if args.cap_split else args.cap
    return s + (f" per GPU, expert-parallel over {world} GPUs, cap {args.cap} per layer in total "
                f"({cap} per GPU)" if args.cap_split else
                f" per GPU, expert-parallel over {world} GPUs, cap {cap} per GPU")


def profile_traffic(name: str, units: float | None = None):
    """DRAM bytes per launch of the dominant kernel from a committed ncu summary
    (a line ``traffic_bytes_per_launch: N``), or None.  When the summary also
    names the routed experts of the captured launch (``experts_per_captured_launch:
    n``) and ``units`` gives the bench's experts per launch, the traffic is scaled
    by that ratio (weight traffic grows in proportion to the routed experts)."""
    path = os.path.join(ROOT, "profiles", name)
    vals = {}
    try:
        with open(path) as f:
            for line in f:
                for key in ("traffic_bytes_per_launch", "experts_per_captured_launch"):
                    if line.strip().startswith(key + ":"):
                        vals[key] = float(line.split(":", 1)[1].strip().split()[0])
    except OSError:
        pass
    t = vals.get("traffic_bytes_per_launch")
    if t is not None and units and vals.get("experts_per_captured_launch"):
        t *= units / vals["experts_per_captured_launch"]
    return t


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


def algorithmic_bytes(unique_experts: int, tokens: int, launches: int, shape=None) -> int:
    """Bytes a layer forward must move (expert weights read once per group,
    activations in and out, routing ids and weights)."""
    shape = shape or SHAPE
    return (unique_experts * shape.expert_bytes + tokens * shape.hidden * 2 * 2
            + tokens * shape.top_k * (4 + 4)) if launches else 0


def paged_point(masters, dev, shape, B, C, routes, x, warmup, steps, hbm_peak, h2d, layers=None,
                prefetch=None):
    """Decode (or prefill) of a paged stack at cap C: ``routes[s][layer] =
    (ids, w)`` on the device, ``x`` [B, H]; warm-up steps untimed, then
    ``steps`` timed with CUDA events.  Returns the point's figures: tok/s
    of the stack of ``layers`` layers (default: as many as masters),
    page-in GB/s against the measured H2D peak and the step roofline (the
    slower of the HBM bytes at the HBM peak and the page-in bytes at the H2D
    peak, over the measured time).

    ``prefetch``: a co-occurrence table (the reference's cross-layer
    prefetch, fused_moe.py:1170-1233): after each layer's forward the
    experts it routed to are recorded for the step, max(8, C // 2) experts
    are predicted for the next layer (normalised scores, decay 0.5) and
    paged into it speculatively on its copy stream, and each finished step
    is learned online; the host work is inside the timed region, as in the
    reference."""
    from wisp_b200.integrations.vllm.fused_moe import WispMoEState
    L = len(masters)
    states = [WispMoEState(h13, h2, C, "paged", dev, i) for i, (h13, h2) in enumerate(masters)]
    out = torch.empty_like(x)
    seen = None
    if prefetch is not None:
        from wisp_b200.integrations.vllm.cooccur import predict_layer
        seen = [[sorted(set(routes[s][li][0].reshape(-1).tolist())) for li in range(L)]
                for s in range(warmup + steps)]

    def step(s):
        obs = {}
        for li in range(L):
            states[li].forward(x, routes[s][li][1], routes[s][li][0], out=out)
            if prefetch is None:
                continue
            obs[li] = seen[s][li]
            if li + 1 < L:
                pred = predict_layer(prefetch, obs, li + 1, k=max(8, C // 2), normalize=True, decay=0.5)
                if pred:
                    states[li + 1].prefetch_async(set(pred))
        if prefetch is not None:
            prefetch.observe_step(obs)

    for s in range(warmup):
        step(s)
    torch.cuda.synchronize()
    tel0 = [st.telemetry() for st in states]
    st0 = [st.stats() for st in states]
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for s in range(warmup, warmup + steps):
        step(s)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    for st in states:
        st.synchronize()
    tel1 = [st.telemetry() for st in states]
    st1 = [st.stats() for st in states]
    for st in states:
        st.close()
    d = {k: sum(t1[k] - t0[k] for t0, t1 in zip(tel0, tel1)) for k in tel0[0]}
    T = x.shape[0]
    pb = d["pagein_bytes"]
    hb = algorithmic_bytes(d["unique_experts"], T * L * steps, d["kernel_launches"], shape)
    sec = ms * 1e-3
    stack = layers or L
    return {"tok_s": T * steps / sec * L / stack, "ms_per_layer_step": ms / (steps * L),
            "pagein_gbs": pb / sec / 1e9, "pagein_frac_of_h2d_peak": pb / sec / 1e9 / h2d,
            "step_roofline_frac": max(hb / (hbm_peak * 1e9), pb / (h2d * 1e9)) / sec,
            "misses": sum(x1[1] - x0[1] for x0, x1 in zip(st0, st1)),
            "hits": sum(x1[2] - x0[2] for x0, x1 in zip(st0, st1)),
            "launches": d["kernel_launches"], "layers_timed": L, "stack_layers": stack, "steps": steps}


def one_gpu_235b(args, dev, hbm_peak, h2d):
    """configs[4]'s layer shape and routing on one GPU: all 128 experts of
    each layer paged at 16 slots, decode batch 64, the workload's layers."""
    a = workload_args(args, "qwen3-235b")
    s = SHAPE
    host_memory_check(a.layers * s.experts * s.expert_bytes, 1)
    mm = make_masters(a.layers, dev, shape=s)
    steps, warm = 3, 2
    tids, tw = wl.zipf_trace(warm + steps, a.layers, a.batch, s.experts, s.top_k, ZIPF, REUSE, seed=0)
    routes = [[(torch.from_numpy(tids[t, li]).to(dev), torch.from_numpy(tw[t, li]).to(dev))
               for li in range(a.layers)] for t in range(warm + steps)]
    x = wl.hidden_states(a.batch, s.hidden, seed=0).to(dev)
    r = paged_point(mm, dev, s, a.batch, a.cap, routes, x, warm, steps, hbm_peak, h2d)
    r["workload"] = workload_name(a, 1)
    del mm
    release_pinned()
    return r


def sweep_phase(masters, dev, hbm_peak, h2d):
    """Every BASELINE configuration besides the headline, one line each:
    configs[0] (one Qwen3-30B-A3B layer, 256 decode tokens at batch 1, cap 8,
    routed on the GPU from Zipf-biased logits), configs[1] at batch 1/4/16 x
    cap 8/16/24/32 (the 48-layer stack), configs[2] (a paged prefill chunk
    at cap 32, uniform top-8: every group pages) and configs[3] (Mixtral-8x7B
    decode at batch 1/8, cap 2/4).  Stacks longer than the layers timed
    report tok/s scaled by layer count (each layer pages its own cache)."""
    from wisp_b200.integrations.vllm.fused_moe import select_experts
    q = wl.QWEN3_30B
    out = {}
    # configs[0]
    logits = wl.router_logits(256, q.experts, seed=0).to(dev)
    w, ids = select_experts(logits, q.top_k)
    x256 = wl.hidden_states(256, q.hidden, seed=0).to(dev)
    from wisp_b200.integrations.vllm.fused_moe import WispMoEState
    st = WispMoEState(masters[0][0], masters[0][1], 8, "paged", dev, 0)
    o = torch.empty((1, q.hidden), dtype=torch.bfloat16, device=dev)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tel0 = st.telemetry()
    a.record()
    for t in range(256):
        st.forward(x256[t:t + 1], w[t:t + 1], ids[t:t + 1], out=o)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    tel1 = st.telemetry()
    f, miss, hits, ev = st.stats()
    st.close()
    pb = tel1["pagein_bytes"] - tel0["pagein_bytes"]
    out["cfg0_layer_b1_cap8"] = {"tok_s_one_layer": 256 / (ms * 1e-3), "us_per_token": ms * 1e3 / 256,
                                 "pagein_gbs": pb / (ms * 1e-3) / 1e9,
                                 "pagein_frac_of_h2d_peak": pb / (ms * 1e-3) / 1e9 / h2d,
                                 "misses": miss, "hits": hits, "evictions": ev, "forwards": f}
    # configs[1] sweep
    L = len(masters)
    for B in (1, 4, 16):
        steps, warm = 3, 2
        tids, tw = wl.zipf_trace(warm + steps, L, B, q.experts, q.top_k, 1.1, 0.6, seed=11 + B)
        routes = [[(torch.from_numpy(tids[s, li]).to(dev), torch.from_numpy(tw[s, li]).to(dev))
                   for li in range(L)] for s in range(warm + steps)]
        x = wl.hidden_states(B, q.hidden, seed=B).to(dev)
        for C in (8, 16, 24, 32):
            out[f"cfg1_b{B}_cap{C}"] = paged_point(masters, dev, q, B, C, routes, x, warm, steps, hbm_peak, h2d)
        if B == 16:
            # the reference's cross-layer prefetch on the B200 link (off by default
            # there too): a table learned online, warmed on 7 other steps of the
            # same routing process (same per-layer popularity, other draws)
            from wisp_b200.integrations.vllm.cooccur import NativeCooccurTable
            table = NativeCooccurTable()  # the plug-in's table
            wids, _ = wl.zipf_trace(12, L, B, q.experts, q.top_k, 1.1, 0.6, seed=11 + B)
            for s in range(5, 12):
                table.observe_step({li: sorted(set(wids[s, li].reshape(-1).tolist())) for li in range(L)})
            r = paged_point(masters, dev, q, B, 32, routes, x, warm, steps, hbm_peak, h2d, prefetch=table)
            r["prefetch"] = "co-occurrence table, online, predict max(8, cap // 2) for the next layer"
            out["cfg1_b16_cap32_prefetch"] = r
    # prefill chunks of 2048 tokens per sequence, batch 1 and 4, cap 32
    for B, nl in ((1, 2), (4, 1)):
        T = 2048 * B
        tids, tw = wl.uniform_topk(T, q.experts, q.top_k, seed=40 + B)
        routes = [[(torch.from_numpy(tids).to(dev), torch.from_numpy(tw).to(dev)) for _ in range(nl)]]
        x = wl.hidden_states(T, q.hidden, seed=7).to(dev)
        r = paged_point(masters[:nl], dev, q, T, 32, routes, x, 0, 1, hbm_peak, h2d, layers=q.layers)
        r["prefill_tok_s"] = r.pop("tok_s")
        out[f"cfg2_prefill_b{B}_t2048_cap32"] = r
    # Mixtral-8x7B, 4 of its 32 layers timed
    m = wl.MIXTRAL_8X7B
    mm = make_masters(4, dev, shape=m)
    for B in (1, 8):
        steps, warm = 3, 2
        tids, tw = wl.zipf_trace(warm + steps, 4, B, m.experts, m.top_k, 0.8, 0.0, seed=21 + B)
        routes = [[(torch.from_numpy(tids[s, li]).to(dev), torch.from_numpy(tw[s, li]).to(dev))
                   for li in range(4)] for s in range(warm + steps)]
        x = wl.hidden_states(B, m.hidden, seed=B).to(dev)
        for C in (2, 4):
            out[f"cfg3_mixtral_b{B}_cap{C}"] = paged_point(mm, dev, m, B, C, routes, x, warm, steps, hbm_peak,
                                                           h2d, layers=m.layers)
    del mm
    release_pinned()
    return out


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
    host_memory_check(L * SHAPE.experts * SHAPE.expert_bytes, 1)
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
    prefill = None
    if not args.no_resident:
        for rb in sorted({B, 4, 1}, reverse=True):
            res[f"batch{rb}"] = resident_phase(args, masters, dev, hbm_peak, rb)
        # configs[2]'s 2048-token chunk on resident layers: the tensor-core prefill path alone
        pa = argparse.Namespace(**vars(args))
        pa.steps, pa.warmup = 4, 2
        prefill = prefill_only(pa, dev, hbm_peak, peak_src, masters=masters[:8])["prefill"]
        torch.cuda.empty_cache()
    sweep = None
    if args.sweep and args.workload == "qwen3-30b":
        t_sw = time.time()
        sweep = sweep_phase(masters, dev, hbm_peak, h2d)
        sweep["wall_s"] = time.time() - t_sw
    del masters
    release_pinned()
    if sweep is not None:
        # configs[4]'s shapes on one GPU (the same-shape line of the expert-parallel runs)
        t_sw = time.time()
        sweep["qwen3_235b_one_gpu"] = one_gpu_235b(args, dev, hbm_peak, h2d)
        sweep["qwen3_235b_one_gpu"]["wall_s"] = time.time() - t_sw
        use_workload(args.workload)

    roofline = None
    if res:
        r = res[f"batch{B}"]
        roofline = {"bound": "hbm", "kernel": r["kernel"],
                    "region": f"resident decode (cap = E), batch {B}, {r['layers']} layers: whole "
                              f"forward ({r['launches_per_forward']:.0f} launches) timed with CUDA events",
                    "achieved": r["hbm_gbs"], "peak": hbm_peak, "unit": "GB/s",
                    "frac": r["frac"], "peak_src": peak_src,
                    "traffic": profile_traffic(f"{r['kernel']}_resident_decode_b{B}.md",
                                               r["unique_experts_per_forward"]),
                    "traffic_note": "ncu DRAM read + write of one captured launch, scaled to this "
                                    "run's routed experts per launch",
                    "bytes_per_forward": r["bytes_per_forward"], "us_per_forward": r["us_per_forward"]}

    line = {
        "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded Zipf routing trace; random-init N(0,0.02) weights)",
        "config": {"workload": workload_name(args),
                   "layers": L, "batch": B, "cap": C, "experts": SHAPE.experts,
                   "top_k": SHAPE.top_k, "hidden": SHAPE.hidden, "inter": SHAPE.inter,
                   "routing": f"zipf{ZIPF} reuse{REUSE}", "l2": "inputs larger than L2 (each step reads "
                   f"every layer's routed experts, >= {L} x {SHAPE.top_k} x {SHAPE.expert_bytes / 1e6:.1f} MB, "
                   "from HBM)"},
        "gpu_launches": launches,
        "roofline": roofline,
        "step_roofline": step_roof,
        "pagein": {"gbs": pagein_gbs, "h2d_peak_gbs": h2d, "frac": pagein_gbs / h2d,
                   "misses": misses, "hits": hits, "bytes": pagein_bytes},
        "resident_decode": res,
        "resident_prefill": prefill,
        "configs": sweep,
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
            "config": {"workload": f"{SHAPE.name} {r['layers']}-layer expert stack, resident decode "
                                   f"batch {args.batch}"},
            "gpu_launches": r["launches"],
            "roofline": {"bound": "hbm", "kernel": r["kernel"], "achieved": r["hbm_gbs"],
                         "peak": hbm_peak, "unit": "GB/s", "frac": r["frac"], "peak_src": peak_src,
                         "bytes_per_forward": r["bytes_per_forward"], "us_per_forward": r["us_per_forward"]},
            "resident_decode": r}


def prefill_only(args, dev, hbm_peak, peak_src, masters=None):
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
    masters = masters if masters is not None else make_masters(L, dev)
    L = min(L, len(masters))
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
            "config": {"workload": f"{SHAPE.name} prefill, {L} resident layers, T {T}, uniform top-{SHAPE.top_k}"},
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


def run_wisp_ep(args):
    """Expert-parallel stack over the torchrun ranks (one GPU each): rank r owns
    experts [r E/P, (r+1) E/P) of every layer in its own pinned memory and
    pages them into its own slots; each rank decodes its own batch of --batch
    tokens (weak scaling: global batch = P x batch); the (token, k) rows move
    over peer memory (EPExchange).  For the default workload the layer's
    expert cache stays --cap slots in total, split evenly over the GPUs, so
    every shard pages at every P (the same fraction of each shard cached);
    for qwen3-235b --cap is per GPU.  Times are CUDA events, max
    over ranks."""
    import torch.distributed as dist
    from wisp_b200.expert_parallel import EPExchange, EPMoELayer
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    L, B = args.layers, args.batch
    E = SHAPE.experts
    per = E // world
    C = max(2, min(args.cap // world if args.cap_split else args.cap, per))
    total = args.warmup + args.steps
    t0 = time.time()
    host_memory_check(L * per * SHAPE.expert_bytes, world)
    lo, hi = rank * per, (rank + 1) * per
    masters = make_masters(L, dev, lo, hi)
    # a cap that holds the whole shard makes it resident (primed once)
    mode = "resident" if C == per else "paged"
    exchange = EPExchange(SHAPE.hidden, B * SHAPE.top_k, dev)
    layers = [EPMoELayer(h13, h2, E, C, mode, dev, i, exchange=exchange) for i, (h13, h2) in enumerate(masters)]
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
        lay.synchronize()
    tel0 = [lay.local.telemetry() for lay in layers]
    ex0 = exchange.launches
    dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # one nvidia-smi process on rank 0 samples every GPU of the run (queries from
    # inside the ranks' processes stalled the ranks' waits on one another)
    clk = SmiSampler(list(range(world)), enabled=rank == 0)
    with clk:
        ev0.record()
        for s in range(args.warmup, total):
            step(s, x_d, w_d, ids_d, out_d)
        ev1.record()
        torch.cuda.synchronize()
    dist.barrier()
    for lay in layers:
        lay.synchronize()
    tel1 = [lay.local.telemetry() for lay in layers]
    clocks = clk.summary()

    def delta(key):
        return sum(b[key] - a[key] for a, b in zip(tel0, tel1))

    stats = torch.tensor([ev0.elapsed_time(ev1), float(delta("pagein_bytes")),
                          float(delta("kernel_launches") + exchange.launches - ex0),
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
    torch.cuda.synchronize()
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
    exchange.close()
    del masters
    release_pinned()
    dist.barrier()
    h2d = h2d_peak_gbs(dev) if rank == 0 else 0.0
    pagein_gbs = float(stats[1]) / (ms * 1e-3) / 1e9
    steps_layers = args.steps * L
    return {
        "metric": METRIC, "value": world * B * args.steps / (ms * 1e-3), "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded Zipf routing trace; random-init N(0,0.02) weights)",
        "config": {"workload": workload_name(args, world),
                   "layers": L, "batch_per_gpu": B, "global_batch": B * world, "cap_per_gpu": C,
                   "cap_per_layer_total": C * world, "experts_per_gpu": per, "shard_mode": mode,
                   "parallelism": f"ep{world}", "exchange": "peer memory (CUDA IPC over NVLink), no collective",
                   "routing": f"zipf{ZIPF} reuse{REUSE}",
                   "l2": "inputs larger than L2 (each step reads every layer's routed experts from HBM)"},
        "gpu_launches": int(stats[2]),
        "roofline": None,
        "per_gpu": {"pagein_bytes_per_layer_step": float(stats[1]) / world / steps_layers,
                    "unique_experts_per_layer_step": float(stats[3]) / world / steps_layers,
                    "ms_per_layer_step": ms / steps_layers},
        "pagein": {"gbs_all_ranks": pagein_gbs, "h2d_peak_gbs_per_gpu": h2d,
                   "frac_of_per_gpu_peak_x_gpus": pagein_gbs / (h2d * world) if h2d else None,
                   "bytes": float(stats[1])},
        "e2e": {"value": world * B * e2e_steps / (float(e2e_ms[0]) * 1e-3), "unit": "tok/s",
                "h2d_bytes_per_step": int(ids_s.numel() * ids_s.element_size() + w_s.numel()
                                          * w_s.element_size() + x_h.numel() * x_h.element_size()) * world,
                "d2h_bytes_per_step": int(out_h.numel() * out_h.element_size()) * world,
                "steps": e2e_steps},
        "clocks": clocks,
        "setup_s": setup_s,
    }


def run_reference(args):
    """The reference path restated for the host cores, timed on a bounded
    sample: per layer and decode step, the reference's first-fit sub-batching
    and LRU pager (oracle/pager.py, bit-exact with fused_moe.py:264-358 and
    :1102-1168), each page-in a host copy into that layer's scratch slot (the
    reference's H2D copy), and vLLM fused_experts' arithmetic per group: each
    resident expert once over all of the group's tokens routed to it (bf16
    GEMMs with fp32 accumulation, h and a stored bf16, y = (W2 a) * w stored
    bf16), then the routing-order sum over k.  All host threads; the sampled
    layers' mean time per layer is scaled to the workload's layer count."""
    from oracle.pager import PagerOracle, first_fit_groups
    n = len(os.sched_getaffinity(0))
    torch.set_num_threads(n)
    L, B, C = args.layers, args.batch, args.cap
    E, H, I, K = SHAPE.experts, SHAPE.hidden, SHAPE.inter, SHAPE.top_k
    sample_layers = max(1, min(4, L))
    masters = []
    for li in range(sample_layers):
        # one expert's N(0, 0.02) weights copied to every expert: the values do
        # not change the time, and drawing every expert on the CPU takes minutes
        g = torch.Generator().manual_seed(1000 + li)
        w13 = torch.empty(E, 2 * I, H, dtype=torch.bfloat16)
        w2 = torch.empty(E, H, I, dtype=torch.bfloat16)
        b13 = (torch.randn(2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
        b2 = (torch.randn(H, I, generator=g) * 0.02).to(torch.bfloat16)
        for e in range(E):
            w13[e].copy_(b13)
            w2[e].copy_(b2)
        masters.append((w13, w2))
    scratch = [(torch.empty(C, 2 * I, H, dtype=torch.bfloat16), torch.empty(C, H, I, dtype=torch.bfloat16))
               for _ in range(sample_layers)]
    pagers = [PagerOracle(E, C) for _ in range(sample_layers)]
    n_trace = args.warmup + max(args.steps, 128)   # the sample wraps around it
    ids_np, w_np = routing(n_trace, sample_layers, B)
    x = wl.hidden_states(B, H, seed=0)
    silu = torch.nn.functional.silu

    def layer_fwd(li, s):
        s = args.warmup + (s - args.warmup) % (n_trace - args.warmup) if s >= n_trace else s
        ids = ids_np[s, li]
        w = torch.from_numpy(w_np[s, li])
        p = pagers[li]
        p.stats_forward += 1
        out = torch.empty(B, H, dtype=torch.bfloat16)
        for t0, t1 in first_fit_groups(ids, C):
            rec = p.ensure_resident(ids[t0:t1])
            for e, slot in rec.placed:
                scratch[li][0][slot].copy_(masters[li][0][e])
                scratch[li][1][slot].copy_(masters[li][1][e])
            gid = torch.from_numpy(ids[t0:t1].astype(np.int64))
            y = torch.empty(t1 - t0, K, H, dtype=torch.bfloat16)
            for e in torch.unique(gid).tolist():
                rows, cols = (gid == e).nonzero(as_tuple=True)
                slot = p.expert_to_slot[e]
                h = x[t0 + rows] @ scratch[li][0][slot].T                      # bf16 out, fp32 accumulate
                a = (silu(h[:, :I].float()).to(torch.bfloat16).float() * h[:, I:].float()).to(torch.bfloat16)
                y[rows, cols] = ((a @ scratch[li][1][slot].T).float()
                                 * w[t0 + rows, cols].unsqueeze(1)).to(torch.bfloat16)
            acc = y[:, 0].float()
            for k in range(1, K):
                acc = acc + y[:, k].float()
                if K <= 4:
                    acc = acc.to(torch.bfloat16).float()
            out[t0:t1] = acc.to(torch.bfloat16)
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
        if time.perf_counter() - t0 > args.cpu_sample_s:
            break
    dt = time.perf_counter() - t0
    per_layer = dt / (done * sample_layers)
    tok_s = B / (per_layer * L)
    return {"value": tok_s, "unit": "tok/s", "cores": n, "kind": "port",
            "sample": f"{done} decode steps x {sample_layers} layers (of {L}) at batch {B}, cap {C}: each "
                      f"expert computed once per token group (bf16 GEMMs, fp32 accumulation); tok/s = batch / "
                      f"(mean time per layer x {L}) ({dt:.1f} s of CPU work)"}


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
                "data": "synthetic", "config": {"workload": workload_name(args, args.gpus)},
                "cpu_baseline": cpu,
                "e2e": {"value": cpu["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return
    world = int(os.environ.get("WORLD_SIZE", 1))
    if world > 1:
        import datetime

        import torch.distributed as dist
        dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
        line = run_wisp_ep(args)
        if args.sweep and args.workload == "qwen3-30b":
            # configs[4] (the expert-parallel configuration) at this GPU count
            line["configs"] = {"ep_qwen3_235b": run_wisp_ep(workload_args(args, "qwen3-235b", steps=3, warmup=2))}
            use_workload("qwen3-30b")
        dist.barrier()
        dist.destroy_process_group()
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
