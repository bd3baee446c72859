"""Benchmark of the B200 gpt-oss MoE layer (one JSON line on rank 0).

Default workload: the gpt-oss-120b-shaped MoE layer (H = I = 2880, 128 experts,
top-4, MXFP4 experts) over an 8192-token prefill batch, all experts resident
on each GPU at N=1.  A "step" is one layer forward: router, dispatch, gate_up +
SwiGLU, down, weighted combine, replayed from a CUDA graph (at every N).
Inputs are seeded synthetic tensors (no checkpoint exists offline); the
weights (1.69 GB) are larger than L2, so no extra L2 flush is needed between
steps.  The default run also measures BASELINE configs 2 and 3 (20b prefill of
4096 tokens; 120b decode of 1, 8 and 64 tokens) and reports them under
"configs", each with its own roofline.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload gptoss120b-prefill-8192|gptoss120b-decode-T|gptoss20b-prefill-4096|
                              gptoss120b-zipf-16384-streamed]

``--impl reference`` runs the reference's own CPU path -- transformers'
GptOssTopKRouter and block_streamer.gptoss.MXFP4Experts from the installed
package under baseline/_ref -- on rank 0: every step routes all tokens and
runs one group of the hit experts, so that the steps together run the whole
layer once (or a whole number of times); the line says what ran.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import time

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

from blockstreamer_b200 import kernels  # noqa: E402
from blockstreamer_b200.synthetic import (CASES, algorithmic_bytes, algorithmic_flops,  # noqa: E402
                                          expert_bytes, make_layer, make_tokens)

METRIC = "MoE-layer tokens/s at gpt-oss-120b shape"
DEFAULT_WORKLOAD = "gptoss120b-prefill-8192"
BACKWARD_WORKLOAD = "gptoss120b-prefill-8192-backward"
EXTRA_WORKLOADS = ("gptoss20b-prefill-4096", "gptoss120b-decode-1", "gptoss120b-decode-8",
                   "gptoss120b-decode-64")
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
FP4_DENSE_NOMINAL_TFLOPS = 9000.0
L2_BYTES = 126 * 1024 * 1024
# DRAM bytes per launch (read + write) of the expert GEMMs, from one earlier
# ncu capture of the default workload; stored constants, not measured per run.
NCU_TRAFFIC = {("gptoss120b-prefill-8192", "gate_up"): 1501327360,
               ("gptoss120b-prefill-8192", "down"): 924871936}
# decode shapes: steps rotate over this many distinct layers (see measure())
ROT_LAYERS = 8
# a timed region shorter than this runs at the burst clock: its tensor-bound
# kernels are compared with the burst (not the sustained) GEMM peak
SUSTAINED_REGION_S = 1.0


def parse_workload(name: str):
    if name == BACKWARD_WORKLOAD:
        return "gptoss120b", 6, 8192
    if name.startswith("gptoss120b-zipf-"):   # gptoss120b-zipf-<T>-streamed
        return "gptoss120b", 5, int(name.split("-")[2])
    if name.startswith("gptoss120b-prefill-"):
        return "gptoss120b", 4, int(name.rsplit("-", 1)[1])
    if name.startswith("gptoss120b-decode-"):
        return "gptoss120b", 3, int(name.rsplit("-", 1)[1])
    if name.startswith("gptoss20b-prefill-"):
        return "gptoss20b", 2, int(name.rsplit("-", 1)[1])
    raise SystemExit(f"unknown workload {name}")


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


def tensor_peak(peaks, region_s):
    """(peak TFLOP/s, label): burst for a short timed region, sustained for a long one."""
    if region_s >= SUSTAINED_REGION_S and "bf16_tflops_sustained" in peaks:
        return peaks["bf16_tflops_sustained"], "bf16 dense sustained (cuBLAS, seconds-long loop)"
    return peaks["bf16_tflops"], f"bf16 dense burst (cuBLAS; timed region {region_s * 1e3:.0f} ms)"


class ClockSampler:
    """SM clock and clock-event (throttle) reasons, read through NVML every
    ~1 ms by a background thread while the timed region runs (the decode
    regions last a few milliseconds, shorter than nvidia-smi's sampling
    period).  Read-only: no clock or power setting is touched."""

    REASONS = (("hw_slowdown", "HwSlowdown"), ("hw_thermal_slowdown", "HwThermalSlowdown"),
               ("sw_thermal_slowdown", "SwThermalSlowdown"), ("sw_power_cap", "SwPowerCap"))

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []
        self.max_mhz = None
        self._stop = None
        self._thread = None

    def _handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        try:
            pr = torch.cuda.get_device_properties(self.gpu)
            bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.gpu)

    def __enter__(self):
        import threading
        try:
            nv, h = self._handle()
        except Exception:
            return self
        try:
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        except Exception:
            self.max_mhz = None
        masks = [(name, getattr(nv, "nvmlClocksEventReason" + suffix, 0)) for name, suffix in self.REASONS]
        self._stop = threading.Event()

        def poll():
            while not self._stop.is_set():
                try:
                    mhz = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                    bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((mhz, [n for n, m in masks if m and bits & m]))
                except Exception:
                    return
                self._stop.wait(0.001)

        self._thread = threading.Thread(target=poll, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "source": "nvml"}
        reasons = sorted({r for _, rs in self.samples for r in rs})
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples), "source": "nvml, ~1 ms period"}


def dist_setup(n_gpus: int):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- reference arm

def cpu_inputs(key: str, case_id: int, T: int):
    shape = CASES[key]
    return shape, make_layer(shape, case_id), make_tokens(T, shape.hidden, case_id)


def cpu_sample(shape, p, x, experts_in_sample: int = 8):
    """The cpu_baseline of our arm: the oracle port (the reference's bf16
    per-expert loop restated on torch CPU ops) on a bounded sample of the
    workload -- the router over all T tokens plus the full expert work of
    ``experts_in_sample`` of the hit experts; the expert time is scaled to
    all hit experts, as the sample string says."""
    from oracle import moe as omoe
    T = x.shape[0]
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    pe = {k.split(".", 1)[1]: v for k, v in p.items() if k.startswith("experts.")}
    t0 = time.perf_counter()
    _, sc, idx = omoe.router(x.float(), p["router.weight"], p["router.bias"], shape.top_k)
    t_router = time.perf_counter() - t0
    hit = sorted(set(idx.reshape(-1).tolist()))
    subset = hit[:experts_in_sample]
    t0 = time.perf_counter()
    omoe.experts_port(x, idx, sc, pe, experts_subset=subset)
    t_exp = time.perf_counter() - t0
    scale = len(hit) / max(len(subset), 1)
    t_total = t_router + t_exp * scale
    return {"value": T / t_total, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": (f"oracle port: router over all {T} tokens ({t_router:.2f} s) + the bf16 expert "
                       f"loop of {len(subset)} of {len(hit)} hit experts ({t_exp:.2f} s); expert time "
                       f"scaled by {scale:.1f} to all hit experts"),
            "seconds": t_router + t_exp}


def load_reference():
    """The reference's own modules from its installed package (baseline/_ref):
    (MXFP4Experts, GptOssConfig, GptOssTopKRouter), or (None, reason)."""
    ref_dir = os.path.join(REPO, "baseline", "_ref")
    if not os.path.exists(os.path.join(ref_dir, "block_streamer", "gptoss.py")):
        return None, "the reference package is not installed under baseline/_ref"
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    try:
        from block_streamer.gptoss import MXFP4Experts
        from transformers.models.gpt_oss.configuration_gpt_oss import GptOssConfig
        from transformers.models.gpt_oss.modeling_gpt_oss import GptOssTopKRouter
    except Exception as e:  # noqa: BLE001 - reported in the line
        return None, f"importing the reference failed: {type(e).__name__}: {e}"
    return (MXFP4Experts, GptOssConfig, GptOssTopKRouter), None


def run_reference(args, rank, world):
    """The reference arm: transformers' GptOssTopKRouter + the reference's
    MXFP4Experts (block_streamer/gptoss.py:137-177), unmodified, on the host
    cores.  The whole layer takes tens of seconds on a CPU, so its hit experts
    are split into groups: every step routes all T tokens and runs one group
    (its experts' (token, slot) rows through MXFP4Experts.forward, exactly the
    per-expert work of the full layer), and the steps cycle over the groups a
    whole number of times.  layer time = mean router time + the sum over the
    groups of their mean expert time; value = T / layer time."""
    key, case_id, T = parse_workload(args.workload)
    if rank != 0:
        return
    mods, why = load_reference()
    if mods is None:
        print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
        return
    MXFP4Experts, GptOssConfig, GptOssTopKRouter = mods
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    shape, p, x = cpu_inputs(key, case_id, T)
    E, k = shape.experts, shape.top_k
    cfg = GptOssConfig(hidden_size=shape.hidden, intermediate_size=shape.intermediate, num_local_experts=E,
                       num_experts_per_tok=k, swiglu_limit=shape.swiglu_limit)
    router = GptOssTopKRouter(cfg)
    router.weight.data = p["router.weight"]
    router.bias.data = p["router.bias"]
    names = ("gate_up_proj_blocks", "gate_up_proj_scales", "gate_up_proj_bias",
             "down_proj_blocks", "down_proj_scales", "down_proj_bias")

    def group_module(e0, e1):
        gcfg = GptOssConfig(hidden_size=shape.hidden, intermediate_size=shape.intermediate,
                            num_local_experts=e1 - e0, num_experts_per_tok=1,
                            swiglu_limit=shape.swiglu_limit)
        m = MXFP4Experts(gcfg, torch.bfloat16)
        for n in names:
            setattr(m, n, torch.nn.Parameter(p["experts." + n][e0:e1], requires_grad=False))
        return m

    with torch.no_grad():
        _, sc, idx = router(x.float())
    hit = sorted(set(idx.reshape(-1).tolist()))
    per = max(1, math.ceil(len(hit) / max(args.steps, 1)))
    groups = [hit[i:i + per] for i in range(0, len(hit), per)]
    cycles = max(1, args.steps // len(groups))

    def run_group(g):
        # the rows of the group's experts, one per (token, slot), with the
        # experts renumbered into the group module (its experts are a
        # contiguous slice of the layer's; experts of the range that no
        # token picked cost nothing in MXFP4Experts.forward)
        e0, e1 = g[0], g[-1] + 1
        sel = (idx >= e0) & (idx < e1)
        tok, slot = torch.nonzero(sel, as_tuple=True)
        m = group_module(e0, e1)
        t0 = time.perf_counter()
        with torch.no_grad():
            router(x.float())
            t1 = time.perf_counter()
            m(x[tok], (idx[tok, slot] - e0).unsqueeze(1), sc[tok, slot].unsqueeze(1))
        t2 = time.perf_counter()
        return t1 - t0, t2 - t1

    for i in range(args.warmup):          # warm-up: one expert each, untimed
        run_group(hit[i % len(hit): i % len(hit) + 1])
    t_router, t_group = [], [[] for _ in groups]
    wall0 = time.perf_counter()
    for _ in range(cycles):
        for gi, g in enumerate(groups):
            tr, te = run_group(g)
            t_router.append(tr)
            t_group[gi].append(te)
    wall = time.perf_counter() - wall0
    steps = cycles * len(groups)
    layer_s = statistics.mean(t_router) + sum(statistics.mean(v) for v in t_group)
    v = T / layer_s
    sample = (f"reference GptOssTopKRouter + block_streamer.gptoss.MXFP4Experts (baseline/_ref) on "
              f"{threads} host threads: {steps} steps, each routing all {T} tokens and running a group of "
              f"{per} of the {len(hit)} hit experts ({len(groups)} groups, {cycles} full cycle(s) = the "
              f"whole layer {cycles} time(s)); layer time {layer_s:.2f} s = router {statistics.mean(t_router):.3f} s "
              f"+ the groups' expert times; {wall:.1f} s of timed CPU work")
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": world,
            "steps": steps, "warmup": args.warmup, "ms_per_step": 1e3 * wall / steps,
            "layer_ms": 1e3 * layer_s, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic", "config": {"workload": args.workload, "tokens": T},
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- our arm

STAGES = ("router", "dispatch", "gate_up", "down", "combine")
LAUNCHES = {"router": 3, "dispatch": 4, "gate_up": 1, "down": 1, "combine": 1}  # router: 2 at T <= 64
ALGOS = {"auto": kernels.ALGO_AUTO, "gemv": kernels.ALGO_GEMV, "tcgen05": kernels.ALGO_TCGEN05,
         "mx": kernels.ALGO_MX, "fused": kernels.ALGO_FUSED, "tcgen05_pair": kernels.ALGO_TCGEN05_PAIR}


def layer_stages(x, p, k, algo, bufs):
    """The layer as its C-ABI stages (the same kernels bs_moe_forward runs),
    with every output and workspace allocated once up front."""
    dev = x.device
    E = p["experts.gate_up_proj_blocks"].shape[0]
    T, H = x.shape
    I = p["experts.gate_up_proj_blocks"].shape[1] // 2
    S = T * k
    lib = kernels._lib.load()
    bufs["sc"] = torch.empty(T, k, dtype=torch.float32, device=dev)
    bufs["idx"] = torch.empty(T, k, dtype=torch.int32, device=dev)
    bufs["rws"] = torch.empty(lib.bs_router_workspace_bytes(T, H, E, kernels._lib.BS_F32),
                              dtype=torch.uint8, device=dev)
    bufs["d"] = kernels.Dispatch(torch.empty(E + 1, dtype=torch.int32, device=dev),
                                 torch.empty(S, dtype=torch.int32, device=dev),
                                 torch.empty(S, dtype=torch.int32, device=dev),
                                 torch.empty(S, H, dtype=torch.bfloat16, device=dev))
    bufs["dws"] = torch.empty(lib.bs_dispatch_workspace_bytes(T, k, E), dtype=torch.uint8, device=dev)
    bufs["h"] = torch.empty(S, I, dtype=torch.bfloat16, device=dev)
    bufs["y"] = torch.empty(S, H, dtype=torch.bfloat16, device=dev)
    bufs["out"] = torch.empty(T, H, dtype=torch.bfloat16, device=dev)

    def router():
        kernels.router(x, p["router.weight"], p["router.bias"], k, out_scores=bufs["sc"],
                       out_indices=bufs["idx"], workspace=bufs["rws"])

    def dispatch():
        kernels.dispatch(bufs["idx"], E, x, out=bufs["d"], workspace=bufs["dws"])

    def gate_up():
        d = bufs["d"]
        kernels.moe_gate_up(d.x_perm, d.expert_offsets, p["experts.gate_up_proj_blocks"],
                            p["experts.gate_up_proj_scales"], p["experts.gate_up_proj_bias"],
                            algo=algo, out=bufs["h"])

    def down():
        d = bufs["d"]
        kernels.moe_down(bufs["h"], d.expert_offsets, p["experts.down_proj_blocks"],
                         p["experts.down_proj_scales"], p["experts.down_proj_bias"], algo=algo,
                         out=bufs["y"])

    def combine():
        kernels.combine(bufs["y"], bufs["d"].row_of_slot, bufs["sc"], T, out=bufs["out"])

    return [("router", router), ("dispatch", dispatch), ("gate_up", gate_up), ("down", down),
            ("combine", combine)]


def capture(fn):
    """fn's launches as a CUDA graph (fn has run eagerly before, so every
    one-time set-up is done)."""
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


def graphed_stage_ms(stages, steps, world):
    """Per-stage device time: each stage captured in a CUDA graph of its own,
    the graphs replayed in layer order, with events between replays on the
    launch stream (mean over ``steps`` layers; max over ranks)."""
    for _, fn in stages:
        fn()
    torch.cuda.synchronize()
    graphs = [(name, capture(fn)) for name, fn in stages]
    for _, g in graphs:
        g.replay()
    torch.cuda.synchronize()
    barrier(world)
    st = torch.cuda.current_stream()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(len(graphs) + 1)] for _ in range(steps)]
    for i in range(steps):
        evs[i][0].record(st)
        for j, (_, g) in enumerate(graphs):
            g.replay()
            evs[i][j + 1].record(st)
    torch.cuda.synchronize()
    out = {name: max_over_ranks(statistics.mean(evs[i][j].elapsed_time(evs[i][j + 1]) for i in range(steps)),
                                world)
           for j, (name, _) in enumerate(graphs)}
    del graphs
    return out


def time_steps(step, steps, flush_buf, world):
    """Device time of one step (ms): K steps between two events, or, with an
    L2 flush buffer, each step after a 2xL2 write, timed on its own."""
    st = torch.cuda.current_stream()
    barrier(world)
    torch.cuda.synchronize()
    if flush_buf is not None:
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(steps)]
        for a, b in evs:
            flush_buf.fill_(1)
            a.record(st)
            step()
            b.record(st)
        torch.cuda.synchronize()
        ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
    else:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(steps):
            step()
        e1.record(st)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
    barrier(world)
    return max_over_ranks(ms, world)


def e2e_ms(layer_call, x, steps, warmup, world, pipelined):
    """The layer through the public API with host buffers: every step copies
    its tokens in from pinned host memory and its output back out.
    Pipelined (prefill sizes): the copies run on their own streams, so step
    i+1's host->device copy and step i-1's device->host copy overlap step i's
    layer (double-buffered, as a serving loop runs it); timed from the first
    timed step's input copy to the last timed step's output copy.  Otherwise
    (decode sizes, kilobyte copies): copy in, layer, copy out per step."""
    st = torch.cuda.current_stream()
    x_host = x.cpu().pin_memory()
    out_host = [torch.empty_like(x_host).pin_memory() for _ in range(2)]
    x_dev = [torch.empty_like(x) for _ in range(2)]
    if pipelined:
        s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
        comp_done = [None, None]

        def e2e_step(i, first_event=None):
            b = i % 2
            with torch.cuda.stream(s_in):
                if comp_done[b] is not None:
                    s_in.wait_event(comp_done[b])   # the layer two steps back has read x_dev[b]
                if first_event is not None:
                    first_event.record(s_in)
                x_dev[b].copy_(x_host, non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(s_in)
            st.wait_event(ready)
            o = layer_call(x_dev[b])
            done = torch.cuda.Event()
            done.record(st)
            comp_done[b] = done
            o.record_stream(s_out)
            with torch.cuda.stream(s_out):
                s_out.wait_event(done)
                out_host[b].copy_(o, non_blocking=True)

        for i in range(warmup):
            e2e_step(i)
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for i in range(steps):
            e2e_step(i, e0 if i == 0 else None)
        e1.record(s_out)
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1) / steps, world)
    times = []
    for i in range(warmup + steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st)
        x_dev[0].copy_(x_host, non_blocking=True)
        o = layer_call(x_dev[0])
        out_host[0].copy_(o, non_blocking=True)
        b.record(st)
        b.synchronize()
        if i >= warmup:
            times.append(a.elapsed_time(b))
    return max_over_ranks(statistics.mean(times), world)


def measure(workload, args, world, local):
    """One workload on one GPU: value (graph-replayed layer, device-timed),
    per-stage times, e2e through the public API, and the rooflines."""
    key, case_id, T = parse_workload(workload)
    shape = CASES[key]
    k, E, H, I = shape.top_k, shape.experts, shape.hidden, shape.intermediate
    dev = torch.device("cuda", torch.cuda.current_device())
    algo = ALGOS[args.algo]
    # the decode paths: one bs_moe_forward call = 4 launches (route, gate_up,
    # down, combine), or one cooperative launch with --algo fused (T <= 8)
    fused_path = algo == kernels.ALGO_FUSED
    mx_path = fused_path or algo == kernels.ALGO_MX or (algo == kernels.ALGO_AUTO and T <= 64)
    p = make_layer(shape, case_id, device=dev)
    x = make_tokens(T, H, case_id, device=dev)
    gu = (p["experts.gate_up_proj_blocks"], p["experts.gate_up_proj_scales"], p["experts.gate_up_proj_bias"])
    dn = (p["experts.down_proj_blocks"], p["experts.down_proj_scales"], p["experts.down_proj_bias"])
    ws = torch.empty(kernels._lib.load().bs_moe_workspace_bytes(T, H, I, E, k), dtype=torch.uint8, device=dev)

    def layer_fn(lp):
        lgu = (lp["experts.gate_up_proj_blocks"], lp["experts.gate_up_proj_scales"], lp["experts.gate_up_proj_bias"])
        ldn = (lp["experts.down_proj_blocks"], lp["experts.down_proj_scales"], lp["experts.down_proj_bias"])

        def call(xin, workspace=ws):
            return kernels.moe_forward(xin, *lgu, *ldn, k, router_weight=lp["router.weight"],
                                       router_bias=lp["router.bias"], algo=algo, workspace=workspace)
        return call

    layer = layer_fn(p)
    for _ in range(args.warmup):
        out, sc, idx = layer(x)
    torch.cuda.synchronize()
    distinct = int(torch.unique(idx).numel())
    counts = torch.bincount(idx.reshape(-1).long(), minlength=E)
    # When one step's touched weights would fit in L2 (decode shapes), the
    # steps rotate over ROT_LAYERS distinct seeded layers, as a model's layer
    # loop does: each step's weights were last read ROT_LAYERS - 1 steps (far
    # more than L2's worth of other weights) earlier, so they come from HBM,
    # while the kernels' code and the tokens stay cached.
    rotate = distinct * expert_bytes(shape) < 2 * L2_BYTES
    layers = [p] + ([make_layer(shape, 1000 + 10 * case_id + i, device=dev) for i in range(1, ROT_LAYERS)]
                    if rotate else [])
    calls = [layer] + [layer_fn(lp) for lp in layers[1:]]
    distincts = [distinct]
    for c in calls[1:]:
        _, _, idx_r = c(x)
        distincts.append(int(torch.unique(idx_r).numel()))
    torch.cuda.synchronize()
    graphed = not args.no_graph
    graph_ok = None
    if graphed:
        # the whole layer (no host synchronization inside) replayed from a CUDA graph
        graphs = []
        for i, c in enumerate(calls):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                g_out, _, _ = c(x)
            g.replay()
            torch.cuda.synchronize()
            if i == 0:
                graph_ok = bool(torch.equal(g_out, out))
            graphs.append(g)
        replays = [g.replay for g in graphs]
    else:
        replays = [(lambda c=c: c(x)) for c in calls]
    turn = [0]

    def step():
        replays[turn[0] % len(replays)]()
        turn[0] += 1
    assert kernels.device_status(clear=True) == 0

    with ClockSampler(local) as clk:
        ms = time_steps(step, args.steps, None, world)
    value = T / (ms * 1e-3)
    distinct_mean = statistics.mean(distincts)

    # per-stage breakdown: each C-ABI stage from its own graph replay.  The
    # decode paths' launches sit inside one C call; their breakdown comes
    # from the ncu launch list instead.
    if mx_path:
        stage_ms = {"layer": ms}
    else:
        bufs = {}
        stage_ms = graphed_stage_ms(layer_stages(x, p, k, algo, bufs), args.steps, world)
        del bufs

    pipelined = T > 64
    e2e_turn = [0]

    def e2e_call(xin):
        c = calls[e2e_turn[0] % len(calls)]
        e2e_turn[0] += 1
        return c(xin, None)[0]
    ms_e2e = e2e_ms(e2e_call, x, args.steps, args.warmup, world, pipelined)

    # --- roofline of the dominant kernel
    peaks, peak_src = load_peaks()
    S = T * k
    stage_flops = {"gate_up": S * 4.0 * H * I, "down": S * 2.0 * H * I, "router": 2.0 * T * H * E}
    G = H // 32
    gu_bytes = distinct_mean * (2 * I * G * 17 + 2 * I * 2) + S * H * 2 + S * I * 2
    dn_bytes = distinct_mean * (H * (I // 32) * 17 + H * 2) + S * I * 2 + S * H * 2
    stage_bytes = {"gate_up": gu_bytes, "down": dn_bytes, "router": E * H * 4 + T * H * 2,
                   "dispatch": 2 * S * H * 2, "combine": S * H * 2 + T * H * 2,
                   "layer": algorithmic_bytes(T, shape, distinct_mean)}
    dom = max(stage_ms, key=stage_ms.get)
    tensor_bound = (S / max(distinct, 1)) > 64 and dom in ("gate_up", "down")
    dur_s = stage_ms[dom] * 1e-3
    region_s = ms * args.steps * 1e-3
    if tensor_bound:
        achieved = stage_flops[dom] / dur_s / 1e12
        peak, plabel = tensor_peak(peaks, region_s)
        traffic = NCU_TRAFFIC.get((workload, dom))
        roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "traffic": traffic, "kernel": dom,
                "peak_source": f"{peak_src} {plabel}; the MMA runs bf16 x bf16",
                "traffic_source": ("stored constant from one ncu capture of this workload (DRAM read + write "
                                   "per launch), not measured in this run") if traffic else None}
    else:
        achieved = stage_bytes[dom] / dur_s / 1e9
        peak = peaks["hbm_gbs"]
        roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "traffic": None, "kernel": dom,
                "peak_source": f"{peak_src} HBM copy bandwidth"}
        if dom == "layer":
            roof["kernel"] = (("whole layer, one cooperative kernel (decode_fused_kernel)" if fused_path else
                               "whole layer (route, gate_up, down, combine launches)") +
                              ": weights of the touched experts + router weights + tokens over the "
                              "device-timed step; a lower bound for the expert streaming, >97% of the bytes")
    roof["algorithmic"] = {"flops": stage_flops.get(dom), "bytes": stage_bytes.get(dom), "launch_ms": stage_ms[dom]}
    layer_flops = algorithmic_flops(T, shape)
    layer_bytes = algorithmic_bytes(T, shape, distinct_mean)
    t_fp4 = layer_flops / (FP4_DENSE_NOMINAL_TFLOPS * 1e12)
    t_hbm = layer_bytes / (peaks["hbm_gbs"] * 1e9)
    layer_roof = {"flops": layer_flops, "bytes": layer_bytes, "distinct_experts": distinct_mean,
                  "floor_us_fp4_nominal": t_fp4 * 1e6, "floor_us_hbm_measured": t_hbm * 1e6,
                  "frac_of_fp4_hbm_roofline": max(t_fp4, t_hbm) / (ms * 1e-3),
                  "frac_of_bf16_burst_measured": (layer_flops / (ms * 1e-3) / 1e12) / peaks["bf16_tflops"],
                  "stage_ms": stage_ms,
                  "stage_ms_source": ("each C-ABI stage replayed from its own CUDA graph, events between "
                                      "replays" if not mx_path else "whole layer (one C call)")}
    return {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": workload, "tokens": T, "hidden": H, "intermediate": I, "experts": E,
                       "top_k": k,
                       "weights": "MXFP4 e2m1 + e8m0 scales (uniform codes, scales U{%d..%d})" % (
                           shape.scale_lo, shape.scale_hi),
                       "algo": args.algo, "cuda_graph": graphed, "graph_output_equals_eager": graph_ok,
                       "l2": (f"steps rotate over {len(calls)} distinct seeded layers ({len(calls)} x "
                              f"{expert_bytes(shape) * E / 1e9:.2f} GB of weights); each step's touched weights "
                              f"(~{distinct_mean * expert_bytes(shape) / 1e6:.0f} MB) were last read {len(calls) - 1} "
                              "steps earlier, after more than L2 of other weights, so they come from HBM; the "
                              "kernels' code and the tokens stay cached, as in a model's layer loop"
                              if rotate else "inputs larger than L2 (expert weights read per step exceed L2)"),
                       "expert_rows_min_max": [int(counts.min()), int(counts.max())]},
            "roofline": roof, "layer_roofline": layer_roof,
            "e2e": {"value": T / (ms_e2e * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": x.numel() * 2, "d2h_bytes_per_step": x.numel() * 2,
                    "api": "blockstreamer_b200.kernels.moe_forward -> bs_moe_forward",
                    "pipelining": ("copies on their own streams: step i+1's H2D and step i-1's D2H "
                                   "overlap step i's layer (double-buffered)") if pipelined else
                                  "none (decode size: copy, layer, copy back per step)"},
            "clocks": clk.summary(),
            "gpu_launches": (1 if fused_path else 4 if mx_path else sum(LAUNCHES.values())) * args.steps}


def measure_backward(args, local):
    """The expert layer's backward (bs_moe_backward: dL/dx and dL/d routing
    weights) at the default workload, graph-replayed and device-timed: the
    forward's dispatch and projections recomputed, two transposed grouped
    GEMMs, the weighted-sum and un-permute backward."""
    key, case_id, T = parse_workload(DEFAULT_WORKLOAD)
    shape = CASES[key]
    k, E, H, I = shape.top_k, shape.experts, shape.hidden, shape.intermediate
    dev = torch.device("cuda", torch.cuda.current_device())
    p = make_layer(shape, case_id, device=dev)
    x = make_tokens(T, H, case_id, device=dev)
    _, sc, idx = kernels.router(x, p["router.weight"], p["router.bias"], k, index_dtype=torch.int32)
    gout = torch.randn(T, H, generator=torch.Generator(device=dev).manual_seed(9), device=dev).to(torch.bfloat16)
    names = ("gate_up_proj_blocks", "gate_up_proj_scales", "gate_up_proj_bias", "down_proj_blocks",
             "down_proj_scales", "down_proj_bias")
    pe = [p["experts." + n] for n in names]
    for _ in range(args.warmup):
        kernels.moe_backward(x, idx, sc, gout, *pe)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        kernels.moe_backward(x, idx, sc, gout, *pe)
    g.replay()
    torch.cuda.synchronize()
    assert kernels.device_status(clear=True) == 0
    ms = time_steps(g.replay, args.steps, None, 1)
    S = T * k
    # recomputed forward projections (2 * S * H * 3I) + the two transposed GEMMs (same FLOPs)
    flops = 2.0 * (S * 2.0 * H * 3 * I)
    peaks, peak_src = load_peaks()
    peak, plabel = tensor_peak(peaks, ms * args.steps * 1e-3)
    return {"value": T / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms,
            "what": "bs_moe_backward: dL/dx and dL/d routing weights of the expert layer (recomputed forward "
                    "projections, transposed tcgen05 GEMMs for dh and dx), CUDA-graph replay",
            "roofline": {"bound": "tensor", "achieved": flops / (ms * 1e-3) / 1e12, "peak": peak,
                         "unit": "TFLOP/s", "frac": flops / (ms * 1e-3) / 1e12 / peak,
                         "peak_source": f"{peak_src} {plabel}", "flops_per_step": flops}}


def run_ours(args, rank, world, local):
    key, case_id, T_total = parse_workload(args.workload)
    shape = CASES[key]
    if case_id == 5:
        return run_bench_streamed(args, rank, world, shape, case_id, T_total)
    if case_id == 6:   # the expert backward alone (also part of the default run's configs)
        if world > 1:
            raise SystemExit("the backward workload runs on one GPU")
        r = measure_backward(args, local)
        line = {"metric": "expert-layer backward tokens/s at gpt-oss-120b shape", "value": r["value"],
                "unit": r["unit"], "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": args.workload, "tokens": T_total, "what": r["what"]},
                "roofline": r["roofline"]}
        print(json.dumps(line), flush=True)
        return
    if world > 1:
        return run_bench_ep(args, rank, world, local, shape, case_id, T_total)
    line = measure(args.workload, args, world, local)
    torch.cuda.empty_cache()
    if args.workload == DEFAULT_WORKLOAD and not args.no_extra:
        # BASELINE configs 2 and 3 in the same run, each with its own roofline
        extra = {}
        for w in EXTRA_WORKLOADS:
            r = measure(w, args, world, local)
            torch.cuda.empty_cache()
            extra[w] = {n: r[n] for n in ("value", "unit", "ms_per_step", "roofline", "layer_roofline", "e2e",
                                          "clocks", "gpu_launches")}
            extra[w]["config"] = r["config"]
        extra[BACKWARD_WORKLOAD] = measure_backward(args, local)
        torch.cuda.empty_cache()
        line["configs"] = extra
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        shape_c, p_c, x_c = cpu_inputs(key, case_id, T_total)
        cb = cpu_sample(shape_c, p_c, x_c)
        line["cpu_baseline"] = {k2: cb[k2] for k2 in ("value", "unit", "cores", "kind", "sample")}
    if rank == 0:
        print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- expert parallel (N > 1)

def run_bench_ep(args, rank, world, local, shape, case_id, T_total):
    """The same layer split over `world` ranks: experts [r*E/R, (r+1)*E/R) and
    T/R tokens per rank (strong scaling: the 8192-token batch is fixed).
    After timing, every rank checks its output slice against the single-GPU
    layer on the same tokens (outside the timed region)."""
    import torch.distributed as dist
    from blockstreamer_b200.expert_parallel import ExpertParallelMoE, P2PExchange, shard_experts

    dev = torch.device("cuda", local)
    if T_total % world:
        raise SystemExit(f"{T_total} tokens do not split over {world} ranks")
    Tr = T_total // world
    full = make_layer(shape, case_id, device=dev)
    router_w, router_b = full["router.weight"], full["router.bias"]
    full_e = {k.split(".", 1)[1]: v for k, v in full.items() if k.startswith("experts.")}
    local_p = shard_experts(full_e, rank, world)
    x_all = make_tokens(T_total, shape.hidden, case_id, device=dev)
    x = x_all[rank * Tr:(rank + 1) * Tr].contiguous()
    del x_all
    torch.cuda.empty_cache()
    exchange = None
    if args.ep_transport == "p2p":
        exchange = P2PExchange(None, shape.experts, shape.hidden, Tr, shape.top_k, dev)
    layer = ExpertParallelMoE(shape.experts, shape.top_k, exchange=exchange)

    def step():
        return layer(x, router_w, router_b, local_p)

    for _ in range(args.warmup):
        out_eager, _, _ = step()
    torch.cuda.synchronize()
    # The peer-memory path has no host synchronization: one layer call is
    # captured as a CUDA graph (per rank) and replayed, as at N = 1.
    graph = None
    g_out = None
    if exchange is not None and not args.no_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            g_out, _, _ = step()
        torch.cuda.synchronize()
        timed = graph.replay
    else:
        timed = step
    with ClockSampler(local) as clk:
        ms = time_steps(timed, args.steps, None, world)
    value = T_total / (ms * 1e-3)
    result = g_out if g_out is not None else step()[0]
    torch.cuda.synchronize()
    result = result.clone()

    # per-stage breakdown: peer-memory path from per-stage graph replays; the
    # NCCL path (host-synchronizing) from eager events at stage boundaries
    if exchange is not None:
        stages, _ = layer.p2p_stages(x, router_w, router_b, local_p)
        stage_ms = graphed_stage_ms(stages, args.steps, world)
        stage_src = "each stage replayed from its own CUDA graph, events between replays (max over ranks)"
    else:
        stage_ms = {}
        for _ in range(args.steps):
            layer.marks = []
            step()
            torch.cuda.synchronize()
            for (_, a), (name, b) in zip(layer.marks[:-1], layer.marks[1:]):
                stage_ms[name] = stage_ms.get(name, 0.0) + a.elapsed_time(b) / args.steps
        layer.marks = None
        stage_src = "eager launches, events at stage boundaries (rank 0)"

    ms_e2e = e2e_ms(lambda xin: layer(xin, router_w, router_b, local_p)[0], x, args.steps, args.warmup, world,
                    pipelined=exchange is not None)

    # parity: this rank's slice against the single-GPU layer on its tokens
    ref, _, _ = kernels.moe_forward(x, full_e["gate_up_proj_blocks"], full_e["gate_up_proj_scales"],
                                    full_e["gate_up_proj_bias"], full_e["down_proj_blocks"],
                                    full_e["down_proj_scales"], full_e["down_proj_bias"], shape.top_k,
                                    router_weight=router_w, router_bias=router_b)
    torch.cuda.synchronize()
    exact = bool(torch.equal(result, ref))
    rel = float((result.float() - ref.float()).norm() / ref.float().norm().clamp_min(1e-30))
    status = kernels.device_status(clear=True)
    flags = torch.tensor([1.0 if exact else 0.0, rel, float(status)], dtype=torch.float64, device=dev)
    worst = flags.clone()
    dist.all_reduce(worst[1:], op=dist.ReduceOp.MAX)
    dist.all_reduce(worst[:1], op=dist.ReduceOp.MIN)
    all_exact, worst_rel, worst_status = bool(worst[0] > 0.5), float(worst[1]), int(worst[2])
    parity_ok = worst_status == 0 and (all_exact or worst_rel <= 5e-3)
    parity = (("ok: every rank's output bit-identical to the single-GPU layer on its tokens" if all_exact
               else f"ok: max rel-L2 {worst_rel:.2e} against the single-GPU layer") if parity_ok
              else f"FAILED: max rel-L2 {worst_rel:.2e}, device status {worst_status}")

    stats = layer.last_stats
    peaks, peak_src = load_peaks()
    if exchange is not None:
        S_local = int(exchange.local_offsets[-1].item())
        sent = received = None
        collective = ("peer-memory exchange over NVLink (bs_ep_p2p_*: counts, rows and results stored "
                      "into the peers' buffers by the library's kernels, epoch flags, no host sync)")
    else:
        S_local = sum(stats.rows_received)
        sent, received = stats.rows_sent, stats.rows_received
        collective = "NCCL all_to_all_single (counts, dispatch rows, combine rows)"
    exp_ms = stage_ms.get("experts", 0.0)
    exp_flops = S_local * 6.0 * shape.hidden * shape.intermediate
    achieved = exp_flops / (exp_ms * 1e-3) / 1e12 if exp_ms else 0.0
    peak, plabel = tensor_peak(peaks, ms * args.steps * 1e-3)
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "parity": parity,
                "config": {"workload": args.workload, "tokens": T_total, "tokens_per_rank": Tr,
                           "experts_per_rank": shape.experts // world, "parallelism": f"ep{world}",
                           "collective": collective,
                           "l2": "inputs larger than L2 (expert weights + dispatched rows per rank)",
                           "rank0_rows_sent": sent, "rank0_rows_received": received,
                           "rank0_rows_processed": S_local, "cuda_graph": graph is not None},
                "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                             "frac": achieved / peak if peak else None, "traffic": None,
                             "kernel": "experts (gate_up + down, rank 0)",
                             "peak_source": f"{peak_src} {plabel}"},
                "layer_roofline": {"stage_ms": stage_ms, "stage_ms_source": stage_src},
                "e2e": {"value": T_total / (ms_e2e * 1e-3), "unit": "tokens/s",
                        "h2d_bytes_per_step": x.numel() * 2 * world,
                        "d2h_bytes_per_step": x.numel() * 2 * world,
                        "api": "blockstreamer_b200.expert_parallel.ExpertParallelMoE"},
                "clocks": clk.summary(), "gpu_launches": (14 if exchange is not None else 12) * args.steps}
        print(json.dumps(line), flush=True)
    del graph
    if exchange is not None:
        exchange.close()
    if not parity_ok:
        raise SystemExit(3)


# ---------------------------------------------------------------- streamed stack (config 5)

def run_bench_streamed(args, rank, world, shape, case_id, T, layers=4, zipf_s=1.2, groups=4):
    """Config 5: a stack of ``layers`` gpt-oss-120b MoE layers whose packed
    experts live in pinned host memory, T tokens in total, router bias making
    expert popularity Zipf(s) over a seeded expert permutation.

    value = T * layers / step time (tokens through one MoE layer per second,
    whole job).  The engine is blockstreamer_b200.streaming: per layer the
    router runs on resident router weights, only the experts that received
    rows are staged host->device, in ``groups`` id ranges whose grouped GEMMs
    start as each range lands.  At N > 1 every rank keeps only its E/N-expert
    slice of each layer pinned, routes T/N tokens and exchanges rows over peer
    memory (StreamedEPStack).  At N = 1 the reference's own StreamedModel
    (whole-block staging, prefetch_ahead=1) drives the same layers as
    B200GptOssMLP blocks for comparison.  After timing, every rank checks its
    output against the resident layers chained on the same tokens."""
    import types
    import torch.distributed as dist
    from blockstreamer_b200 import B200GptOssMLP
    from blockstreamer_b200.streaming import EXPERT_TENSORS, StreamedEPStack, StreamedMoEStack
    from blockstreamer_b200.synthetic import zipf_router_bias

    dev = torch.device("cuda", torch.cuda.current_device())
    if T % world or shape.experts % world:
        raise SystemExit(f"{T} tokens / {shape.experts} experts do not split over {world} ranks")
    Tr = T // world
    El = shape.experts // world
    lo, hi = rank * El, (rank + 1) * El

    def layer_state(li, device):
        p = make_layer(shape, 10 * case_id + li, device=device)
        p["router.bias"] = zipf_router_bias(shape, zipf_s, 10 * case_id + li).to(device)
        return p

    # this rank's slice of every layer in pinned host memory
    states = []
    for li in range(layers):
        p = layer_state(li, dev)
        states.append({n: (t[lo:hi] if n.startswith("experts.") else t).cpu().pin_memory()
                       for n, t in p.items()})
        del p
    torch.cuda.empty_cache()
    x_all = make_tokens(T, shape.hidden, case_id, device=dev)
    x = x_all[rank * Tr:(rank + 1) * Tr].contiguous()
    del x_all
    exchange = None
    if world == 1:
        stack = StreamedMoEStack(states, shape.top_k, dev, groups=groups)
    else:
        from blockstreamer_b200.expert_parallel import P2PExchange
        exchange = P2PExchange(None, shape.experts, shape.hidden, Tr, shape.top_k, dev)
        stack = StreamedEPStack(states, shape.top_k, exchange, groups=groups)
    for _ in range(args.warmup):
        stack(x)
    torch.cuda.synchronize()
    n0 = len(stack.stats.bytes_staged)
    with ClockSampler(torch.cuda.current_device()) as clk:
        ms = time_steps(lambda: stack(x), args.steps, None, world)
    st_bytes = stack.stats.bytes_staged[n0:]
    st_experts = stack.stats.experts_staged[n0:]
    st_rows = stack.stats.rows_local[n0:]
    h2d_per_step = sum(st_bytes) / args.steps            # this rank's weight bytes staged per step
    out = stack(x)
    torch.cuda.synchronize()

    # parity: the resident layers chained on this rank's tokens, single GPU
    ref = x
    for li in range(layers):
        p = layer_state(li, dev)
        ref, _, _ = kernels.moe_forward(ref, *[p["experts." + n] for n in EXPERT_TENSORS], shape.top_k,
                                        router_weight=p["router.weight"], router_bias=p["router.bias"])
        del p
    torch.cuda.synchronize()
    ok = bool(torch.equal(out, ref))
    del ref
    torch.cuda.empty_cache()

    # host->device copy rate of pinned memory on this box (the bound), per rank
    src = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    dst = torch.empty(1 << 30, dtype=torch.uint8, device=dev)
    barrier(world)
    h2d_gbs = -max_over_ranks(-_copy_gbs(src, dst), world)   # the slowest rank's link
    del src, dst

    # e2e: this rank's tokens in from pinned host memory, the stack's output back out
    x_host = x.cpu().pin_memory()
    out_host = torch.empty_like(x_host).pin_memory()
    x_dev = torch.empty_like(x)

    def e2e_step():
        x_dev.copy_(x_host, non_blocking=True)
        out_host.copy_(stack(x_dev), non_blocking=True)
    e2e = time_steps(e2e_step, args.steps, None, world)

    load = {"rows": sum(st_rows) // max(args.steps, 1), "experts_staged": sum(st_experts) // max(args.steps, 1),
            "staged_bytes": int(h2d_per_step), "parity": ok}
    loads = [None] * world
    if world > 1:
        dist.all_gather_object(loads, load)
    else:
        loads = [load]
    all_ok = all(l["parity"] for l in loads)

    ref_engine = None
    if world == 1 and not args.no_extra:
        ref_engine = _reference_engine_ms(args, shape, states, x, layers, dev)

    line = None
    if rank == 0:
        achieved = max(l["staged_bytes"] for l in loads) / (ms * 1e-3) / 1e9
        full_bytes = layers * El * stack.layers[0].bytes_per_expert
        line = {"metric": METRIC, "value": T * layers / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded weights, Zipf router bias)",
                "config": {"workload": args.workload, "tokens": T, "layers": layers, "zipf_s": zipf_s,
                           "parallelism": f"ep{world}" if world > 1 else "single GPU",
                           "streaming": "blockstreamer_b200.streaming (expert-granular: hit experts only, "
                                        f"{groups} id ranges whose GEMMs start as each lands, 2 device slots)",
                           "value_is": "tokens x layers / step time",
                           "l2": "inputs larger than L2 (up to 1.69 GB of weights staged per layer)"},
                "parity": "ok" if all_ok else "MISMATCH vs resident layers",
                "per_rank_load": [{"rank": r, **l} for r, l in enumerate(loads)],
                "roofline": {"bound": "host link", "achieved": achieved, "peak": h2d_gbs, "unit": "GB/s",
                             "frac": achieved / h2d_gbs, "traffic": max(l["staged_bytes"] for l in loads),
                             "kernel": "host->device weight staging per step (busiest rank, all layers)",
                             "peak_source": "measured pinned 1 GiB host->device copy on this box (slowest rank)",
                             "all_experts_bytes_per_step": full_bytes},
                "e2e": {"value": T * layers / (e2e * 1e-3), "unit": "tokens/s",
                        "h2d_bytes_per_step": x.numel() * 2 * world, "d2h_bytes_per_step": x.numel() * 2 * world,
                        "api": "blockstreamer_b200.streaming.%s" % type(stack).__name__},
                "clocks": clk.summary(),
                "gpu_launches": (sum(LAUNCHES.values()) - 2 + 2 * groups + (2 if world > 1 else 0))
                * layers * args.steps}
        if ref_engine is not None:
            line["reference_engine"] = ref_engine
    if exchange is not None:
        exchange.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if not all_ok:
        raise SystemExit(3)


def _copy_gbs(src, dst):
    st = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dst.copy_(src, non_blocking=True)
    a.record(st)
    for _ in range(3):
        dst.copy_(src, non_blocking=True)
    b.record(st)
    torch.cuda.synchronize()
    return 3 * src.numel() / (a.elapsed_time(b) * 1e-3) / 1e9


def _reference_engine_ms(args, shape, states, x, layers, dev):
    """The same layers as B200GptOssMLP blocks driven by the reference's own
    StreamedModel (whole-block staging, prefetch_ahead=1), for comparison."""
    import types
    ref_dir = os.path.join(REPO, "baseline", "_ref")
    if not os.path.exists(os.path.join(ref_dir, "streamer.py")):
        return {"unavailable": "the reference package is not installed under baseline/_ref"}
    sys.path.insert(0, ref_dir)
    from streamer import StreamedModel  # the reference's own streaming engine
    from blockstreamer_b200 import B200GptOssMLP
    cfg = types.SimpleNamespace(hidden_size=shape.hidden, intermediate_size=shape.intermediate,
                                num_local_experts=shape.experts, num_experts_per_tok=shape.top_k,
                                swiglu_limit=7.0)
    blocks = []
    for s in states:
        mlp = B200GptOssMLP(cfg)
        mlp.load_state_dict(s, strict=True, assign=True)
        blocks.append(mlp)
    model = StreamedModel(blocks, device=dev, prefetch_ahead=1, dtype=None)
    xs = x.view(1, *x.shape)
    for _ in range(args.warmup):
        model(xs)
    torch.cuda.synchronize()
    b0 = model.stats()["transfer_bytes"]
    ms = time_steps(lambda: model(xs), args.steps, None, 1)
    h2d = (model.stats()["transfer_bytes"] - b0) / args.steps
    model.close()
    return {"engine": "reference StreamedModel (baseline/_ref/streamer.py), prefetch_ahead=1, whole-block staging",
            "ms_per_step": ms, "value": x.shape[0] * layers / (ms * 1e-3), "unit": "tokens/s",
            "h2d_bytes_per_step": h2d}


def run_trace(args):
    """One step of the workload under torch.profiler (CPU + CUDA activity), the
    role of the reference's trace export (benchmark.py:153-174): the chrome
    trace goes to DIR/trace.json, and a summary (kernels by total time, copies,
    and how long copies and kernels ran at the same time) is printed."""
    from blockstreamer_b200.streaming import EXPERT_TENSORS, StreamedMoEStack
    from blockstreamer_b200.synthetic import zipf_router_bias
    key, case_id, T = parse_workload(args.workload)
    shape = CASES[key]
    dev = torch.device("cuda", 0)
    os.makedirs(args.trace, exist_ok=True)
    if case_id == 5:      # the streamed stack (2 layers keep the trace small)
        states = []
        for li in range(2):
            p = make_layer(shape, 10 * case_id + li, device=dev)
            p["router.bias"] = zipf_router_bias(shape, 1.2, 10 * case_id + li).to(dev)
            states.append({n: t.cpu().pin_memory() for n, t in p.items()})
            del p
        stack = StreamedMoEStack(states, shape.top_k, dev)
        x = make_tokens(T, shape.hidden, case_id, device=dev)
        step = lambda: stack(x)
        what = "blockstreamer_b200.streaming.StreamedMoEStack, 2 layers"
    else:
        p = make_layer(shape, case_id, device=dev)
        x = make_tokens(T, shape.hidden, case_id, device=dev)
        w = [p["experts." + n] for n in EXPERT_TENSORS]
        step = lambda: kernels.moe_forward(x, *w, shape.top_k, router_weight=p["router.weight"],
                                           router_bias=p["router.bias"])
        what = "kernels.moe_forward -> bs_moe_forward, one layer, eager"
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    acts = [torch.profiler.ProfilerActivity.CPU, torch.profiler.ProfilerActivity.CUDA]
    with torch.profiler.profile(activities=acts) as prof:
        step()
        torch.cuda.synchronize()
    path = os.path.join(args.trace, "trace.json")
    prof.export_chrome_trace(path)
    with open(path) as f:
        events = json.load(f)["traceEvents"]
    kern = [e for e in events if e.get("cat") == "kernel"]
    copies = [e for e in events if e.get("cat") in ("gpu_memcpy", "gpu_memset")]
    by_name = {}
    for e in kern:
        n = e["name"].replace("(anonymous namespace)::", "").split("(")[0]
        c, d = by_name.get(n, (0, 0.0))
        by_name[n] = (c + 1, d + float(e["dur"]))

    def spans(evs):
        return sorted((float(e["ts"]), float(e["ts"]) + float(e["dur"])) for e in evs)

    def union(iv):
        out = []
        for a, b in iv:
            if out and a <= out[-1][1]:
                out[-1][1] = max(out[-1][1], b)
            else:
                out.append([a, b])
        return out

    ku, cu = union(spans(kern)), union(spans(copies))
    both = 0.0
    i = j = 0
    while i < len(ku) and j < len(cu):
        lo, hi = max(ku[i][0], cu[j][0]), min(ku[i][1], cu[j][1])
        both += max(0.0, hi - lo)
        if ku[i][1] < cu[j][1]:
            i += 1
        else:
            j += 1
    allv = spans(kern + copies)
    summary = {"workload": args.workload, "what": what, "trace": path,
               "gpu_activity": bool(kern), "span_us": (allv[-1][1] - allv[0][0]) if allv else 0.0,
               "kernel_busy_us": sum(b - a for a, b in ku), "copy_busy_us": sum(b - a for a, b in cu),
               "copy_and_kernel_overlap_us": both, "copies": len(copies),
               "kernels": [{"name": n, "launches": c, "total_us": round(d, 1)}
                           for n, (c, d) in sorted(by_name.items(), key=lambda kv: -kv[1][1])]}
    print(json.dumps(summary), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD)
    ap.add_argument("--algo", choices=sorted(ALGOS), default="auto")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="default workload: skip measuring configs 2 and 3 in the same run")
    ap.add_argument("--no-graph", action="store_true", help="launch every step eagerly")
    ap.add_argument("--ep-transport", choices=["p2p", "nccl"], default="p2p",
                    help="N > 1: exchange rows over peer memory (library kernels) or NCCL all-to-all")
    ap.add_argument("--trace", metavar="DIR", default=None,
                    help="instead of timing: profile one step of the workload with torch.profiler, write "
                         "DIR/trace.json and print a summary of its GPU activity (1 GPU)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.trace:
        return run_trace(args)
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        return run_reference(args, rank, world)
    rank, world, local = dist_setup(args.gpus)
    try:
        run_ours(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
