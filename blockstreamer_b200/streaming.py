"""Expert-granular weight streaming for MoE layers whose packed experts live in
pinned host memory.

The reference streams whole blocks: ``StreamedModel`` copies every parameter
of block i + 1 host->device while block i computes (streamer.py:108-149, the
pinned ring of block_streamer/diskpool.py:25-47,145-180).  For an MoE layer
that moves every expert's 13.2 MB (gpt-oss-120b) even when the router sends
it no token, and no expert GEMM can start before the whole block has landed.

Here the unit of staging is the expert:

* the router and the dispatch run on the layer's resident router weights
  (1.5 MB), and the host reads the per-expert row counts -- the one host
  synchronization per layer;
* only experts with rows are copied (``hit_only``), runs of consecutive expert
  ids as one copy per tensor, on a copy stream of their own;
* the hit experts are cut into ``groups`` contiguous id ranges of about equal
  bytes; an event after each range's copies lets the grouped GEMMs of range g
  run on the compute stream while range g + 1 is still crossing the host link;
* two device slots alternate between layers, so layer l + 1's copies never
  overwrite weights that layer l's GEMMs still read (an event recorded after
  a slot's last GEMM gates its next copy).

Unused experts keep whatever an earlier layer left in their slot: they own no
rows, so no kernel reads them.  ``StreamedEPStack`` is the same over expert
parallelism: each rank keeps only its slice of every layer pinned and stages
the experts of that slice that received rows from any rank.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import kernels

EXPERT_TENSORS = ("gate_up_proj_blocks", "gate_up_proj_scales", "gate_up_proj_bias",
                  "down_proj_blocks", "down_proj_scales", "down_proj_bias")


def plan_groups(hit: list[int], groups: int) -> list[tuple[int, int, list[tuple[int, int]]]]:
    """Cut the ascending expert ids ``hit`` into at most ``groups`` contiguous
    id ranges holding about the same number of experts (every expert stages
    the same bytes).  Returns (first id, one past the last id, runs) per range,
    where runs are the [a, b) spans of consecutive hit ids inside it, each
    copied as one slice per tensor."""
    if groups < 1:
        raise ValueError("plan_groups: groups must be >= 1")
    hit = sorted(set(int(e) for e in hit))
    n = len(hit)
    if n == 0:
        return []
    groups = min(groups, n)
    out = []
    for g in range(groups):
        members = hit[(g * n) // groups:((g + 1) * n) // groups]
        runs = []
        for e in members:
            if runs and runs[-1][1] == e:
                runs[-1][1] = e + 1
            else:
                runs.append([e, e + 1])
        out.append((members[0], members[-1] + 1, [(a, b) for a, b in runs]))
    return out


def _pinned(t: torch.Tensor) -> torch.Tensor:
    t = t.detach().contiguous()
    if t.device.type != "cpu":
        t = t.cpu()
    return t if t.is_pinned() else t.pin_memory()


class HostLayer:
    """One MoE layer: router weights resident on the device, the six packed
    expert tensors ([E, ...], checkpoint names without the ``experts.``
    prefix) pinned in host memory."""

    def __init__(self, state: dict[str, torch.Tensor], device, expert_slice: tuple[int, int] | None = None):
        self.router_weight = state["router.weight"].to(device)
        self.router_bias = state["router.bias"].to(device)
        lo, hi = expert_slice if expert_slice is not None else (0, state["experts." + EXPERT_TENSORS[0]].shape[0])
        self.experts = {n: _pinned(state["experts." + n][lo:hi]) for n in EXPERT_TENSORS}
        self.num_local = hi - lo
        self.bytes_per_expert = sum(t[0].numel() * t.element_size() for t in self.experts.values())


@dataclass
class StageStats:
    experts_staged: list = field(default_factory=list)   # per layer call
    bytes_staged: list = field(default_factory=list)
    rows_local: list = field(default_factory=list)       # rows this rank's experts computed


class ExpertStager:
    """Device slots for one layer's expert tensors and the copy stream that
    fills them from a ``HostLayer``."""

    def __init__(self, like: HostLayer, device, slots: int = 2):
        self.device = torch.device(device)
        self.slots = [{n: torch.empty(t.shape, dtype=t.dtype, device=self.device)
                       for n, t in like.experts.items()} for _ in range(slots)]
        self._free = [None] * slots
        self.copy_stream = torch.cuda.Stream(self.device)

    def stage(self, layer: HostLayer, hit: list[int], groups: int, slot: int):
        """Queue the copies of experts ``hit`` of ``layer`` into ``slot``;
        returns [(first id, end id, event)] per range and the bytes queued."""
        dst = self.slots[slot]
        plan = plan_groups(hit, groups)
        ranges, nbytes = [], 0
        with torch.cuda.stream(self.copy_stream):
            if self._free[slot] is not None:
                self.copy_stream.wait_event(self._free[slot])
            for e0, e1, runs in plan:
                for a, b in runs:
                    for n, src in layer.experts.items():
                        dst[n][a:b].copy_(src[a:b], non_blocking=True)
                    nbytes += (b - a) * layer.bytes_per_expert
                ev = torch.cuda.Event()
                ev.record(self.copy_stream)
                ranges.append((e0, e1, ev))
        return ranges, nbytes

    def release(self, slot: int):
        """Record, on the current (compute) stream, the end of ``slot``'s reads."""
        ev = torch.cuda.Event()
        ev.record()
        self._free[slot] = ev


def _grouped_experts(x_rows, offsets, w, ranges, h, y, alpha, limit, algo):
    """gate_up + SwiGLU and down over each staged id range once its copies landed."""
    cur = torch.cuda.current_stream()
    for e0, e1, ev in ranges:
        cur.wait_event(ev)
        off = offsets[e0:e1 + 1]
        kernels.moe_gate_up(x_rows, off, w["gate_up_proj_blocks"][e0:e1], w["gate_up_proj_scales"][e0:e1],
                            w["gate_up_proj_bias"][e0:e1], alpha=alpha, limit=limit, algo=algo, out=h)
        kernels.moe_down(h, off, w["down_proj_blocks"][e0:e1], w["down_proj_scales"][e0:e1],
                         w["down_proj_bias"][e0:e1], algo=algo, out=y)


class StreamedMoEStack:
    """A stack of MoE layers (each layer's output feeds the next) whose
    experts stream from pinned host memory, one GPU."""

    def __init__(self, states: list[dict], top_k: int, device, groups: int = 4, hit_only: bool = True,
                 alpha: float = kernels.ALPHA, limit: float = kernels.LIMIT, algo: int = kernels.ALGO_AUTO):
        self.device = torch.device(device)
        self.layers = [HostLayer(s, self.device) for s in states]
        self.k, self.groups, self.hit_only = top_k, groups, hit_only
        self.alpha, self.limit, self.algo = alpha, limit, algo
        self.E = self.layers[0].num_local
        self.stager = ExpertStager(self.layers[0], self.device)
        self.stats = StageStats()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        T = x.shape[0]
        for li, layer in enumerate(self.layers):
            slot = li % len(self.stager.slots)
            with torch.cuda.nvtx.range(f"stream.layer{li}.route"):
                sc, idx = kernels.router(x, layer.router_weight, layer.router_bias, self.k,
                                         index_dtype=torch.int32)[1:]
                d = kernels.dispatch(idx, self.E, x)
                off = d.expert_offsets.cpu()                                   # host sync
                counts = off[1:] - off[:-1]
            hit = [e for e in range(self.E) if counts[e] > 0] if self.hit_only else list(range(self.E))
            with torch.cuda.nvtx.range(f"stream.layer{li}.stage"):
                ranges, nbytes = self.stager.stage(layer, hit, self.groups, slot)
            S, H = d.x_perm.shape
            I = layer.experts["gate_up_proj_blocks"].shape[1] // 2
            h = torch.empty(S, I, dtype=torch.bfloat16, device=self.device)
            y = torch.empty(S, H, dtype=torch.bfloat16, device=self.device)
            with torch.cuda.nvtx.range(f"stream.layer{li}.experts"):
                _grouped_experts(d.x_perm, d.expert_offsets, self.stager.slots[slot], ranges, h, y,
                                 self.alpha, self.limit, self.algo)
            self.stager.release(slot)
            x = kernels.combine(y, d.row_of_slot, sc, T)
            self.stats.experts_staged.append(len(hit))
            self.stats.bytes_staged.append(nbytes)
            self.stats.rows_local.append(S)
        return x

    __call__ = forward


class StreamedEPStack:
    """The streamed stack over expert parallelism: rank r keeps experts
    [r E/R, (r+1) E/R) of every layer pinned, routes its own tokens, exchanges
    rows over peer memory (``expert_parallel.P2PExchange``), stages the
    experts of its slice that received rows from any rank, computes them and
    returns the rows.  Collective: every rank calls ``forward`` in step.

    ``states``: per layer, the router tensors and either the layer's full
    expert tensors ([E, ...], sliced here) or only this rank's slice
    ([E/R, ...], as a rank that pins nothing else holds them)."""

    def __init__(self, states: list[dict], top_k: int, exchange, groups: int = 4, hit_only: bool = True,
                 alpha: float = kernels.ALPHA, limit: float = kernels.LIMIT, algo: int = kernels.ALGO_AUTO):
        self.ex = exchange
        self.device = exchange.device
        R, me, E = exchange.R, exchange.me, exchange.E
        self.El = E // R
        self.layers = []
        for st in states:
            rows = st["experts." + EXPERT_TENSORS[0]].shape[0]
            if rows == E:
                sl = (me * self.El, (me + 1) * self.El)
            elif rows == self.El:
                sl = None
            else:
                raise ValueError(f"StreamedEPStack: {rows} experts per layer is neither {E} nor this rank's {self.El}")
            self.layers.append(HostLayer(st, self.device, expert_slice=sl))
        self.k, self.groups, self.hit_only = top_k, groups, hit_only
        self.alpha, self.limit, self.algo = alpha, limit, algo
        self.E = E
        self.stager = ExpertStager(self.layers[0], self.device)
        I = self.layers[0].experts["gate_up_proj_blocks"].shape[1] // 2
        self.h = torch.empty(exchange.cap, I, dtype=torch.bfloat16, device=self.device)
        self.y = torch.empty(exchange.cap, exchange.H, dtype=torch.bfloat16, device=self.device)
        self.stats = StageStats()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        ex, T = self.ex, x.shape[0]
        for li, layer in enumerate(self.layers):
            slot = li % len(self.stager.slots)
            with torch.cuda.nvtx.range(f"stream_ep.layer{li}.route"):
                sc, idx = kernels.router(x, layer.router_weight, layer.router_bias, self.k,
                                         index_dtype=torch.int32)[1:]
                d = kernels.dispatch(idx, self.E)
            with torch.cuda.nvtx.range(f"stream_ep.layer{li}.exchange_dispatch"):
                ex.dispatch(x, d.expert_offsets, d.token_of_row)
                loc = ex.local_offsets.cpu()                                   # host sync
            counts = (loc[1:] - loc[:-1]).tolist()
            hit = [e for e in range(self.El) if counts[e] > 0] if self.hit_only else list(range(self.El))
            with torch.cuda.nvtx.range(f"stream_ep.layer{li}.stage"):
                ranges, nbytes = self.stager.stage(layer, hit, self.groups, slot)
            with torch.cuda.nvtx.range(f"stream_ep.layer{li}.experts"):
                _grouped_experts(ex.recv, ex.local_offsets, self.stager.slots[slot], ranges, self.h, self.y,
                                 self.alpha, self.limit, self.algo)
            self.stager.release(slot)
            with torch.cuda.nvtx.range(f"stream_ep.layer{li}.exchange_combine"):
                ex.give_back(self.y)
            x = kernels.combine(ex.yback[: T * self.k], d.row_of_slot, sc, T)
            self.stats.experts_staged.append(len(hit))
            self.stats.bytes_staged.append(nbytes)
            self.stats.rows_local.append(int(loc[-1]))
        return x

    __call__ = forward
