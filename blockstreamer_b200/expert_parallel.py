"""Expert-parallel gpt-oss MoE layer over torch.distributed (NCCL on GPUs).

The reference runs every expert on one GPU (BlockStreamer has no distributed
backend, README.md:22-30).  The layer shards naturally by expert: with R ranks,
rank r owns experts [r*E/R, (r+1)*E/R) (slices along dim 0 of every
``experts.*`` tensor, as ``block_streamer/adapters.py:33-56`` slices fused
experts) and its own share of the tokens.  One forward:

1. router on the local tokens (router weights replicated);
2. dispatch by GLOBAL expert id, so the rows bound for each destination rank
   are contiguous and, within it, grouped by expert;
3. all-to-all of the per-expert row counts (int32), then one device->host copy
   of the per-rank row totals (NCCL's uneven all-to-all takes host split sizes);
4. all-to-all of the permuted rows (bf16);
5. regroup the received [source][expert] segments into expert-major order;
6. local grouped gate_up + SwiGLU and down on the rank's experts;
7. gather back to [source][expert] order and reverse all-to-all;
8. local weighted combine (fp32 sum, one bf16 rounding).

The exchange is the only collective; each rank's kernels are the single-GPU
ones.  ``ops`` abstracts the per-rank compute so that the orchestration can be
checked with CPU ranks (gloo) against a single-process evaluation.

On GPUs the exchange can instead run over peer memory (``P2PExchange``,
``bs_ep_p2p_*``): each rank's rows are stored straight into the destination
rank's buffer in the expert-major order its grouped GEMMs read, and each
result straight back into its source's buffer in dispatch order, by the
library's own kernels with epoch flags -- no host synchronization (NCCL's
uneven all-to-all needs the split sizes on the host), no regroup or ungroup
pass, no library collective on the data path.
"""

from __future__ import annotations

import contextlib
import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _lib, kernels


@contextlib.contextmanager
def nvtx(name: str):
    """An NVTX range around one stage's launches (seen by nsys / ncu; no cost
    without a profiler attached)."""
    if torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


class CudaOps:
    """Per-rank compute on the library's sm_100a kernels."""

    def __init__(self, algo: int = kernels.ALGO_AUTO):
        self.algo = algo

    def router(self, x, weight, bias, top_k):
        _, sc, idx = kernels.router(x, weight, bias, top_k, index_dtype=torch.int32)
        return sc, idx

    def dispatch(self, idx, num_experts, x):
        d = kernels.dispatch(idx, num_experts, x)
        return d.expert_offsets, d.row_of_slot, d.x_perm

    def regroup(self, recv_counts, x_recv):
        return kernels.ep_regroup(recv_counts, x_recv)

    def experts(self, x_grouped, offsets, p, alpha, limit):
        h = kernels.moe_gate_up(x_grouped, offsets, p["gate_up_proj_blocks"], p["gate_up_proj_scales"],
                                p["gate_up_proj_bias"], alpha=alpha, limit=limit, algo=self.algo)
        return kernels.moe_down(h, offsets, p["down_proj_blocks"], p["down_proj_scales"],
                                p["down_proj_bias"], algo=self.algo)

    def ungroup(self, y_grouped, row_map):
        return kernels.gather_rows(y_grouped, row_map)

    def combine(self, y, row_of_slot, scores, num_tokens):
        return kernels.combine(y, row_of_slot, scores, num_tokens)


def shard_experts(params: dict, rank: int, world: int) -> dict:
    """This rank's contiguous slice of every expert tensor (dim 0)."""
    out = {}
    for name, t in params.items():
        E = t.shape[0]
        if E % world:
            raise ValueError(f"{E} experts do not split over {world} ranks")
        el = E // world
        out[name] = t[rank * el:(rank + 1) * el].contiguous()
    return out


class _DeviceBytes:
    """A raw device allocation seen by torch (zero-copy, __cuda_array_interface__)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


class P2PExchange:
    """One rank's peer-memory exchange buffer and its peers' mappings.

    Collective over ``group``: every rank constructs it with the same
    arguments.  ``max_tokens`` bounds the tokens a rank dispatches per call;
    the receive area holds every rank's rows (R * max_tokens * top_k), so no
    routing can overflow it."""

    def __init__(self, group, num_experts: int, hidden: int, max_tokens: int, top_k: int, device):
        self.group = group
        self.R = dist.get_world_size(group)
        self.me = dist.get_rank(group)
        self.E, self.H, self.k = num_experts, hidden, top_k
        self.src_rows = max_tokens * top_k
        self.cap = self.R * self.src_rows
        self.device = torch.device(device)
        lib = _lib.load()
        nbytes = lib.bs_ep_p2p_bytes(self.R, self.E, self.H, self.cap, self.src_rows)
        base, handle = ctypes.c_void_p(), (ctypes.c_char * 64)()
        with torch.cuda.device(self.device):
            _lib.call("bs_ep_p2p_alloc", nbytes, ctypes.byref(base), handle)
        self.base = base.value
        handles = [None] * self.R
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.peers = []
        with torch.cuda.device(self.device):
            for s, hs in enumerate(handles):
                if s == self.me:
                    self.peers.append(self.base)
                    continue
                pb = ctypes.c_void_p()
                _lib.call("bs_ep_p2p_open", ctypes.create_string_buffer(hs, 64), ctypes.byref(pb))
                self.peers.append(pb.value)
        self.bases = torch.tensor(self.peers, dtype=torch.int64, device=self.device)
        ro, yo = ctypes.c_size_t(), ctypes.c_size_t()
        _lib.call("bs_ep_p2p_layout", self.R, self.E, self.H, self.cap, self.src_rows, ctypes.byref(ro),
                  ctypes.byref(yo))
        raw = torch.as_tensor(_DeviceBytes(self.base, nbytes), device=self.device)
        self.recv = raw[ro.value: ro.value + self.cap * self.H * 2].view(torch.bfloat16).view(self.cap, self.H)
        self.yback = raw[yo.value: yo.value + self.src_rows * self.H * 2].view(torch.bfloat16).view(
            self.src_rows, self.H)
        self.local_offsets = torch.zeros(self.E // self.R + 1, dtype=torch.int32, device=self.device)
        self._closed = False

    def dispatch(self, x: torch.Tensor, expert_offsets: torch.Tensor, token_of_row: torch.Tensor):
        """Send this rank's rows (stream-ordered, no host sync; capturable in a CUDA graph)."""
        with torch.cuda.device(self.device):
            _lib.call("bs_ep_p2p_dispatch", x.data_ptr(), self.H, expert_offsets.data_ptr(),
                      token_of_row.data_ptr(), self.base, self.bases.data_ptr(), self.R, self.E, self.me,
                      self.cap, self.src_rows, self.local_offsets.data_ptr(),
                      torch.cuda.current_stream(self.device).cuda_stream)

    def give_back(self, y: torch.Tensor):
        with torch.cuda.device(self.device):
            _lib.call("bs_ep_p2p_return", y.data_ptr(), self.H, self.base, self.bases.data_ptr(), self.R,
                      self.E, self.me, self.cap, self.src_rows,
                      torch.cuda.current_stream(self.device).cuda_stream)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def close(self):
        """Collective: unmap the peers, then free this rank's buffer."""
        if self._closed:
            return
        self._closed = True
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for s, pb in enumerate(self.peers):
                if s != self.me:
                    _lib.call("bs_ep_p2p_close", pb)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            _lib.call("bs_ep_p2p_free", self.base)


@dataclass
class EPStats:
    rows_sent: list
    rows_received: list


class ExpertParallelMoE:
    """One gpt-oss MoE layer sharded by expert over a process group."""

    def __init__(self, num_experts: int, top_k: int, group=None, ops=None,
                 alpha: float = kernels.ALPHA, limit: float = kernels.LIMIT,
                 exchange: P2PExchange | None = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not split over {self.world} ranks")
        self.E = num_experts
        self.El = num_experts // self.world
        self.top_k = top_k
        self.ops = ops if ops is not None else CudaOps()
        self.alpha, self.limit = alpha, limit
        self.last_stats: EPStats | None = None
        # peer-memory exchange (GPUs); None: NCCL / gloo all-to-all
        self.exchange = exchange
        self._h = self._y = None
        # optional: a list that receives (stage name, CUDA event) at stage ends
        self.marks: list | None = None

    def _mark(self, name):
        if self.marks is not None and torch.cuda.is_available():
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.marks.append((name, ev))

    def forward(self, x: torch.Tensor, router_weight: torch.Tensor, router_bias: torch.Tensor,
                local_experts: dict):
        """x: this rank's tokens [T_r, H].  ``local_experts`` holds this rank's
        slice of the six expert tensors (names without the ``experts.`` prefix).
        Returns (out [T_r, H], scores [T_r, k], indices [T_r, k] global)."""
        if self.exchange is not None:
            return self._forward_p2p(x, router_weight, router_bias, local_experts)
        R, El, k = self.world, self.El, self.top_k
        T, H = x.shape
        ops = self.ops
        self._mark("start")
        sc, idx = ops.router(x, router_weight, router_bias, k)
        self._mark("router")
        offsets, row_of_slot, x_perm = ops.dispatch(idx, self.E, x)
        self._mark("dispatch")
        counts = (offsets[1:] - offsets[:-1]).to(torch.int32).contiguous()       # [E], by destination
        recv_counts = torch.empty_like(counts)
        dist.all_to_all_single(recv_counts, counts, group=self.group)         # [R * El], source-major
        sizes = torch.cat([counts.view(R, El).sum(1), recv_counts.view(R, El).sum(1)]).cpu().tolist()
        send_rows, recv_rows = sizes[:R], sizes[R:]
        x_recv = torch.empty(sum(recv_rows), H, dtype=x.dtype, device=x.device)
        dist.all_to_all_single(x_recv, x_perm[: sum(send_rows)].contiguous(), recv_rows, send_rows,
                               group=self.group)
        self._mark("all_to_all_dispatch")
        if x_recv.shape[0]:
            x_grouped, loc_off, row_map = ops.regroup(recv_counts.view(R, El), x_recv)
            self._mark("regroup")
            y_grouped = ops.experts(x_grouped, loc_off, local_experts, self.alpha, self.limit)
            self._mark("experts")
            y_recv = ops.ungroup(y_grouped, row_map)
            self._mark("ungroup")
        else:
            y_recv = x_recv
        y_back = torch.empty(T * k, H, dtype=x.dtype, device=x.device)
        dist.all_to_all_single(y_back, y_recv, send_rows, recv_rows, group=self.group)
        self._mark("all_to_all_combine")
        out = ops.combine(y_back, row_of_slot, sc, T)
        self._mark("combine")
        self.last_stats = EPStats(send_rows, recv_rows)
        return out, sc, idx

    def _forward_p2p(self, x, router_weight, router_bias, p):
        ex, k = self.exchange, self.top_k
        T, H = x.shape
        if T * k > ex.src_rows:
            raise ValueError(f"{T} tokens exceed the exchange's {ex.src_rows // k} per rank")
        self._mark("start")
        with nvtx("ep.router"):
            sc, idx = self.ops.router(x, router_weight, router_bias, k)
        self._mark("router")
        with nvtx("ep.dispatch"):
            d = kernels.dispatch(idx, self.E)
        self._mark("dispatch")
        with nvtx("ep.exchange_dispatch"):
            ex.dispatch(x, d.expert_offsets, d.token_of_row)
        self._mark("exchange_dispatch")
        if self._h is None:
            I = p["gate_up_proj_blocks"].shape[1] // 2
            self._h = torch.empty(ex.cap, I, dtype=torch.bfloat16, device=x.device)
            self._y = torch.empty(ex.cap, H, dtype=torch.bfloat16, device=x.device)
        algo = getattr(self.ops, "algo", kernels.ALGO_AUTO)
        with nvtx("ep.experts"):
            kernels.moe_gate_up(ex.recv, ex.local_offsets, p["gate_up_proj_blocks"], p["gate_up_proj_scales"],
                                p["gate_up_proj_bias"], alpha=self.alpha, limit=self.limit, algo=algo,
                                out=self._h)
            kernels.moe_down(self._h, ex.local_offsets, p["down_proj_blocks"], p["down_proj_scales"],
                             p["down_proj_bias"], algo=algo, out=self._y)
        self._mark("experts")
        with nvtx("ep.exchange_combine"):
            ex.give_back(self._y)
        self._mark("exchange_combine")
        with nvtx("ep.combine"):
            out = kernels.combine(ex.yback[: T * k], d.row_of_slot, sc, T)
        self._mark("combine")
        return out, sc, idx

    def p2p_stages(self, x, router_weight, router_bias, p):
        """The peer-memory layer as ordered (stage name, callable) pairs with
        every buffer allocated once: calling them in order is one layer call
        (the same kernels as ``forward``), and each can be captured in a CUDA
        graph of its own to time the stages.  Returns (stages, out)."""
        ex, k, E = self.exchange, self.top_k, self.E
        if ex is None:
            raise ValueError("p2p_stages needs the peer-memory exchange")
        T, H = x.shape
        dev = x.device
        I = p["gate_up_proj_blocks"].shape[1] // 2
        lib = _lib.load()
        sc = torch.empty(T, k, dtype=torch.float32, device=dev)
        idx = torch.empty(T, k, dtype=torch.int32, device=dev)
        rws = torch.empty(max(lib.bs_router_workspace_bytes(T, H, E, _lib.BS_F32), 16), dtype=torch.uint8,
                          device=dev)
        d = kernels.Dispatch(torch.empty(E + 1, dtype=torch.int32, device=dev),
                             torch.empty(T * k, dtype=torch.int32, device=dev),
                             torch.empty(T * k, dtype=torch.int32, device=dev), None)
        dws = torch.empty(max(lib.bs_dispatch_workspace_bytes(T, k, E), 16), dtype=torch.uint8, device=dev)
        h = torch.empty(ex.cap, I, dtype=torch.bfloat16, device=dev)
        y = torch.empty(ex.cap, H, dtype=torch.bfloat16, device=dev)
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        algo = getattr(self.ops, "algo", kernels.ALGO_AUTO)

        def router():
            kernels.router(x, router_weight, router_bias, k, out_scores=sc, out_indices=idx, workspace=rws)

        def dispatch():
            kernels.dispatch(idx, E, out=d, workspace=dws)

        def exchange_dispatch():
            ex.dispatch(x, d.expert_offsets, d.token_of_row)

        def experts():
            kernels.moe_gate_up(ex.recv, ex.local_offsets, p["gate_up_proj_blocks"], p["gate_up_proj_scales"],
                                p["gate_up_proj_bias"], alpha=self.alpha, limit=self.limit, algo=algo, out=h)
            kernels.moe_down(h, ex.local_offsets, p["down_proj_blocks"], p["down_proj_scales"],
                             p["down_proj_bias"], algo=algo, out=y)

        def exchange_combine():
            ex.give_back(y)

        def combine():
            kernels.combine(ex.yback[: T * k], d.row_of_slot, sc, T, out=out)

        return [("router", router), ("dispatch", dispatch), ("exchange_dispatch", exchange_dispatch),
                ("experts", experts), ("exchange_combine", exchange_combine), ("combine", combine)], out

    __call__ = forward
