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
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import kernels


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


@dataclass
class EPStats:
    rows_sent: list
    rows_received: list


class ExpertParallelMoE:
    """One gpt-oss MoE layer sharded by expert over a process group."""

    def __init__(self, num_experts: int, top_k: int, group=None, ops=None,
                 alpha: float = kernels.ALPHA, limit: float = kernels.LIMIT):
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

    __call__ = forward
