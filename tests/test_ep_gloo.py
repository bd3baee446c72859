"""Expert-parallel orchestration on CPU ranks (gloo): counts exchange, uneven
all-to-all split sizes, regroup/ungroup orderings and the combine must give the
same layer output as a single-process evaluation.  The per-rank compute is
restated on the CPU (oracle math); the CUDA kernels behind the same interface
are exercised on GPUs by bench.py --gpus N."""

import datetime
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from blockstreamer_b200.expert_parallel import ExpertParallelMoE, shard_experts
from blockstreamer_b200.synthetic import LayerShape, make_layer, make_tokens
from oracle import moe as omoe


class CpuOps:
    """The per-rank steps on the CPU (test reference for the orchestration)."""

    def router(self, x, w, b, k):
        _, sc, idx = omoe.router(x.float(), w, b, k)
        return sc, idx.to(torch.int32)

    def dispatch(self, idx, E, x):
        k = idx.shape[1]
        flat = idx.reshape(-1).long()
        order = torch.sort(flat, stable=True).indices
        offsets = torch.zeros(E + 1, dtype=torch.int32)
        offsets[1:] = torch.cumsum(torch.bincount(flat, minlength=E), 0)
        row_of_slot = torch.empty_like(order, dtype=torch.int32)
        row_of_slot[order] = torch.arange(order.numel(), dtype=torch.int32)
        return offsets, row_of_slot, x[order // k]

    def regroup(self, recv_counts, x_recv):
        R, El = recv_counts.shape
        c = recv_counts.long()
        seg = torch.cumsum(torch.cat([torch.zeros(1, dtype=torch.long), c.reshape(-1)]), 0)
        eo = torch.cat([torch.zeros(1, dtype=torch.long), torch.cumsum(c.sum(0), 0)])
        row_map = torch.empty(x_recv.shape[0], dtype=torch.long)
        for s in range(R):
            for e in range(El):
                n = int(c[s, e])
                start = int(seg[s * El + e])
                dst = int(eo[e] + c[:s, e].sum())
                row_map[start:start + n] = torch.arange(dst, dst + n)
        xg = torch.empty_like(x_recv)
        xg[row_map] = x_recv
        return xg, eo.to(torch.int32), row_map

    def experts(self, xg, offsets, p, alpha, limit):
        y = torch.empty(xg.shape[0], p["down_proj_blocks"].shape[1], dtype=torch.float32)
        for e in range(offsets.numel() - 1):
            a, b = int(offsets[e]), int(offsets[e + 1])
            if a == b:
                continue
            wgu = omoe.dequant_expert(p["gate_up_proj_blocks"][e], p["gate_up_proj_scales"][e], torch.float32)
            g = xg[a:b].float() @ wgu + p["gate_up_proj_bias"][e].float()
            gate, up = g[:, ::2].clamp(max=limit), g[:, 1::2].clamp(-limit, limit)
            h = (up + 1) * gate * torch.sigmoid(alpha * gate)
            wd = omoe.dequant_expert(p["down_proj_blocks"][e], p["down_proj_scales"][e], torch.float32)
            y[a:b] = h @ wd + p["down_proj_bias"][e].float()
        return y

    def ungroup(self, yg, row_map):
        return yg[row_map]

    def combine(self, y, row_of_slot, sc, T):
        k = sc.shape[1]
        return (y[row_of_slot.long()].reshape(T, k, -1) * sc[..., None]).sum(1)


SHAPE = LayerShape(128, 128, 8, 2, 124, 130)
T_TOTAL = 48


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        p = make_layer(SHAPE, 9)
        x = make_tokens(T_TOTAL, SHAPE.hidden, 9).float()
        Tr = T_TOTAL // world
        local = shard_experts({k.split(".", 1)[1]: v for k, v in p.items() if k.startswith("experts.")},
                              rank, world)
        layer = ExpertParallelMoE(SHAPE.experts, SHAPE.top_k, ops=CpuOps())
        out, sc, idx = layer(x[rank * Tr:(rank + 1) * Tr], p["router.weight"], p["router.bias"], local)
        q.put((rank, out, layer.last_stats.rows_sent, layer.last_stats.rows_received))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, traceback.format_exc(), None, None))


def _reference():
    p = make_layer(SHAPE, 9)
    x = make_tokens(T_TOTAL, SHAPE.hidden, 9).float()
    ops = CpuOps()
    sc, idx = ops.router(x, p["router.weight"], p["router.bias"], SHAPE.top_k)
    pe = {k.split(".", 1)[1]: v for k, v in p.items() if k.startswith("experts.")}
    offsets, ros, xp = ops.dispatch(idx, SHAPE.experts, x)
    y = ops.experts(xp, offsets, pe, 1.702, 7.0)
    return ops.combine(y, ros, sc, T_TOTAL)


@pytest.mark.parametrize("world", [2, 4])
def test_expert_parallel_matches_single_process(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    res = {}
    for _ in range(world):
        r, out, sent, recv = q.get(timeout=120)
        res[r] = (out, sent, recv)
    for pr in procs:
        pr.join(timeout=60)
    for r, (out, sent, recv) in res.items():
        assert not isinstance(out, str), out
    ref = _reference()
    Tr = T_TOTAL // world
    got = torch.cat([res[r][0] for r in range(world)])
    assert torch.allclose(got, ref, rtol=1e-5, atol=1e-4 * ref.abs().max().item())
    # every row sent is received by its destination
    for r in range(world):
        for d in range(world):
            assert res[r][1][d] == res[d][2][r]
        assert sum(res[r][1]) == Tr * SHAPE.top_k


def _failing_worker(rank, world, port, q):
    try:
        _init(rank, world, port, timeout_s=5)
        if rank == 1:
            raise RuntimeError("rank 1 fails before the count exchange")
        p = make_layer(SHAPE, 9)
        x = make_tokens(T_TOTAL // world, SHAPE.hidden, 9).float()
        local = shard_experts({k.split(".", 1)[1]: v for k, v in p.items() if k.startswith("experts.")},
                              rank, world)
        layer = ExpertParallelMoE(SHAPE.experts, SHAPE.top_k, ops=CpuOps())
        layer(x, p["router.weight"], p["router.bias"], local)
        q.put((rank, "completed"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, type(e).__name__ + ": " + str(e)[:200]))


def test_peer_failure_surfaces_as_error_not_hang():
    """A rank that dies before the exchange makes the survivor's collective fail
    within the process-group timeout (host-side failure injection)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    msgs = dict(q.get(timeout=120) for _ in range(2))
    for pr in procs:
        pr.join(timeout=60)
        if pr.is_alive():
            pr.kill()
    assert "rank 1 fails" in msgs[1]
    assert msgs[0] != "completed"
