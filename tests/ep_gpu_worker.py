"""One rank of the multi-GPU expert-parallel parity check (run by torchrun
from tests/test_gpu_ep.py; not collected by pytest).

Each rank owns E/R experts and T/R tokens.  For each case the layer output of
the rank's tokens is compared with the single-GPU layer on all tokens (the
same library kernels, so routing and results must agree), once through the
peer-memory exchange and once through NCCL all-to-all, over three successive
calls (the peer-memory flags and buffers are reused across calls) and, for
the peer-memory path, two replays of a captured CUDA graph; the two exchanges
must give bit-identical outputs.  Then the expert-granular streamed stack
over the same exchange (each rank pinning only its slice of two layers) must
equal the resident layers chained on the rank's tokens.  Last, rank 0 calls
the exchange while rank 1 does not: rank 0's bounded waits must run out and
report BS_ERR_TIMEOUT.
Exits non-zero on any mismatch."""

import datetime
import os
import sys

import torch
import torch.distributed as dist

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)

from blockstreamer_b200 import _lib, kernels  # noqa: E402
from blockstreamer_b200.expert_parallel import CudaOps, ExpertParallelMoE, P2PExchange, shard_experts  # noqa: E402
from blockstreamer_b200.streaming import EXPERT_TENSORS, StreamedEPStack  # noqa: E402
from blockstreamer_b200.synthetic import CASES, LayerShape, make_layer, make_tokens, zipf_router_bias  # noqa: E402


def rel_l2(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    cases = [("small", LayerShape(512, 512, 16, 4), 7, 64 * world),
             ("gptoss120b", CASES["gptoss120b"], 4, 256 * world)]
    algo = kernels.ALGO_TCGEN05
    ok = True
    for name, shape, case_id, T in cases:
        full = make_layer(shape, case_id, device=dev)
        x_all = make_tokens(T, shape.hidden, case_id, device=dev)
        pe = {k.split(".", 1)[1]: v for k, v in full.items() if k.startswith("experts.")}
        ref, _, idx_ref = kernels.moe_forward(
            x_all, pe["gate_up_proj_blocks"], pe["gate_up_proj_scales"], pe["gate_up_proj_bias"],
            pe["down_proj_blocks"], pe["down_proj_scales"], pe["down_proj_bias"], shape.top_k,
            router_weight=full["router.weight"], router_bias=full["router.bias"], algo=algo)
        Tr = T // world
        sl = slice(rank * Tr, (rank + 1) * Tr)
        x = x_all[sl].contiguous()
        local_p = shard_experts(pe, rank, world)
        outs = {}
        for transport in ("p2p", "nccl"):
            ex = P2PExchange(None, shape.experts, shape.hidden, Tr, shape.top_k, dev) if transport == "p2p" else None
            layer = ExpertParallelMoE(shape.experts, shape.top_k, ops=CudaOps(algo), exchange=ex)
            for call in range(3):
                out, _, idx = layer(x, full["router.weight"], full["router.bias"], local_p)
                torch.cuda.synchronize()
                same = (idx.long() == idx_ref[sl].long()).all(1)
                rel = rel_l2(out[same], ref[sl][same])
                good = bool(same.float().mean() >= 0.99) and rel <= 1e-3
                print(f"rank {rank} {name} {transport} call {call}: routing match {same.float().mean():.4f} "
                      f"rel_l2 vs single GPU {rel:.2e} {'ok' if good else 'MISMATCH'}", flush=True)
                ok &= good
            outs[transport] = out.clone()
            if ex is not None:
                # the peer-memory path has no host sync: capture one call, replay it
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    g_out, _, _ = layer(x, full["router.weight"], full["router.bias"], local_p)
                for rep in range(2):
                    g.replay()
                    torch.cuda.synchronize()
                    same_g = torch.equal(g_out, outs[transport])
                    print(f"rank {rank} {name} p2p graph replay {rep}: equal to eager {same_g}", flush=True)
                    ok &= same_g
                del g
            status = kernels.device_status(clear=True)
            if status:
                print(f"rank {rank} {name} {transport}: device status {status}", flush=True)
                ok = False
            if ex is not None:
                ex.close()
        same_bits = torch.equal(outs["p2p"], outs["nccl"])
        print(f"rank {rank} {name}: p2p and nccl outputs bit-identical: {same_bits}", flush=True)
        ok &= same_bits
    # The streamed stack over expert parallelism: each rank pins only its
    # slice of two Zipf-routed layers and stages the hit experts of it; its
    # output must equal the resident layers chained on the same tokens.
    shape = cases[0][1]
    T = 64 * world
    Tr = T // world
    states = []
    for li in range(2):
        st = make_layer(shape, 30 + li, device=dev)
        st["router.bias"] = zipf_router_bias(shape, 1.6, 30 + li).to(dev) * 4.0
        states.append(st)
    x_all = make_tokens(T, shape.hidden, 31, device=dev)
    x = x_all[rank * Tr:(rank + 1) * Tr].contiguous()
    ex = P2PExchange(None, shape.experts, shape.hidden, Tr, shape.top_k, dev)
    lo, hi = rank * (shape.experts // world), (rank + 1) * (shape.experts // world)
    host = [{n: (t[lo:hi] if n.startswith("experts.") else t).cpu() for n, t in st.items()} for st in states]
    # tensor-core kernels on both sides (at 64 tokens AUTO would take the
    # decode path for the resident layers, a different algorithm)
    stack = StreamedEPStack(host, shape.top_k, ex, groups=2, algo=kernels.ALGO_TCGEN05)
    for call in range(2):
        out = stack(x)
        torch.cuda.synchronize()
    ref = x
    for st in states:
        ref, _, _ = kernels.moe_forward(ref, *[st["experts." + n] for n in EXPERT_TENSORS], shape.top_k,
                                        router_weight=st["router.weight"], router_bias=st["router.bias"],
                                        algo=kernels.ALGO_TCGEN05)
    same = torch.equal(out, ref)
    print(f"rank {rank} streamed EP stack: staged experts per layer {stack.stats.experts_staged[-2:]} "
          f"of {hi - lo}, equal to resident layers: {same}", flush=True)
    ok &= same
    ex.close()

    # A peer that never takes part: rank 0 sends, rank 1 does not.  Rank 0's
    # waits for rank 1's counts and rows run out (bounded, ~2 s each) and
    # report BS_ERR_TIMEOUT through the status word; the context stays usable.
    shape = cases[0][1]
    ex = P2PExchange(None, shape.experts, shape.hidden, 64, shape.top_k, dev)
    kernels.device_status(clear=True)
    if rank == 0:
        x0 = make_tokens(64, shape.hidden, 9, device=dev)
        idx0 = torch.randint(0, shape.experts, (64, shape.top_k), device=dev, dtype=torch.int32)
        d0 = kernels.dispatch(idx0, shape.experts)
        ex.dispatch(x0, d0.expert_offsets, d0.token_of_row)
        torch.cuda.synchronize()
        status = kernels.device_status(clear=True)
        alive = float(torch.ones(4, device=dev).sum().item()) == 4.0
        timed_out = status == _lib.BS_ERR_TIMEOUT
        print(f"rank 0 absent peer: device status {status} (timeout reported: {timed_out}), context usable: {alive}",
              flush=True)
        ok &= bool(timed_out) and alive
    dist.barrier()
    ex.close()
    flag = torch.tensor([0 if ok else 1], device=dev)
    dist.all_reduce(flag)
    dist.destroy_process_group()
    sys.exit(1 if int(flag.item()) else 0)


if __name__ == "__main__":
    main()
