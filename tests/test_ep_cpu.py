"""Expert-parallel data movement on CPU ranks (gloo, world size 2 and 4).

The orchestration of gpt-oss-tvm_b200/ep.py (count exchange, all-to-all-v
splits, source-major <-> expert-major reorder, return path, combine) runs
with a reference backend whose "experts" are simple per-expert affine maps,
and each rank's output is compared with a single-process computation.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import REPO


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class TorchBackend:
    """Reference for the device steps, on CPU tensors (test only)."""

    def __init__(self, E, El, k, H, world, rank):
        self.E, self.El, self.k, self.H, self.world, self.rank = E, El, k, H, world, rank
        g = torch.Generator().manual_seed(7)
        self.Wr = torch.randn(H, E, generator=g)

    def route(self, x):
        logits = x @ self.Wr
        vals, idx = torch.topk(logits, self.k, dim=1)
        w = torch.softmax(vals, dim=1)
        return w, idx.to(torch.int32)

    @staticmethod
    def expert_fn(e, rows):
        return rows * (e + 1) + e

    def route_and_pack(self, x):
        M = x.shape[0]
        self.w, idx = self.route(x)
        flat = idx.reshape(-1).to(torch.int64)
        order = torch.argsort(flat, stable=True)  # expert-major, token ascending
        self.rev = torch.empty_like(order)
        self.rev[order] = torch.arange(order.numel())
        tok = order // self.k
        send = x[tok].contiguous()
        counts = torch.bincount(flat, minlength=self.E).to(torch.int32)
        return send, counts.view(self.world, self.El)

    def recv_buffer(self, rows):
        return torch.empty(rows, self.H)

    def back_buffer(self, rows):
        return torch.empty(rows, self.H)

    def experts(self, recv_rows, recv_counts):
        P, El = self.world, self.El
        c = recv_counts.tolist()
        # source-major segments -> compute per expert -> back to source-major
        out = torch.empty_like(self.recv_ref[:recv_rows])
        off = 0
        for s in range(P):
            for e in range(El):
                n = c[s][e]
                seg = self.recv_ref[off:off + n]
                out[off:off + n] = self.expert_fn(self.rank * El + e, seg)
                off += n
        return out

    def combine(self, back, x, out):
        M = x.shape[0]
        y = back[self.rev].view(M, self.k, self.H)
        out.copy_(x + (y * self.w.unsqueeze(-1)).sum(1))
        return out


class _Blk:
    def __init__(self, E, El, k, H, rank):
        self.num_experts, self.num_local_experts, self.experts_per_token = E, El, k
        self.hidden_size = H
        self.expert_offset = rank * El


def _worker(rank, world, port, E, H, M, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import sys
    sys.path.insert(0, REPO)
    import importlib
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ep = importlib.import_module("gpt-oss-tvm_b200.ep")
    El, k = E // world, 4
    be = TorchBackend(E, El, k, H, world, rank)
    # recv buffer must be visible to the backend's expert step
    orig_recv = be.recv_buffer

    def recv_buffer(rows):
        be.recv_ref = orig_recv(rows)
        return be.recv_ref

    be.recv_buffer = recv_buffer
    runner = ep.ExpertParallelMoE(_Blk(E, El, k, H, rank), M, backend=be)
    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn(M, H, generator=g)
    out = runner.forward(x)
    # single-process reference
    w, idx = be.route(x)
    ref = x.clone()
    for m in range(M):
        for r in range(k):
            e = int(idx[m, r])
            ref[m] += w[m, r] * be.expert_fn(e, x[m])
    err = float((out - ref).abs().max())
    q.put((rank, err, runner.last_splits))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_expert_parallel_dispatch_combine_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 16, 32, 37, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, splits in res:
        assert err < 1e-4, f"rank {rank}: max err {err}"
        assert sum(splits[0]) == 37 * 4
