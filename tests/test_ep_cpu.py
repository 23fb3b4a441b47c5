"""Expert-parallel data movement on CPU ranks (gloo, world size 2 and 4).

The orchestration of gpt-oss-tvm_b200/ep.py runs with reference backends
whose "experts" are simple per-expert affine maps, and each rank's output is
compared with a single-process computation:
  * the all-to-all path (count exchange, all-to-all-v splits, source-major <->
    expert-major reorder, return path, combine);
  * the peer-memory path (count all-gather, rows written straight into the
    owning rank's buffers at the rows ``peer_layout`` gives, outputs written
    straight back), with shared-memory CPU tensors standing in for the IPC
    buffers and the same ordering collectives.
``peer_layout`` itself is also checked against an explicit simulation of
the all-to-all + reorder layout.
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


# ---------------------------------------------------------------- peer path --
def _ep_module():
    import importlib
    import sys
    sys.path.insert(0, REPO)
    return importlib.import_module("gpt-oss-tvm_b200.ep")


@pytest.mark.parametrize("world,El", [(2, 3), (4, 2), (8, 4)])
def test_peer_layout_matches_all_to_all_reorder(world, El):
    """Row of (source s, local expert e, i-th row) on rank d: peer_layout's
    dst_base + i equals its position after the all-to-all (source-major
    blocks) and the expert-major reorder."""
    ep = _ep_module()
    g = torch.Generator().manual_seed(world * 10 + El)
    ca = torch.randint(0, 6, (world, world * El), generator=g)
    for d in range(world):
        # what rank d holds after the reorder: expert-major, source-major inside an expert
        held = [(s, e, i) for e in range(El) for s in range(world) for i in range(int(ca[s, d * El + e]))]
        pos = {key: n for n, key in enumerate(held)}
        for s in range(world):
            dst_base, _, _ = ep.peer_layout(ca, s, El)
            for e in range(El):
                for i in range(int(ca[s, d * El + e])):
                    assert int(dst_base[d, e]) + i == pos[(s, e, i)]
        _, indptr, recv = ep.peer_layout(ca, d, El)
        assert recv == len(held)
        for e in range(El):
            assert int(indptr[e + 1] - indptr[e]) == int(ca[:, d * El + e].sum())


class TorchPeerBackend(TorchBackend):
    """Reference backend of the peer path: this rank writes other ranks' rows
    directly into their (shared-memory) buffers."""

    def __init__(self, E, El, k, H, world, rank, shared):
        super().__init__(E, El, k, H, world, rank)
        self.shared = shared  # per rank: dict(act=[cap, H], origin=[cap], back=[M*k, H])

    def setup_peer(self, group, rank):
        self.peer = {"one": torch.ones(1, dtype=torch.int32)}

    def route(self, x):
        self.w, idx = self.route_fn(x)
        flat = idx.reshape(-1).to(torch.int64)
        order = torch.argsort(flat, stable=True)
        self.rev = torch.empty_like(order)
        self.rev[order] = torch.arange(order.numel())
        self.send_tok = order // self.k
        self.send_exp = flat[order]
        self.x = x
        counts = torch.bincount(flat, minlength=self.E).to(torch.int32)
        self.indptr = torch.zeros(self.E + 1, dtype=torch.int64)
        self.indptr[1:] = torch.cumsum(counts, 0)
        return counts

    def route_fn(self, x):
        return TorchBackend.route(self, x)

    def layout_peer(self, counts_all, rank):
        ep = _ep_module()
        self.dst_base, self.indptr_local, self.recv_rows = ep.peer_layout(counts_all, rank, self.El)

    def dispatch_peer(self, M):
        dst_base = self.dst_base
        for r in range(self.send_tok.numel()):
            eg = int(self.send_exp[r])
            d, e = eg // self.El, eg % self.El
            dst = int(dst_base[d, e]) + r - int(self.indptr[eg])
            self.shared[d]["act"][dst] = self.x[self.send_tok[r]]
            self.shared[d]["origin"][dst] = (self.rank << 24) | r

    def experts_peer(self):
        indptr_local = self.indptr_local
        me = self.shared[self.rank]
        for e in range(self.El):
            for row in range(int(indptr_local[e]), int(indptr_local[e + 1])):
                o = int(me["origin"][row])
                self.shared[o >> 24]["back"][o & 0xFFFFFF] = self.expert_fn(self.rank * self.El + e, me["act"][row])

    def combine_peer(self, x, out):
        return self.combine(self.shared[self.rank]["back"][: x.shape[0] * self.k], x, out)


def _peer_worker(rank, world, port, E, H, M, shared, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ep = _ep_module()
    El, k = E // world, 4
    be = TorchPeerBackend(E, El, k, H, world, rank, shared)
    runner = ep.ExpertParallelMoE(_Blk(E, El, k, H, rank), M, backend=be, peer=True)
    errs = []
    for step in range(2):  # a second step reuses every buffer
        g = torch.Generator().manual_seed(100 + 7 * step + rank)
        x = torch.randn(M, H, generator=g)
        out = runner.forward(x)
        w, idx = be.route_fn(x)
        ref = x.clone()
        for m in range(M):
            for r in range(k):
                e = int(idx[m, r])
                ref[m] += w[m, r] * be.expert_fn(e, x[m])
        errs.append(float((out - ref).abs().max()))
    q.put((rank, max(errs), runner.last_splits))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_expert_parallel_peer_path_gloo(world):
    E, H, M, k = 16, 32, 37, 4
    cap = world * M * k
    shared = [dict(act=torch.zeros(cap, H).share_memory_(), origin=torch.zeros(cap, dtype=torch.int64).share_memory_(),
                   back=torch.zeros(M * k, H).share_memory_()) for _ in range(world)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, E, H, M, shared, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, splits in res:
        assert err < 1e-4, f"rank {rank}: max err {err}"
        assert sum(splits[0]) == M * k
