"""Expert-parallel host logic on CPU: gloo ranks run EPMoELayer's real
collective sequence (counts, rows, records, results) with the CUDA route /
pack / combine kernels and the expert compute replaced by torch stand-ins.

Checks the combine against a direct computation, the order in which each
owner receives its rows ((source rank, pair) order, local ids), that an
expert id out of range on one rank raises on every rank with no collective
left waiting, and that sources of different call sizes have their rows
computed in their own classes (one local call per run of same-class
sources, each forced to its class, the size rule restored after)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from wisp_b200 import _lib
from wisp_b200.expert_parallel import EPMoELayer

E, H, K, T = 8, 16, 3, 5


class _FakeExperts:
    """y = x * (global id + 1) * w, stored bf16; records the ids it saw."""

    def __init__(self, rank, per):
        self.rank, self.per, self.seen, self.classes = rank, per, [], []
        self.hidden_size, self.device = H, torch.device("cpu")

    def compute_class(self, pairs):
        return "tc" if pairs >= 10 else "cuda"

    def configure(self, compute_class=None):
        self.classes.append(compute_class)

    def forward(self, x, w, ids, out):
        self.seen.append(ids.reshape(-1).clone())
        g = ids.reshape(-1).long() + self.rank * self.per
        out.copy_((x.float() * (g + 1).view(-1, 1).float() * w.reshape(-1, 1)).to(torch.bfloat16))


class _CpuEP(EPMoELayer):
    """The route/pack and combine kernels restated in torch (CPU tensors)."""

    def _route_pack(self, x, w, ids, T_, K_, H_, send_x, send_meta, counts, pos):
        flat = ids.reshape(-1).long()
        bad = int(((flat < 0) | (flat >= self.num_experts)).sum())
        counts[self.world] = bad
        if bad:
            counts[: self.world] = 0
            pos.fill_(-1)
            return
        dest = flat // self.experts_per_rank
        order = torch.argsort(dest, stable=True)
        pos[order] = torch.arange(flat.numel(), dtype=torch.int32)
        send_x.copy_(x[order // K_])
        send_meta[:, 0] = (flat - dest * self.experts_per_rank)[order].to(torch.int32)
        send_meta[:, 1] = w.reshape(-1)[order].view(torch.int32)
        counts[: self.world] = torch.bincount(dest, minlength=self.world)

    def _combine(self, back, pos, T_, K_, out):
        acc = torch.zeros((T_, back.shape[1]), dtype=torch.float32)
        p = pos.view(T_, K_).long()
        for k in range(K_):
            acc += back[p[:, k]].float()
        out.copy_(acc.to(torch.bfloat16))


def _routing(rank, seed):
    g = torch.Generator().manual_seed(seed * 100 + rank)
    ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).to(torch.int32)
    w = torch.rand((T, K), generator=g)
    x = torch.randn((T, H), generator=g).to(torch.bfloat16)
    return x, w, ids


def _worker(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        per = E // world
        local = _FakeExperts(rank, per)
        layer = _CpuEP(None, None, E, per, local=local, device="cpu")
        for seed in range(3):
            x, w, ids = _routing(rank, seed)
            out = layer.forward(x, w, ids)
            # direct: sum over k in routing order of the bf16 rows
            acc = torch.zeros((T, H))
            for k in range(K):
                y = (x.float() * (ids[:, k].long() + 1).view(-1, 1).float() * w[:, k:k + 1]).to(torch.bfloat16)
                acc += y.float()
            assert torch.equal(out, acc.to(torch.bfloat16)), f"rank {rank} seed {seed}: combine differs"
            # this owner saw every source's pairs for it, sources in rank order, pairs in (t, k) order
            expect = []
            for src in range(world):
                _, _, sids = _routing(src, seed)
                flat = sids.reshape(-1).long()
                mine = flat[(flat // per) == rank]
                expect.append(mine - rank * per)
            seen = local.seen[-1] if len(torch.cat(expect)) else torch.empty(0, dtype=torch.int32)
            assert torch.equal(seen.long(), torch.cat(expect)), f"rank {rank}: receive order"
            if len(torch.cat(expect)):
                # every source called with T * K = 15 pairs: one call, forced to that
                # class, then back to the size rule
                assert local.classes[-2:] == ["tc", "auto"], local.classes
        # an id out of range on rank 1 only: every rank raises, nothing left pending
        x, w, ids = _routing(rank, 9)
        if rank == 1:
            ids[2, 1] = E
        with pytest.raises(_lib.WispError):
            layer.forward(x, w, ids)
        # and the group still works afterwards
        x, w, ids = _routing(rank, 10)
        layer.forward(x, w, ids)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_ep_collectives_gloo(world):
    mp.start_processes(_worker, args=(world, _free_port()), nprocs=world, start_method="spawn")


def _mixed_worker(rank, world, port):
    """Rank r routes T_r tokens: the fake layer's class rule (>= 10 pairs:
    "tc") puts ranks 0 and 1 on one side and ranks 2 and 3 on the other, so
    an owner receives runs of sources [tc, tc, cuda, cuda]."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        per = E // world
        Ts = [5, 4, 3, 2][:world]   # x K = 3: 15, 12 pairs ("tc"); 9, 6 ("cuda")
        local = _FakeExperts(rank, per)
        layer = _CpuEP(None, None, E, per, local=local, device="cpu")
        g = torch.Generator().manual_seed(7 + rank)
        T = Ts[rank]
        ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).to(torch.int32)
        w = torch.rand((T, K), generator=g)
        x = torch.randn((T, H), generator=g).to(torch.bfloat16)
        out = layer.forward(x, w, ids)
        acc = torch.zeros((T, H))
        for k in range(K):
            acc += (x.float() * (ids[:, k].long() + 1).view(-1, 1).float() * w[:, k:k + 1]).to(torch.bfloat16).float()
        assert torch.equal(out, acc.to(torch.bfloat16)), f"rank {rank}: combine differs"
        # what this owner received from each source, and the calls it made
        counts = torch.zeros(world, dtype=torch.int64)
        for src in range(world):
            gs = torch.Generator().manual_seed(7 + src)
            sids = torch.stack([torch.randperm(E, generator=gs)[:K] for _ in range(Ts[src])])
            counts[src] = int(((sids.reshape(-1) // per) == rank).sum())
        expect_runs = []
        for src in range(world):
            cls = "tc" if Ts[src] * K >= 10 else "cuda"
            if counts[src]:
                if expect_runs and expect_runs[-1][0] == cls:
                    expect_runs[-1][1] += int(counts[src])
                else:
                    expect_runs.append([cls, int(counts[src])])
        assert local.classes == [c for c, _ in expect_runs] + ["auto"], (rank, local.classes, expect_runs)
        assert [len(v) for v in local.seen] == [n for _, n in expect_runs], (rank, expect_runs)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_ep_mixed_call_sizes_gloo():
    mp.start_processes(_mixed_worker, args=(4, _free_port()), nprocs=4, start_method="spawn")
