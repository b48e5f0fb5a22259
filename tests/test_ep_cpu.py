"""Expert-parallel host logic on CPU: gloo ranks run EPMoELayer's forward
(dispatch, receive, the per-class local calls, return, combine) with the
peer-memory exchange replaced by a stand-in that moves the same rows and
records with gloo all-to-alls, and the expert compute by a torch stand-in.

Checks the combine against a direct computation, the order in which each
owner receives its rows ((source rank, pair) order, local ids), that an
expert id out of range on one rank raises on every rank with nothing left
waiting, and that sources of different call sizes have their rows computed
in their own classes (one local call per run of same-class sources, each
forced to its class, the size rule restored after)."""
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

    def class_threshold(self):
        return 10

    def configure(self, compute_class=None):
        self.classes.append(compute_class)

    def forward(self, x, w, ids, out):
        self.seen.append(ids.reshape(-1).clone())
        g = ids.reshape(-1).long() + self.rank * self.per
        out.copy_((x.float() * (g + 1).view(-1, 1).float() * w.reshape(-1, 1)).to(torch.bfloat16))

    def synchronize(self):
        pass


class _GlooExchange:
    """The peer-memory exchange's four steps restated with gloo collectives
    on CPU tensors: same rows, records, order and combine arithmetic."""

    def __init__(self, rank, world):
        self.rank, self.world, self.hidden = rank, world, H

    def dispatch(self, x, w, ids, e_local):
        flat = ids.reshape(-1).long()
        self.T, self.K = ids.shape
        P = flat.numel()
        bad = bool(((flat < 0) | (flat >= e_local * self.world)).any())
        owner = flat // e_local
        send_rows, send_recs, counts = [], [], []
        for d in range(self.world):
            sel = (owner == d).nonzero().reshape(-1) if not bad else torch.empty(0, dtype=torch.long)
            counts.append(-1 if bad else int(sel.numel()))
            send_rows.append(x[sel // self.K].float())
            send_recs.append(torch.stack([(flat[sel] - d * e_local).float(), w.reshape(-1)[sel].float(),
                                          sel.float()], dim=1) if len(sel) else torch.zeros(0, 3))
        head = torch.tensor([[c, P] for c in counts], dtype=torch.int64)
        rhead = torch.empty_like(head)
        dist.all_to_all_single(rhead, head)
        self.counts = [int(v) for v in rhead[:, 0]]
        self.src_pairs = [int(v) for v in rhead[:, 1]]
        ok = all(c >= 0 for c in self.counts)
        scount = [max(c, 0) for c in counts]
        rcount = [max(c, 0) for c in self.counts]
        rows = torch.empty((sum(rcount), H))
        recs = torch.empty((sum(rcount), 3))
        dist.all_to_all_single(rows, torch.cat(send_rows) if sum(scount) else torch.empty(0, H), rcount, scount)
        dist.all_to_all_single(recs, torch.cat(send_recs) if sum(scount) else torch.empty(0, 3), rcount, scount)
        self.ok, self.rows, self.recs, self.scount, self.rcount = ok, rows, recs, scount, rcount

    def receive(self, class_min_pairs=0):
        if not self.ok:
            raise _lib.WispError(_lib.WISP_ERR_BAD_EXPERT, "a rank routed an expert id out of range")
        R = sum(self.rcount)
        # runs of consecutive same-class sources; rows ordered by expert within a run, stably
        order, row, prev = [], 0, None
        for c, pairs in zip(self.rcount, self.src_pairs):
            cls = class_min_pairs > 0 and pairs >= class_min_pairs
            if c and (prev is None or cls != prev):
                order.append([row, row + c])
                prev = cls
            elif c:
                order[-1][1] += c
            row += c
        perm = torch.cat([r0 + torch.argsort(self.recs[r0:r1, 0], stable=True) for r0, r1 in order]) \
            if order else torch.empty(0, dtype=torch.long)
        self.perm = perm
        self.rows, self.recs_sorted = self.rows[perm], self.recs[perm]
        self.x = self.rows.to(torch.bfloat16)
        self.ids = self.recs_sorted[:, 0].to(torch.int32).reshape(R, 1)
        self.w = self.recs_sorted[:, 1].reshape(R, 1).contiguous()
        self.y = torch.empty((R, H), dtype=torch.bfloat16)
        return self.counts, self.src_pairs

    def received(self, R):
        return self.x[:R], self.w[:R], self.ids[:R], self.y[:R]

    def send_back(self):
        back = torch.empty((sum(self.scount), H))
        y = torch.empty_like(self.y)
        y[self.perm] = self.y                       # back to (source, pair) order
        dist.all_to_all_single(back, y.float(), self.scount, self.rcount)
        pairs = torch.empty((sum(self.scount), 3))
        dist.all_to_all_single(pairs, self.recs, self.scount, self.rcount)
        self.back = torch.zeros((self.T * self.K, H))
        self.back[pairs[:, 2].long()] = back

    def combine(self, out, T_, K_):
        acc = torch.zeros((T_, H))
        b = self.back.view(T_, K_, H)
        for k in range(K_):
            acc = acc + b[:, k]
            if K_ <= 4:
                acc = acc.to(torch.bfloat16).float()
        out.copy_(acc.to(torch.bfloat16))

    def synchronize(self):
        pass


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
        layer = EPMoELayer(None, None, E, per, local=local, device="cpu", exchange=_GlooExchange(rank, world))
        for seed in range(3):
            x, w, ids = _routing(rank, seed)
            out = layer.forward(x, w, ids)
            # direct: sum over k in routing order of the bf16 rows (bf16 partial sums: top-3)
            acc = torch.zeros((T, H))
            for k in range(K):
                y = (x.float() * (ids[:, k].long() + 1).view(-1, 1).float() * w[:, k:k + 1]).to(torch.bfloat16)
                acc = (acc + y.float()).to(torch.bfloat16).float()
            assert torch.equal(out, acc.to(torch.bfloat16)), f"rank {rank} seed {seed}: combine differs"
            # this owner saw every source's pairs for it (one run: every source has 15
            # pairs), ordered by local expert, stably
            expect = []
            for src in range(world):
                _, _, sids = _routing(src, seed)
                flat = sids.reshape(-1).long()
                mine = flat[(flat // per) == rank]
                expect.append(mine - rank * per)
            expect = torch.cat(expect)
            expect = expect[torch.argsort(expect, stable=True)]
            seen = local.seen[-1] if len(expect) else torch.empty(0, dtype=torch.int32)
            assert torch.equal(seen.long(), expect), f"rank {rank}: receive order"
            if len(expect):
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
def test_ep_host_logic_gloo(world):
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
        layer = EPMoELayer(None, None, E, per, local=local, device="cpu", exchange=_GlooExchange(rank, world))
        g = torch.Generator().manual_seed(7 + rank)
        T = Ts[rank]
        ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).to(torch.int32)
        w = torch.rand((T, K), generator=g)
        x = torch.randn((T, H), generator=g).to(torch.bfloat16)
        out = layer.forward(x, w, ids)
        acc = torch.zeros((T, H))
        for k in range(K):
            y = (x.float() * (ids[:, k].long() + 1).view(-1, 1).float() * w[:, k:k + 1]).to(torch.bfloat16)
            acc = (acc + y.float()).to(torch.bfloat16).float()
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


def test_owner_reserves_its_largest_receive():
    """An owner's call size is what it receives, which varies per call; its
    layer reserves the largest receive (every source's pairs, one expert per
    row) when built, so no call in a run grows the workspace."""
    class _Reserving(_FakeExperts):
        def __init__(self):
            super().__init__(0, 4)
            self.reserved = []

        def reserve(self, num_tokens, top_k):
            self.reserved.append((num_tokens, top_k))

    class _Ex:
        world, rank, hidden, max_pairs = 4, 1, H, 96

    local = _Reserving()
    EPMoELayer(None, None, 16, 4, local=local, device="cpu", exchange=_Ex())
    assert local.reserved == [(4 * 96, 1)]
