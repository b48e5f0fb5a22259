"""Expert parallelism on the GPU.

* Ranks emulated on one GPU: every rank's dispatch kernel, paged shard and
  combine kernel run for real; the all-to-all is done in the test by slicing
  the send buffers the way the collective would.  The output must be
  byte-identical to the one-GPU layer over all experts, and each paged rank's
  pager state must equal the oracle pager over its shard fed the rows it
  received, in (source rank, pair) order.  Call sizes on either side of the
  tensor-core threshold (74 pairs at these shapes), also mixed across ranks: each owner
  computes a source's rows in the class of that source's call size.
* Two real ranks over NCCL (needs two GPUs; skipped otherwise): the same
  byte identity through torch.distributed.
"""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

from oracle.pager import PagerOracle, forward_pager
from wisp_b200 import workloads as wl
from wisp_b200.expert_parallel import EPMoELayer, shard_range

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _weights(E, H, I, seed):
    g = torch.Generator().manual_seed(seed)
    return ((torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16),
            (torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16), g)


def emulated_forward(layers, xs, ws, idss):
    """One EP forward of every rank, the all-to-alls done by slicing.  Returns
    the outputs, each rank's received rows / records / results."""
    P = len(layers)
    plans = [layers[r].begin(xs[r], ws[r], idss[r]) for r in range(P)]
    counts = [p.counts_dev.cpu().tolist() for p in plans]
    for r, c in enumerate(counts):
        assert c[P] == 0, f"rank {r}: ids out of range"
    for r in range(P):
        plans[r].send_counts = counts[r][:P]
        plans[r].recv_counts = [counts[s][r] for s in range(P)]
    offs = [np.concatenate([[0], np.cumsum(c[:P])]) for c in counts]
    recv_x, recv_m = [], []
    for r in range(P):
        recv_x.append(torch.cat([plans[s].send_x[offs[s][r]:offs[s][r + 1]] for s in range(P)]))
        recv_m.append(torch.cat([plans[s].send_meta[offs[s][r]:offs[s][r + 1]] for s in range(P)]))
    src_pairs = [plans[s].num_tokens * plans[s].top_k for s in range(P)]
    recv_y = [layers[r].compute(recv_x[r], recv_m[r], plans[r].recv_counts, src_pairs) for r in range(P)]
    outs = []
    for s in range(P):
        parts = []
        for r in range(P):
            start = sum(counts[q][r] for q in range(s))
            parts.append(recv_y[r][start:start + counts[s][r]])
        outs.append(layers[s].finish(plans[s], torch.cat(parts)))
    return outs, recv_x, recv_m, recv_y


@pytest.mark.parametrize("P,cap,mode,K,Ts", [
    (2, 8, "resident", 4, (6, 6)), (2, 3, "paged", 4, (6, 6)), (4, 2, "paged", 4, (6, 6, 6, 6)),
    (4, 4, "resident", 4, (6, 6, 6, 6)),
    (4, 4, "resident", 8, (10, 10, 10, 10)),  # 80 pairs per source: tensor cores (threshold 74), owners ~80 rows
    (2, 8, "resident", 8, (12, 3)),           # one source above the threshold, one below
    (2, 8, "paged", 8, (12, 12)),
])
def test_ep_emulated_ranks_match_one_gpu(P, cap, mode, K, Ts):
    from wisp_b200.integrations.vllm.fused_moe import WispMoEState
    E, H, I = 16, 512, 256
    w13, w2, g = _weights(E, H, I, 3)
    layers = []
    oracles = []
    for r in range(P):
        lo, hi = shard_range(E, r, P)
        layers.append(EPMoELayer(w13[lo:hi], w2[lo:hi], E, cap, mode, DEV, 0, rank=r, world_size=P))
        oracles.append(PagerOracle(E // P, cap))
    full = WispMoEState(w13, w2, E, "resident", DEV, 0)
    full.prime_identity()
    for step in range(4):
        xs, ws, idss = [], [], []
        for r in range(P):
            T = Ts[r]
            w, ids = wl.softmax_topk(torch.randn(T, E, generator=g), K)
            xs.append(torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV))
            ws.append(w.to(DEV))
            idss.append(ids.to(DEV))
        outs, _, recv_m, _ = emulated_forward(layers, xs, ws, idss)
        for r in range(P):
            layers[r].local.synchronize()
            ref = full.forward(xs[r], ws[r], idss[r])
            assert torch.equal(outs[r], ref), f"step {step} rank {r}: EP output differs from one GPU"
            s2e, tick, clock, stats = layers[r].local._read()
            if mode == "resident":  # no paging: the identity map stays
                assert s2e == list(range(E // P)), (step, r)
                continue
            forward_pager(oracles[r], recv_m[r][:, 0].cpu().numpy().reshape(-1, 1))
            o = oracles[r]
            assert s2e == o.slot_to_expert and tick == o.lru_tick and clock == o.lru_clock, (step, r)
            assert stats == [o.stats_forward, o.stats_miss, o.stats_hits, o.stats_evict], (step, r)
    for layer in layers:
        layer.close()
    full.close()


def test_ep_dispatch_rejects_out_of_range_ids():
    E, H, K, T, P = 16, 64, 2, 3, 2
    layer = EPMoELayer(None, None, E, 4, local=type("L", (), {"hidden_size": H, "device": DEV})(),
                       device=DEV, rank=0, world_size=P)
    x = torch.randn(T, H).to(torch.bfloat16).to(DEV)
    w = torch.full((T, K), 0.5).to(DEV)
    ids = torch.tensor([[0, 1], [2, E], [3, 4]], dtype=torch.int64).to(DEV)
    plan = layer.begin(x, w, ids)
    assert plan.counts_dev.cpu().tolist()[P] == 1
    assert (plan.pair_pos.cpu() == -1).all()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_nccl_two_ranks_match_one_gpu():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(ROOT, "tests", "ep_nccl_check.py")]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "ep nccl ok" in r.stdout
