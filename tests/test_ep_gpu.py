"""Expert parallelism on the GPU.

* Ranks emulated on one GPU (``EPExchange.emulated``): every rank's
  dispatch, receive, paged shard, return and combine kernels run for real and
  store into the other ranks' buffers directly; the steps are issued rank by
  rank in an order in which every wait finds its data already written (all
  dispatches before any receive, all returns before any combine).  The
  output must be byte-identical to the one-GPU layer over all experts, and
  each paged rank's pager state must equal the oracle pager over its shard
  fed the rows it received, in (source rank, pair) order.  Call sizes on
  either side of the tensor-core threshold (74 pairs at these shapes), also
  mixed across ranks: each owner computes a source's rows in the class of
  that source's call size.
* An id out of range on one rank fails every rank's receive alike, and the
  group keeps working; a source that never dispatches makes the receive's
  bounded wait run out with a timeout status (no GPU fault, no hang).
* Real ranks (2 and 4 GPUs; skipped on fewer): ``ep_nccl_check.py`` under
  torch.distributed.run at Qwen3-30B-A3B layer shapes.
"""
import os
import socket
import subprocess
import sys

import pytest
import torch

from oracle.pager import PagerOracle, forward_pager
from wisp_b200 import _lib
from wisp_b200 import workloads as wl
from wisp_b200.expert_parallel import EPExchange, EPMoELayer, shard_range

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _weights(E, H, I, seed):
    g = torch.Generator().manual_seed(seed)
    return ((torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16),
            (torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16), g)


def emulated_forward(layers, xs, ws, idss):
    """One EP forward of every rank in this process.  Returns the outputs and
    the local ids each rank received (in the order its pager saw them)."""
    P = len(layers)
    shapes = [layers[r].begin(xs[r], ws[r], idss[r]) for r in range(P)]
    arrivals = [layers[r].arrive() for r in range(P)]
    recv_ids = [layers[r].exchange.received(sum(arrivals[r][0]))[2].reshape(-1).cpu() for r in range(P)]
    for r in range(P):
        layers[r].compute(*arrivals[r])
    for r in range(P):
        layers[r].exchange.send_back()
    outs = []
    for r in range(P):
        T, K = shapes[r]
        out = torch.empty((T, xs[r].shape[1]), dtype=torch.bfloat16, device=DEV)
        layers[r].exchange.combine(out, T, K)
        outs.append(out)
    return outs, recv_ids


@pytest.mark.parametrize("P,cap,mode,K,Ts", [
    (2, 8, "resident", 4, (6, 6)), (2, 3, "paged", 4, (6, 6)), (4, 2, "paged", 4, (6, 6, 6, 6)),
    (4, 4, "resident", 4, (6, 6, 6, 6)),
    (4, 4, "resident", 8, (10, 10, 10, 10)),  # 80 pairs per source: tensor cores (threshold 74), owners ~80 rows
    (2, 8, "resident", 8, (12, 3)),           # one source above the threshold, one below
    (2, 8, "paged", 8, (12, 12)),
    (4, 3, "paged", 8, (12, 0, 5, 12)),       # a rank with no tokens still takes part
])
def test_ep_emulated_ranks_match_one_gpu(P, cap, mode, K, Ts):
    from wisp_b200.integrations.vllm.fused_moe import WispMoEState
    E, H, I = 16, 512, 256
    w13, w2, g = _weights(E, H, I, 3)
    exs = EPExchange.emulated(P, H, max(Ts) * K, DEV)
    layers, oracles = [], []
    for r in range(P):
        lo, hi = shard_range(E, r, P)
        layers.append(EPMoELayer(w13[lo:hi], w2[lo:hi], E, cap, mode, DEV, 0, exchange=exs[r]))
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
        outs, recv_ids = emulated_forward(layers, xs, ws, idss)
        for r in range(P):
            layers[r].synchronize()
            if Ts[r] == 0:
                assert outs[r].numel() == 0
                continue
            ref = full.forward(xs[r], ws[r], idss[r])
            assert torch.equal(outs[r], ref), f"step {step} rank {r}: EP output differs from one GPU"
        for r in range(P):
            s2e, tick, clock, stats = layers[r].local._read()
            if mode == "resident":  # no paging: the identity map stays
                assert s2e == list(range(E // P)), (step, r)
                continue
            for r0, n in layers[r].last_runs:   # one pager call per run of same-class sources
                forward_pager(oracles[r], recv_ids[r][r0:r0 + n].numpy().reshape(-1, 1))
            o = oracles[r]
            assert s2e == o.slot_to_expert and tick == o.lru_tick and clock == o.lru_clock, (step, r)
            assert stats == [o.stats_forward, o.stats_miss, o.stats_hits, o.stats_evict], (step, r)
    for layer in layers:
        layer.close()
    for e in exs:
        e.close()
    full.close()


class _NoCompute:
    hidden_size = 64
    device = DEV

    def forward(self, x, w, ids, out):
        out.zero_()

    def synchronize(self):
        pass


def test_ep_out_of_range_id_fails_every_rank_alike():
    E, H, K, T, P = 16, 64, 2, 3, 2
    exs = EPExchange.emulated(P, H, T * K, DEV)
    layers = [EPMoELayer(None, None, E, 4, local=_NoCompute(), device=DEV, exchange=exs[r]) for r in range(P)]
    x = torch.randn(T, H).to(torch.bfloat16).to(DEV)
    w = torch.full((T, K), 0.5).to(DEV)
    good = torch.tensor([[0, 9], [2, 15], [3, 8]], dtype=torch.int64).to(DEV)
    bad = torch.tensor([[0, 1], [2, E], [3, 4]], dtype=torch.int64).to(DEV)
    layers[0].begin(x, w, bad)
    layers[1].begin(x, w, good)
    for r in range(P):
        with pytest.raises(_lib.WispError) as ei:
            layers[r].arrive()
        assert ei.value.code == _lib.WISP_ERR_BAD_EXPERT
    # the group keeps working: a clean forward on both ranks
    outs, _ = emulated_forward(layers, [x, x], [w, w], [good, good])
    for r in range(P):
        layers[r].synchronize()
        assert outs[r].shape == (T, H)
    for e in exs:
        e.close()


def test_ep_missing_source_times_out_with_status():
    """Rank 1 never dispatches: rank 0's receive waits on a flag nothing sets,
    gives up after its (short) limit and reports a timeout."""
    E, H, K, T, P = 16, 64, 2, 3, 2
    exs = EPExchange.emulated(P, H, T * K, DEV)
    for e in exs:
        e.configure(wait_ns=50_000_000)
    layer = EPMoELayer(None, None, E, 4, local=_NoCompute(), device=DEV, exchange=exs[0])
    x = torch.randn(T, H).to(torch.bfloat16).to(DEV)
    w = torch.full((T, K), 0.5).to(DEV)
    ids = torch.tensor([[0, 9], [2, 15], [3, 8]], dtype=torch.int64).to(DEV)
    layer.begin(x, w, ids)
    with pytest.raises(_lib.WispError) as ei:
        layer.arrive()
    assert ei.value.code == _lib.WISP_ERR_TIMEOUT
    exs[0].synchronize()                      # reported by the receive itself, nothing left pending
    for e in exs:
        e.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("ranks", [2, 4])
def test_ep_real_ranks_match_one_gpu(ranks):
    if torch.cuda.device_count() < ranks:
        pytest.skip(f"needs {ranks} GPUs")
    cmd = ["timeout", "-k", "30", "900", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={ranks}", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(ROOT, "tests", "ep_nccl_check.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=960, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "ep multi-gpu ok" in r.stdout
