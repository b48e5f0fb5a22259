"""Multi-GPU check of EPMoELayer (launched by tests/test_ep_gpu.py under
torch.distributed.run, one GPU per rank, 2 or 4 ranks).

Qwen3-30B-A3B layer shapes (H 2048, I 768, E 128, top-8).  Every rank's EP
output must be byte-identical to a one-GPU layer over all experts on the same
tokens, for paged shards (cap 8 per rank) and resident shards, at call sizes
on both sides of the tensor-core threshold and mixed across ranks; each paged
rank's pager state must equal the oracle pager over its shard fed the rows it
received.  torch.distributed (NCCL) only builds the exchange (IPC handles)
and reduces the verdict; the rows move over peer memory.
"""
import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from oracle.pager import PagerOracle, forward_pager  # noqa: E402
from wisp_b200 import workloads as wl  # noqa: E402
from wisp_b200.expert_parallel import EPExchange, EPMoELayer, shard_range  # noqa: E402
from wisp_b200.integrations.vllm.fused_moe import WispMoEState  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    shape = wl.QWEN3_30B
    E, H, I, K = shape.experts, shape.hidden, shape.inter, shape.top_k
    g = torch.Generator().manual_seed(11)
    w13 = (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16)
    lo, hi = shard_range(E, rank, world)
    ex = EPExchange(H, 32 * K, dev)
    ex.configure(wait_ns=20_000_000_000)
    per = E // world
    paged = EPMoELayer(w13[lo:hi], w2[lo:hi], E, 8, "paged", dev, 0, exchange=ex)
    resident = EPMoELayer(w13[lo:hi], w2[lo:hi], E, per, "resident", dev, 1, exchange=ex)
    oracle = PagerOracle(per, 8)
    full = WispMoEState(w13, w2, E, "resident", dev, 0)
    full.prime_identity()
    gr = torch.Generator().manual_seed(100 + rank)
    ok = 1
    for step in range(6):
        # 16 tokens (128 pairs: tensor cores), 2 tokens (16 pairs: CUDA cores), mixed across ranks
        T = [16, 2, 16 if rank % 2 else 2, 32, 1, 7][step]
        w, ids = wl.softmax_topk(torch.randn(T, E, generator=gr), K)
        x = torch.randn(T, H, generator=gr).to(torch.bfloat16).to(dev)
        ref = full.forward(x, w.to(dev), ids.to(dev))
        for layer in (paged, resident):
            out = layer.forward(x, w.to(dev), ids.to(dev))
            layer.synchronize()
            if not torch.equal(out, ref):
                print(f"rank {rank} step {step} {layer.local.mode}: EP output differs", flush=True)
                ok = 0
            if layer is paged:
                R = sum(layer.last_counts)
                recv = ex.received(R)[2].reshape(-1).cpu().numpy().reshape(-1, 1)
                for r0, n in layer.last_runs:   # one pager call per run of same-class sources
                    forward_pager(oracle, recv[r0:r0 + n])
                s2e, tick, clock, stats = layer.local._read()
                if (s2e, tick, clock) != (oracle.slot_to_expert, oracle.lru_tick, oracle.lru_clock) or \
                        stats != oracle.stats():
                    print(f"rank {rank} step {step}: pager state differs from the oracle", flush=True)
                    ok = 0
    flag = torch.tensor([ok], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.barrier()
    paged.close()
    resident.close()
    ex.close()
    full.close()
    dist.destroy_process_group()
    if int(flag.item()) != 1:
        sys.exit(1)
    if rank == 0:
        print("ep multi-gpu ok", flush=True)


if __name__ == "__main__":
    main()
