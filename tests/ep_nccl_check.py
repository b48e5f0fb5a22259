"""Two-rank NCCL check of EPMoELayer (launched by tests/test_ep_gpu.py under
torch.distributed.run, one GPU per rank): every rank's EP output must be
byte-identical to a one-GPU layer over all experts on the same tokens."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from wisp_b200 import workloads as wl  # noqa: E402
from wisp_b200.expert_parallel import EPMoELayer, shard_range  # noqa: E402
from wisp_b200.integrations.vllm.fused_moe import WispMoEState  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    E, H, I, K = 16, 512, 256, 4
    g = torch.Generator().manual_seed(11)
    w13 = (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16)
    lo, hi = shard_range(E, rank, world)
    layer = EPMoELayer(w13[lo:hi], w2[lo:hi], E, 3, "paged", dev, 0)
    full = WispMoEState(w13, w2, E, "resident", dev, 0)
    full.prime_identity()
    gr = torch.Generator().manual_seed(100 + rank)
    ok = 1
    for step in range(5):
        # call sizes on both sides of the tensor-core threshold (74 pairs here), and mixed
        T = (20 if rank == 0 else 8) if step % 2 else 24
        w, ids = wl.softmax_topk(torch.randn(T, E, generator=gr), K)
        x = torch.randn(T, H, generator=gr).to(torch.bfloat16).to(dev)
        out = layer.forward(x, w.to(dev), ids.to(dev))
        ref = full.forward(x, w.to(dev), ids.to(dev))
        torch.cuda.synchronize()
        if not torch.equal(out, ref):
            print(f"rank {rank} step {step}: EP output differs", flush=True)
            ok = 0
    layer.local.synchronize()
    flag = torch.tensor([ok], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    layer.close()
    full.close()
    dist.destroy_process_group()
    if int(flag.item()) != 1:
        sys.exit(1)
    if rank == 0:
        print("ep nccl ok", flush=True)


if __name__ == "__main__":
    main()
