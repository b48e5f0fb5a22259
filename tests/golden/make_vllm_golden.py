"""Golden outputs of vLLM's ``fused_experts`` -- the expert compute the
reference's paged forward calls (src/wisp/integrations/vllm/fused_moe.py:
1106-1118 and 1155-1167: slot scratch ``w13`` / ``w2``, global ``topk_ids``,
``expert_map`` from expert to slot, ``global_num_experts`` = E, unquantized
bf16, SiLU) -- for seeded cases, computed by vLLM's own Triton MoE kernels on
a GPU.  vLLM is the reference's pinned dependency for this math (the image's
vllm 0.22); the reference holds no numeric fixture of its own.

Inputs are not stored: ``case_tensors`` regenerates them from the case's seed
with a CPU ``torch.Generator`` (the same torch build gives the same values);
the file keeps the seeds, shapes, float64 checksums of the inputs and vLLM's
bf16 outputs, so the tests can rebuild the inputs and know they did.

    python tests/golden/make_vllm_golden.py OUT.npz      # needs a GPU and vLLM
"""
from __future__ import annotations

import sys

import numpy as np
import torch

# (name, E, H, I, T, K, cap, seed): the experts (every routed one, then
# others up to cap) sit in a seeded permutation of the slots, as the pager
# leaves them; cap == E holds every expert, as in a resident layer
CASES = [
    ("resident_e16_h512_t5_k4", 16, 512, 256, 5, 4, 16, 101),
    ("paged_e32_h2048_t3_k8", 32, 2048, 768, 3, 8, 24, 102),
    ("paged_e32_h1024_t8_k2", 32, 1024, 512, 8, 2, 20, 103),
    ("resident_e16_h2048_t16_k8", 16, 2048, 768, 16, 8, 16, 104),
    ("resident_e8_h1024_t40_k2", 8, 1024, 512, 40, 2, 8, 105),
]


def case_tensors(E, H, I, T, K, cap, seed):
    """Weights, hidden states, routing and the expert -> slot map of a case.
    Routing draws top-k of softmax(randn) logits; with cap < E every routed
    expert gets a slot and the others fill the rest, all in a seeded order."""
    g = torch.Generator().manual_seed(seed)
    w13 = (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g)
    w, ids = torch.softmax(logits, -1).topk(K, -1)
    w = (w / w.sum(-1, keepdim=True)).to(torch.float32)
    ids = ids.to(torch.int32)
    routed = sorted(set(ids.reshape(-1).tolist()))
    assert len(routed) <= cap, "a case must route to at most cap experts"
    others = [e for e in torch.randperm(E, generator=g).tolist() if e not in routed]
    resident = routed + others[: cap - len(routed)]
    slots = torch.randperm(cap, generator=g).tolist()
    emap = torch.full((E,), -1, dtype=torch.int32)
    for e, s in zip(resident, slots):
        emap[e] = s
    return w13, w2, x, w, ids, emap


def checksum(*ts):
    return np.array([float(t.double().sum()) for t in ts])


def main(out_path):
    from vllm.model_executor.layers.fused_moe.activation import MoEActivation
    from vllm.model_executor.layers.fused_moe.fused_moe import fused_experts

    dev = torch.device("cuda:0")
    data = {"names": np.array([c[0] for c in CASES]), "cases": np.array([c[1:] for c in CASES], dtype=np.int64)}
    for name, E, H, I, T, K, cap, seed in CASES:
        w13, w2, x, w, ids, emap = case_tensors(E, H, I, T, K, cap, seed)
        s13 = torch.zeros(cap, 2 * I, H, dtype=torch.bfloat16)
        s2 = torch.zeros(cap, H, I, dtype=torch.bfloat16)
        for e in range(E):
            if emap[e] >= 0:
                s13[emap[e]] = w13[e]
                s2[emap[e]] = w2[e]
        out = fused_experts(hidden_states=x.to(dev), w1=s13.to(dev), w2=s2.to(dev),
                            topk_weights=w.to(dev), topk_ids=ids.to(dev), inplace=False,
                            activation=MoEActivation.SILU, global_num_experts=E, expert_map=emap.to(dev))
        torch.cuda.synchronize()
        data[name + "/out"] = out.cpu().view(torch.int16).numpy()
        data[name + "/checksum"] = checksum(w13, w2, x, w, ids, emap)
        print(name, "ok", flush=True)
    data["vllm_version"] = np.array(__import__("vllm").__version__)
    np.savez_compressed(out_path, **data)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "tests/golden/vllm_fused_experts.npz")
