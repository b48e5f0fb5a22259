"""Golden outputs of vLLM's block-quantised FP8 ``fused_experts`` -- the expert
compute of the reference's FP8 paging path (src/wisp/integrations/vllm/
fused_moe_fp8.py:302-312: slot scratch w13 / w2 in float8_e4m3fn with their
per-128x128-block fp32 scales, global ``topk_ids``, ``expert_map`` to the
slots, dynamic per-token-group activation quantisation, Triton backend) --
for seeded cases, computed by vLLM's own kernels on a GPU.

Inputs are not stored: ``case_tensors`` regenerates them from the case's seed
(CPU ``torch.Generator``); the file keeps the seeds, shapes, float64 checksums
of the inputs and vLLM's bf16 outputs.

    VLLM_USE_DEEP_GEMM=0 python tests/golden/make_vllm_fp8_golden.py OUT.npz   # needs a GPU and vLLM
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

BLOCK = 128
FP8_MAX = 448.0

# (name, E, H, I, T, K, cap, seed)
CASES = [
    ("fp8_resident_e16_h512_t5_k4", 16, 512, 256, 5, 4, 16, 201),
    ("fp8_paged_e32_h2048_t3_k8", 32, 2048, 768, 3, 8, 24, 202),
    ("fp8_paged_e32_h1024_t8_k2", 32, 1024, 512, 8, 2, 20, 203),
    ("fp8_resident_e16_h2048_t16_k8", 16, 2048, 768, 16, 8, 16, 204),
]


def quantize_blocks(w: torch.Tensor):
    """[E, N, K] float -> (float8_e4m3fn weights, fp32 scales [E, N/128, K/128])
    with scale = block amax / 448 (the dequantisation factor vLLM calls
    weight_scale_inv)."""
    E, N, K = w.shape
    b = w.reshape(E, N // BLOCK, BLOCK, K // BLOCK, BLOCK)
    amax = b.abs().amax(dim=(2, 4)).clamp_min(1e-12)
    scale = (amax / FP8_MAX).to(torch.float32)
    q = (b / scale[:, :, None, :, None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q.reshape(E, N, K), scale


def case_tensors(E, H, I, T, K, cap, seed):
    g = torch.Generator().manual_seed(seed)
    w13, s13 = quantize_blocks(torch.randn(E, 2 * I, H, generator=g) * 0.02)
    w2, s2 = quantize_blocks(torch.randn(E, H, I, generator=g) * 0.02)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g)
    w, ids = torch.softmax(logits, -1).topk(K, -1)
    w = (w / w.sum(-1, keepdim=True)).to(torch.float32)
    ids = ids.to(torch.int32)
    routed = sorted(set(ids.reshape(-1).tolist()))
    assert len(routed) <= cap
    others = [e for e in torch.randperm(E, generator=g).tolist() if e not in routed]
    resident = routed + others[: cap - len(routed)]
    slots = torch.randperm(cap, generator=g).tolist()
    emap = torch.full((E,), -1, dtype=torch.int32)
    for e, s in zip(resident, slots):
        emap[e] = s
    return w13, w2, s13, s2, x, w, ids, emap


def checksum(*ts):
    return np.array([float(t.to(torch.float64).sum()) for t in ts])


def main(out_path):
    os.environ.setdefault("VLLM_USE_DEEP_GEMM", "0")
    from vllm.model_executor.layers.fused_moe.activation import MoEActivation
    from vllm.model_executor.layers.fused_moe.config import fp8_w8a8_moe_quant_config
    from vllm.model_executor.layers.fused_moe.fused_moe import fused_experts

    dev = torch.device("cuda:0")
    data = {"names": np.array([c[0] for c in CASES]), "cases": np.array([c[1:] for c in CASES], dtype=np.int64)}
    for name, E, H, I, T, K, cap, seed in CASES:
        w13, w2, s13, s2, x, w, ids, emap = case_tensors(E, H, I, T, K, cap, seed)
        sw13 = torch.zeros(cap, 2 * I, H, dtype=torch.float8_e4m3fn)
        sw2 = torch.zeros(cap, H, I, dtype=torch.float8_e4m3fn)
        ss13 = torch.ones(cap, *s13.shape[1:], dtype=torch.float32)
        ss2 = torch.ones(cap, *s2.shape[1:], dtype=torch.float32)
        for e in range(E):
            if emap[e] >= 0:
                sw13[emap[e]], sw2[emap[e]] = w13[e], w2[e]
                ss13[emap[e]], ss2[emap[e]] = s13[e], s2[e]
        qc = fp8_w8a8_moe_quant_config(w1_scale=ss13.to(dev), w2_scale=ss2.to(dev), a1_scale=None,
                                       a2_scale=None, block_shape=[BLOCK, BLOCK])
        out = fused_experts(hidden_states=x.to(dev), w1=sw13.to(dev), w2=sw2.to(dev), topk_weights=w.to(dev),
                            topk_ids=ids.to(dev), inplace=False, activation=MoEActivation.SILU,
                            global_num_experts=E, expert_map=emap.to(dev), quant_config=qc)
        torch.cuda.synchronize()
        data[name + "/out"] = out.cpu().view(torch.int16).numpy()
        data[name + "/checksum"] = checksum(w13, w2, s13, s2, x, w, ids, emap)
        print(name, "ok", flush=True)
    data["vllm_version"] = np.array(__import__("vllm").__version__)
    np.savez_compressed(out_path, **data)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "tests/golden/vllm_fp8_fused_experts.npz")
