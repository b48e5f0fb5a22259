"""fp32 restatement of the reference layer's expert math (CPU oracle).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

The reference computes the layer with vLLM's ``fused_experts`` on the slot
scratch plus ``expert_map`` (src/wisp/integrations/vllm/fused_moe.py:1106-1118
and :1155-1168).  Its semantics, per token ``t`` and routed position ``k``
with expert ``e = topk_ids[t, k]`` and weight ``w = topk_weights[t, k]``:

    h      = W13[e] @ x[t]            (fp32 accumulate; stored bf16)
    g, u   = h[:I], h[I:]             (gate = first I rows of w13, up = next I)
    a      = silu(g) * u              (silu(g) stored bf16 before the product --
                                       vLLM's silu_and_mul --, a stored bf16)
    y      = (W2[e] @ a) * w          (fp32 accumulate, weight applied in fp32,
                                       stored bf16)
    out[t] = sum over k, in routing order, of y   (vLLM's moe_sum: for top-k
                                       <= 4 every partial sum stored bf16, above
                                       an fp32 sum; stored bf16)

The storage points are pinned by golden outputs of vLLM's ``fused_experts``
(vllm 0.22, its Triton kernels run on a GPU by
``tests/golden/make_vllm_golden.py``; ``tests/test_vllm_golden.py``): with
them this restatement matches vLLM's bytes on 99-100 % of the elements at
top-2 and top-4 and within mean-rel 5e-4 at top-8 (fp32 accumulation order).

``moe_reference(..., emulate_storage=True)`` reproduces those bf16 storage
points (including the bf16 output) with fp32 arithmetic between them: the
tolerance target of the parity tests.  ``emulate_storage=False`` keeps
everything in fp32, output included (rounding that output to bf16 alone
already costs about 1.4e-3 mean relative error).
"""
from __future__ import annotations

import torch


def _bf16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(torch.float32)


def moe_reference(x, w13, w2, topk_weights, topk_ids, emulate_storage: bool = True,
                  return_partials: bool = False):
    """x [T,H] bf16; w13 [E,2I,H]; w2 [E,H,I] (bf16, indexed by GLOBAL expert
    id); topk_weights [T,k] fp32; topk_ids [T,k].  Returns ``[T,H]`` as fp32
    values; with ``return_partials`` also the per-(t,k) weighted expert
    outputs ``[T,k,H]``."""
    x = x.float()
    T, K = topk_ids.shape
    H = x.shape[1]
    I = w2.shape[2]
    r = _bf16 if emulate_storage else (lambda v: v)
    ids = topk_ids.long()
    tw = topk_weights.float()
    Y = torch.zeros(T, K, H, dtype=torch.float32)
    for e in torch.unique(ids).tolist():
        rows, cols = (ids == e).nonzero(as_tuple=True)
        h = r(x[rows] @ w13[e].float().T)                # [n, 2I]
        g, u = h[:, :I], h[:, I:]
        a = r(r(g * torch.sigmoid(g)) * u)               # [n, I]
        y = (a @ w2[e].float().T) * tw[rows, cols][:, None]
        Y[rows, cols] = r(y)
    out = torch.zeros(T, H, dtype=torch.float32)
    rs = r if K <= 4 else (lambda v: v)                  # bf16 partial sums up to top-4
    for k in range(K):                                   # routing order
        out = rs(out + Y[:, k])
    out = r(out)                                         # the layer output is stored bf16
    return (out, Y) if return_partials else out


def compare(out_bf16: torch.Tensor, ref_fp32: torch.Tensor) -> dict:
    """Parity figures used by the tests: max-abs and mean-relative error
    (``mean|a-b| / mean|b|``) of a bf16 output against an fp32 reference."""
    a = out_bf16.float()
    d = (a - ref_fp32).abs()
    return {"max_abs": float(d.max()) if d.numel() else 0.0,
            "mean_rel": float(d.mean() / ref_fp32.abs().mean().clamp_min(1e-30)) if d.numel() else 0.0}
