"""fp32 restatement of the reference's block-FP8 expert math (CPU oracle).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

The reference's FP8 paging path computes the layer with vLLM's
``fused_experts`` on float8_e4m3fn slot scratch with per-128x128-block fp32
scales (src/wisp/integrations/vllm/fused_moe_fp8.py:302-312, block-quantised
W8A8, Triton backend).  Per token ``t`` and routed position ``k`` (expert
``e``, weight ``w``), with 128-wide groups along every reduction:

    xq, xs = quant(x[t])          per group of 128: s = max(amax, 1e-10) / 448 (a
                                  division: the product with 1/448 differs in
                                  the last bit for some amax, which moves whole
                                  groups of codes), q = clamp(x / s, +-448) in
                                  float8_e4m3fn
    h[n]   = sum over groups b of (xq_b . W13q[e][n]_b) * xs_b * S13[e][n/128][b]
                                  (fp32; stored bf16)
    a      = silu(g) * u          (silu(g) stored bf16 first, a stored bf16)
    aq, as = quant(a)
    y[n]   = (sum over b of (aq_b . W2q[e][n]_b) * as_b * S2[e][n/128][b]) * w
                                  (fp32; stored bf16)
    out[t] = routing-order sum of y over k (bf16 partial sums for top-k <= 4)

Pinned by golden outputs of vLLM's own FP8 kernels
(``tests/golden/make_vllm_fp8_golden.py``, ``tests/test_fp8.py``): bit-exact
on every golden case.
"""
from __future__ import annotations

import torch

BLOCK = 128
FP8_MAX = 448.0


def _bf16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(torch.float32)


def quant_groups(v: torch.Tensor):
    """[n, C] float -> (fp8 values as float [n, C], scales [n, C/128])."""
    n, C = v.shape
    g = v.float().reshape(n, C // BLOCK, BLOCK)
    amax = g.abs().amax(dim=2).clamp_min(1e-10)
    s = amax / FP8_MAX
    q = (g / s[:, :, None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn).float()
    return q.reshape(n, C), s


def _block_gemm(aq, as_, wq, ws):
    """aq [n, C] fp8 values, as_ [n, C/128], wq [N, C] fp8 values, ws [N/128, C/128]
    -> [n, N] fp32: sum over groups of the group dot product times both scales."""
    n, C = aq.shape
    N = wq.shape[0]
    nb = C // BLOCK
    out = torch.zeros(n, N, dtype=torch.float32)
    wsr = ws.repeat_interleave(BLOCK, dim=0)[:N]  # [N, nb]
    for b in range(nb):
        part = aq[:, b * BLOCK:(b + 1) * BLOCK] @ wq[:, b * BLOCK:(b + 1) * BLOCK].T
        out += part * as_[:, b:b + 1] * wsr[:, b][None, :]
    return out


def moe_reference_fp8(x, w13q, w2q, s13, s2, topk_weights, topk_ids):
    """x [T,H] bf16; w13q [E,2I,H] / w2q [E,H,I] float8_e4m3fn; s13 [E,2I/128,H/128]
    / s2 [E,H/128,I/128] fp32 (indexed by GLOBAL expert id); returns [T,H] fp32
    values of the bf16 output."""
    T, K = topk_ids.shape
    H = x.shape[1]
    I = w2q.shape[2]
    ids = topk_ids.long()
    tw = topk_weights.float()
    xq, xs = quant_groups(x.float())
    Y = torch.zeros(T, K, H, dtype=torch.float32)
    for e in torch.unique(ids).tolist():
        rows, cols = (ids == e).nonzero(as_tuple=True)
        h = _bf16(_block_gemm(xq[rows], xs[rows], w13q[e].float(), s13[e]))
        g, u = h[:, :I], h[:, I:]
        a = _bf16(_bf16(g * torch.sigmoid(g)) * u)
        aq, as_ = quant_groups(a)
        y = _block_gemm(aq, as_, w2q[e].float(), s2[e]) * tw[rows, cols][:, None]
        Y[rows, cols] = _bf16(y)
    out = Y[:, 0].clone()
    for k in range(1, K):
        out = out + Y[:, k]
        if K <= 4:
            out = _bf16(out)
    return _bf16(out)


__all__ = ["moe_reference_fp8", "quant_groups", "BLOCK", "FP8_MAX"]
