"""Seeded synthetic inputs for the paged fused-MoE layer.

The reference publishes no dataset for this path; its benches are
engine-level.  These generators give the shapes, sizes and value
distributions named in the benchmark configurations:

* ``qwen3_30b`` / ``mixtral_8x7b`` / ``qwen3_235b`` shapes (``MoEShape``);
* expert weights ``N(0, 0.02)`` in bf16, one seed per layer
  (``layer_weights``), laid out like vLLM's ``w13_weight [E, 2I, H]`` and
  ``w2_weight [E, H, I]`` (src/wisp/integrations/vllm/fused_moe.py:726-759);
* router logits ``N(0,1)`` plus a Zipf bias, softmax top-k with
  renormalisation (``logits_routing``), the Qwen3/Mixtral routing that
  ``select_experts`` computes at fused_moe.py:1054-1076;
* Zipf expert popularity with temporal reuse (``zipf_trace``) and uniform
  top-k (``uniform_topk``) for the multi-layer decode and prefill configs.

All randomness is drawn from explicit seeds so every arm (GPU kernels, CPU
oracle, golden fixtures) sees the same routing.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch


@dataclass(frozen=True)
class MoEShape:
    name: str
    hidden: int          # H
    inter: int           # I (moe_intermediate)
    experts: int         # E
    top_k: int           # k
    layers: int

    @property
    def expert_bytes(self) -> int:
        """bf16 bytes of one expert: w13 [2I,H] + w2 [H,I]."""
        return 3 * self.hidden * self.inter * 2


QWEN3_30B = MoEShape("qwen3-30b-a3b", 2048, 768, 128, 8, 48)
MIXTRAL_8X7B = MoEShape("mixtral-8x7b", 4096, 14336, 8, 2, 32)
QWEN3_235B = MoEShape("qwen3-235b-a22b", 4096, 1536, 128, 8, 94)


def layer_weights(shape: MoEShape, layer: int, seed0: int = 0, experts=None, std: float = 0.02):
    """CPU bf16 ``(w13 [E,2I,H], w2 [E,H,I])`` for one layer: torch
    ``manual_seed(seed0 + layer)``, then ``randn * std`` (w13 first)."""
    E = shape.experts if experts is None else experts
    g = torch.Generator().manual_seed(seed0 + layer)
    w13 = (torch.randn(E, 2 * shape.inter, shape.hidden, generator=g) * std).to(torch.bfloat16)
    w2 = (torch.randn(E, shape.hidden, shape.inter, generator=g) * std).to(torch.bfloat16)
    return w13, w2


def zipf_bias(E: int, s: float, seed: int) -> np.ndarray:
    """``b_e = -s * ln(1 + pi(e))`` with ``pi`` a seeded permutation, so that
    ``softmax(b)`` is the Zipf(s) pmf over a shuffled expert order."""
    perm = np.random.default_rng(seed).permutation(E)
    return (-s * np.log1p(perm.astype(np.float64))).astype(np.float32)


def softmax_topk(logits: torch.Tensor, k: int, renormalize: bool = True):
    """fp32 softmax over experts, top-k (descending weight), optional
    renormalisation; ids are int32.  Matches vLLM's softmax ``select_experts``
    semantics for Qwen3/Mixtral."""
    p = torch.softmax(logits.float(), dim=-1)
    w, ids = torch.topk(p, k, dim=-1)
    if renormalize:
        w = w / w.sum(dim=-1, keepdim=True)
    return w.contiguous(), ids.to(torch.int32).contiguous()


def router_logits(T: int, E: int, seed: int = 0, zipf_s: float = 1.1) -> torch.Tensor:
    """Config-1 router logits ``N(0,1) + zipf_bias`` (fp32, CPU)."""
    g = torch.Generator().manual_seed(seed + 1)
    return torch.randn(T, E, generator=g) + torch.from_numpy(zipf_bias(E, zipf_s, seed))


def logits_routing(T: int, E: int, k: int, seed: int = 0, zipf_s: float = 1.1):
    """Config-1 routing: logits ``N(0,1) + zipf_bias`` -> softmax top-k."""
    return softmax_topk(router_logits(T, E, seed, zipf_s), k)


def hidden_states(T: int, H: int, seed: int = 0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed + 2)
    return torch.randn(T, H, generator=g).to(torch.bfloat16)


def _gumbel_topk(logp: np.ndarray, k: int, rng: np.random.Generator, n: int) -> np.ndarray:
    """``n`` draws of ``k`` distinct experts, sampled without replacement with
    probabilities ``exp(logp)`` (Gumbel top-k)."""
    gum = rng.gumbel(size=(n, logp.shape[0]))
    return np.argpartition(-(logp[None, :] + gum), k - 1, axis=1)[:, :k]


def zipf_trace(steps: int, layers: int, batch: int, E: int, k: int, s: float,
               p_reuse: float, seed: int = 0):
    """Multi-layer decode routing trace.

    Per layer a Zipf(s) popularity over a seeded expert permutation; token
    ``(t, b)`` reuses ``(t-1, b)``'s expert set at that layer with
    probability ``p_reuse``, else draws ``k`` distinct experts by popularity.
    Weights are the renormalised softmax of ``N(0,1)`` logits over the chosen
    set, ids sorted by weight descending.

    Returns ``ids [steps, layers, batch, k] int32`` and ``w`` (fp32, same
    shape)."""
    rng = np.random.default_rng(seed)
    ids = np.empty((steps, layers, batch, k), np.int32)
    for layer in range(layers):
        logp = zipf_bias(E, s, seed * 1000 + layer).astype(np.float64)
        draws = _gumbel_topk(logp, k, rng, steps * batch).reshape(steps, batch, k)
        reuse = rng.random((steps, batch)) < p_reuse
        for t in range(steps):
            if t > 0:
                r = reuse[t]
                draws[t, r] = ids[t - 1, layer, r]
            ids[t, layer] = draws[t]
    logits = rng.standard_normal((steps, layers, batch, k)).astype(np.float32)
    w = np.exp(logits - logits.max(-1, keepdims=True))
    w /= w.sum(-1, keepdims=True)
    order = np.argsort(-w, axis=-1, kind="stable")
    w = np.take_along_axis(w, order, -1).astype(np.float32)
    ids = np.take_along_axis(ids, order, -1)
    return ids, w


def uniform_topk(T: int, E: int, k: int, seed: int = 0):
    """Uniform-random ``k`` distinct experts per token with renormalised
    softmax weights (the prefill configuration)."""
    rng = np.random.default_rng(seed)
    ids = np.argsort(rng.random((T, E)), axis=1)[:, :k].astype(np.int32)
    logits = rng.standard_normal((T, k)).astype(np.float32)
    w = np.exp(logits - logits.max(-1, keepdims=True))
    w /= w.sum(-1, keepdims=True)
    order = np.argsort(-w, axis=-1, kind="stable")
    return np.take_along_axis(ids, order, -1), np.take_along_axis(w, order, -1).astype(np.float32)
