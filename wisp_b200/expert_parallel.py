"""Expert-parallel paged MoE layer over NCCL all-to-all.

Rank ``r`` of ``P`` owns experts ``[r*E/P, (r+1)*E/P)`` in its own pinned host
memory and pages only those into its own HBM slots.  A forward:

1. routes and packs (``wisp_ep_dispatch``): every (token, k) pair goes to its
   owner, pairs of one owner in (t, k) order, each with its local expert id
   and routing weight;
2. exchanges the per-owner row counts (and whether any rank saw an id out of
   range, so every rank raises together rather than leaving the others
   waiting in the next collective), then the rows and their records;
3. runs the owner's paged layer on the rows it received, one expert per row
   (``top_k`` 1): the pager sees the received rows in (source rank, pair)
   order, so a rank's slot maps and hit/miss sequence are those of a one-GPU
   layer over its shard fed that sequence.  The rows of each source are
   computed in the numeric class (CUDA-core or tensor-core kernels) that a
   one-GPU call of that source's size would use: the counts exchange carries
   every rank's pair count, and the owner forces that class for the call
   (sources of both classes: one call per run of sources of one class, so
   the pager then sees that many calls);
4. returns the weighted rows to their source and sums them over k in routing
   order (``wisp_ep_combine``).

Each (t, k) row is computed with the same arithmetic as on one GPU and the
combine adds the same values in the same order, so the output is
byte-identical to the one-GPU layer over all experts.

This path has no counterpart in the reference (one GPU per model there); it
is the expert-parallel sharding of the layer behind ``install_wisp_moe``.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _lib


@dataclass
class DispatchPlan:
    """One forward's send side: rows in owner order and where each pair went."""
    num_tokens: int
    top_k: int
    send_x: torch.Tensor        # [T*k, H] bf16, owner order
    send_meta: torch.Tensor     # [T*k, 2] int32: local expert id, weight bits
    pair_pos: torch.Tensor      # [T*k] int32: send row of pair t*k+j
    counts_dev: torch.Tensor    # [world + 1] int64: rows per owner, then bad ids
    send_counts: list[int] | None = None
    recv_counts: list[int] | None = None
    src_pairs: list[int] | None = None   # every source rank's (token, k) pair count


class EPMoELayer:
    """One MoE layer sharded over the ranks of ``group`` (default: the world).

    ``cpu_w13_shard [E/P, 2I, H]`` and ``cpu_w2_shard [E/P, H, I]`` are this
    rank's experts (bf16 host masters, pinned here if they are not).
    ``cap_experts`` is this rank's slot count (``WISP_CAP_EXPERTS`` per GPU);
    ``mode`` is ``"paged"`` or ``"resident"``.  ``local`` replaces the
    one-GPU layer that computes the received rows (tests)."""

    def __init__(self, cpu_w13_shard: torch.Tensor | None, cpu_w2_shard: torch.Tensor | None,
                 num_experts: int, cap_experts: int, mode: str = "paged", device=None,
                 layer_idx: int = 0, group=None, rank: int | None = None,
                 world_size: int | None = None, local=None) -> None:
        self.group = group
        self.world = int(world_size if world_size is not None else dist.get_world_size(group))
        self.rank = int(rank if rank is not None else dist.get_rank(group))
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not split evenly over {self.world} ranks")
        self.num_experts = int(num_experts)
        self.experts_per_rank = self.num_experts // self.world
        if local is None:
            from .integrations.vllm.fused_moe import WispMoEState
            if cpu_w13_shard.shape[0] != self.experts_per_rank:
                raise ValueError(f"rank {self.rank} shard has {cpu_w13_shard.shape[0]} experts, "
                                 f"expected {self.experts_per_rank}")
            local = WispMoEState(cpu_w13_shard, cpu_w2_shard, cap_experts, mode, device, layer_idx)
            if mode == "resident":  # the whole shard in HBM (cap == experts per rank)
                local.prime_identity()
        self.local = local
        self.device = torch.device(device) if device is not None else getattr(local, "device", None)
        self.hidden = int(getattr(local, "hidden_size", 0))

    # ---- phases (forward runs them in order; tests may run them per rank) ----
    def begin(self, x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor) -> DispatchPlan:
        """Route and pack this rank's pairs (no communication)."""
        T, K = int(topk_ids.shape[0]), int(topk_ids.shape[-1])
        H = int(x.shape[-1])
        if x.dtype != torch.bfloat16:
            raise TypeError("wisp_b200 expert parallelism moves bf16 hidden states; got %s" % x.dtype)
        x = x.contiguous()
        w = topk_weights.to(torch.float32).contiguous()
        ids = topk_ids if topk_ids.dtype in (torch.int32, torch.int64) else topk_ids.to(torch.int64)
        ids = ids.contiguous()
        P = T * K
        send_x = torch.empty((P, H), dtype=torch.bfloat16, device=x.device)
        send_meta = torch.empty((P, 2), dtype=torch.int32, device=x.device)
        pos = torch.empty((P,), dtype=torch.int32, device=x.device)
        counts = torch.empty((self.world + 1,), dtype=torch.int64, device=x.device)
        self._route_pack(x, w, ids, T, K, H, send_x, send_meta, counts, pos)
        return DispatchPlan(T, K, send_x, send_meta, pos, counts)

    def _route_pack(self, x, w, ids, T, K, H, send_x, send_meta, counts, pos) -> None:
        _lib.check(_lib.lib().wisp_ep_dispatch(
            x.data_ptr(), ids.data_ptr(), int(ids.dtype == torch.int64), w.data_ptr(), T, K, H,
            self.experts_per_rank, self.world, send_x.data_ptr(), send_meta.data_ptr(),
            counts.data_ptr(), pos.data_ptr(), _lib.stream_ptr(torch.cuda.current_stream(x.device))),
            "wisp_ep_dispatch")

    def exchange_counts(self, plan: DispatchPlan) -> None:
        """All-to-all of (rows for you, ids out of range here, this rank's
        pair count); one host read."""
        n = plan.counts_dev[: self.world]
        bad = plan.counts_dev[self.world:].expand(self.world)
        pairs = torch.full_like(n, plan.num_tokens * plan.top_k)
        send = torch.stack([n, bad, pairs], dim=1).contiguous()
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        host = torch.cat([send, recv]).cpu().tolist()
        plan.send_counts = [int(r[0]) for r in host[: self.world]]
        plan.recv_counts = [int(r[0]) for r in host[self.world:]]
        plan.src_pairs = [int(r[2]) for r in host[self.world:]]
        if any(int(r[1]) for r in host[self.world:]):  # (every rank's flag, this one's included)
            raise _lib.WispError(_lib.WISP_ERR_BAD_EXPERT,
                                 f"wisp: a rank routed an expert id outside [0, {self.num_experts})")

    def exchange_rows(self, plan: DispatchPlan) -> tuple[torch.Tensor, torch.Tensor]:
        R = sum(plan.recv_counts)
        H = plan.send_x.shape[1]
        recv_x = torch.empty((R, H), dtype=plan.send_x.dtype, device=plan.send_x.device)
        recv_meta = torch.empty((R, 2), dtype=torch.int32, device=plan.send_x.device)
        dist.all_to_all_single(recv_x, plan.send_x, plan.recv_counts, plan.send_counts, group=self.group)
        dist.all_to_all_single(recv_meta, plan.send_meta, plan.recv_counts, plan.send_counts,
                               group=self.group)
        return recv_x, recv_meta

    def compute(self, recv_x: torch.Tensor, recv_meta: torch.Tensor, recv_counts: list[int] | None = None,
                src_pairs: list[int] | None = None) -> torch.Tensor:
        """This rank's experts on the rows it received (one expert per row),
        each source's rows in the numeric class of a one-GPU call of that
        source's size (``recv_counts`` / ``src_pairs`` per source rank; without
        them the class follows the received row count)."""
        R = int(recv_x.shape[0])
        recv_y = torch.empty_like(recv_x)
        if not R:
            return recv_y
        w = recv_meta.view(torch.float32)[:, 1:2]
        ids = recv_meta[:, 0:1]
        classify = getattr(self.local, "compute_class", None)
        if classify is None or recv_counts is None or src_pairs is None:
            self.local.forward(recv_x, w, ids, out=recv_y)
            return recv_y
        runs = []  # [class, first row, rows]: consecutive sources of one class
        row = 0
        for cnt, pairs in zip(recv_counts, src_pairs):
            cls = classify(int(pairs))
            if cnt and runs and runs[-1][0] == cls:
                runs[-1][2] += cnt
            elif cnt:
                runs.append([cls, row, cnt])
            row += cnt
        try:
            for cls, r0, n in runs:
                self.local.configure(compute_class=cls)
                self.local.forward(recv_x[r0:r0 + n], w[r0:r0 + n], ids[r0:r0 + n], out=recv_y[r0:r0 + n])
        finally:
            self.local.configure(compute_class="auto")
        return recv_y

    def exchange_back(self, plan: DispatchPlan, recv_y: torch.Tensor) -> torch.Tensor:
        back = torch.empty_like(plan.send_x)
        dist.all_to_all_single(back, recv_y, plan.send_counts, plan.recv_counts, group=self.group)
        return back

    def finish(self, plan: DispatchPlan, back: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Routing-order sum of the returned rows."""
        if out is None:
            out = torch.empty((plan.num_tokens, back.shape[1]), dtype=back.dtype, device=back.device)
        self._combine(back, plan.pair_pos, plan.num_tokens, plan.top_k, out)
        return out

    def _combine(self, back, pos, T, K, out) -> None:
        _lib.check(_lib.lib().wisp_ep_combine(
            back.data_ptr(), pos.data_ptr(), T, K, int(back.shape[1]), out.data_ptr(),
            _lib.stream_ptr(torch.cuda.current_stream(back.device))), "wisp_ep_combine")

    # ---- the forward -------------------------------------------------------------
    def forward(self, x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """x [T,H] bf16, topk_weights [T,k], topk_ids [T,k] global expert ids;
        returns [T,H] bf16.  Collective: every rank of the group calls it."""
        plan = self.begin(x, topk_weights, topk_ids)
        self.exchange_counts(plan)
        recv_x, recv_meta = self.exchange_rows(plan)
        recv_y = self.compute(recv_x, recv_meta, plan.recv_counts, plan.src_pairs)
        back = self.exchange_back(plan, recv_y)
        return self.finish(plan, back, out)

    def close(self) -> None:
        if hasattr(self.local, "close"):
            self.local.close()


def shard_range(num_experts: int, rank: int, world: int) -> tuple[int, int]:
    """Experts owned by ``rank``: ``[lo, hi)``."""
    per = num_experts // world
    return rank * per, (rank + 1) * per


__all__ = ["EPMoELayer", "DispatchPlan", "shard_range"]
