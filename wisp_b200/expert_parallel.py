"""Expert-parallel paged MoE layer, exchanging tokens over peer memory.

Rank ``r`` of ``P`` owns experts ``[r*E/P, (r+1)*E/P)`` in its own pinned host
memory and pages only those into its own HBM slots.  A forward:

1. ``dispatch`` (one kernel): every (token, k) pair goes to its owner --
   the kernel stores the token's row and a record (local expert id, routing
   weight, pair index) straight into the owner's receive segment over
   NVLink, pairs of one owner in (t, k) order, then publishes its counts;
2. ``receive`` (one kernel, then the host reads the counts): the owner waits
   for every source, compacts the rows and learns how many it got -- the
   only host round trip of the exchange.  The rows keep their run of
   consecutive same-class sources (below) and are ordered by local expert
   within a run, stably, so a run pages each of its experts once;
3. the owner's paged layer runs on those rows, one expert per row (``top_k``
   1): a rank's slot maps and hit/miss sequence are those of a one-GPU layer
   over its shard fed the rows in that order.  The rows of each source are
   computed in the numeric class
   (CUDA-core or tensor-core kernels) that a one-GPU call of that source's
   size would use: the receive reports every source's pair count, and the
   owner forces that class for the call (sources of both classes: one call
   per run of sources of one class, so the pager then sees that many calls);
4. ``send_back`` (one kernel) stores each weighted row into its source's
   return buffer at the pair's index, and ``combine`` (one kernel) waits for
   every owner and sums each token's k rows in routing order.

Each (t, k) row is computed with the same arithmetic as on one GPU and the
combine adds the same values in the same order, so the output is
byte-identical to the one-GPU layer over all experts.  No collective library
runs on the data path: ``torch.distributed`` only all-gathers the CUDA IPC
handles once, when the exchange is built.

This path has no counterpart in the reference (one GPU per model there); it
is the expert-parallel sharding of the layer behind ``install_wisp_moe``.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib


def _device_tensor(ptr: int, numel: int, dtype: torch.dtype, device) -> torch.Tensor:
    from .integrations.vllm.fused_moe import _device_view
    esize = torch.empty((), dtype=dtype).element_size()
    return _device_view(ptr, numel * esize, dtype, (numel,), device)


class EPExchange:
    """This rank's peer-memory exchange for an expert-parallel group.

    One exchange serves every layer of a model (the layers run one after
    another).  ``max_pairs`` bounds one call's (token, k) pairs on any rank;
    ``hidden`` is the row width.  Build it collectively (every rank of
    ``group``); :meth:`emulated` builds all ranks of a group inside one
    process on one device (tests)."""

    def __init__(self, hidden: int, max_pairs: int, device=None, group=None, rank: int | None = None,
                 world: int | None = None, _connect: bool = True) -> None:
        self.group = group
        self.world = int(world if world is not None else dist.get_world_size(group))
        self.rank = int(rank if rank is not None else dist.get_rank(group))
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.hidden, self.max_pairs = int(hidden), int(max_pairs)
        L = _lib.lib()
        h = ctypes.c_void_p()
        _lib.check(L.wisp_ep_group_create(self.rank, self.world, self.device.index, self.max_pairs,
                                          self.hidden, ctypes.byref(h)), "wisp_ep_group_create")
        self._h = h
        ptrs = [ctypes.c_void_p() for _ in range(4)]
        _lib.check(L.wisp_ep_group_buffers(h, *[ctypes.byref(p) for p in ptrs]), "wisp_ep_group_buffers")
        n = self.world * self.max_pairs
        self.x_recv = _device_tensor(ptrs[0].value, n * self.hidden, torch.bfloat16, self.device).view(n, self.hidden)
        self.ids_recv = _device_tensor(ptrs[1].value, n, torch.int32, self.device).view(n, 1)
        self.w_recv = _device_tensor(ptrs[2].value, n, torch.float32, self.device).view(n, 1)
        self.y_recv = _device_tensor(ptrs[3].value, n * self.hidden, torch.bfloat16, self.device).view(n, self.hidden)
        self.launches = 0
        if _connect:
            buf = (ctypes.c_char * 64)()
            _lib.check(L.wisp_ep_group_ipc_handle(h, buf), "wisp_ep_group_ipc_handle")
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(buf), group=group)
            _lib.check(L.wisp_ep_group_connect(h, b"".join(handles)), "wisp_ep_group_connect")

    @classmethod
    def emulated(cls, world: int, hidden: int, max_pairs: int, device) -> list["EPExchange"]:
        """``world`` ranks of one group in this process, on one device: rank r's
        kernels store into the other ranks' buffers directly.  Issue every
        rank's ``dispatch`` before any ``receive`` and every ``send_back``
        before any ``combine`` (the waits then find their data already there)."""
        exs = [cls(hidden, max_pairs, device, rank=r, world=world, _connect=False) for r in range(world)]
        arr = (ctypes.c_void_p * world)(*[e._h.value for e in exs])
        for e in exs:
            _lib.check(_lib.lib().wisp_ep_group_connect_local(e._h, arr), "wisp_ep_group_connect_local")
        return exs

    def configure(self, wait_ns: int) -> None:
        _lib.check(_lib.lib().wisp_ep_group_config(self._h, int(wait_ns)), "wisp_ep_group_config")

    def _stream(self) -> int:
        return _lib.stream_ptr(torch.cuda.current_stream(self.device))

    # ---- the four steps ---------------------------------------------------------
    def dispatch(self, x: torch.Tensor, w: torch.Tensor, ids: torch.Tensor, experts_per_rank: int) -> None:
        T, K = int(ids.shape[0]), int(ids.shape[-1])
        _lib.check(_lib.lib().wisp_ep_dispatch(
            self._h, x.data_ptr(), ids.data_ptr(), int(ids.dtype == torch.int64), w.data_ptr(), T, K,
            int(experts_per_rank), self._stream()), "wisp_ep_dispatch")
        self.launches += 1

    def receive(self, class_min_pairs: int = 0) -> tuple[list[int], list[int]]:
        """Rows from each source and each source's pair count (host lists);
        raises on every rank alike when any rank routed an id out of range.
        The rows are compacted by run of consecutive same-class sources
        (sources of at least ``class_min_pairs`` pairs are one class; 0: one
        class) and ordered by local expert within a run, stably."""
        counts = (ctypes.c_int32 * self.world)()
        pairs = (ctypes.c_int32 * self.world)()
        total = ctypes.c_int32(0)
        rc = _lib.lib().wisp_ep_receive(self._h, int(class_min_pairs), self._stream(), counts, pairs,
                                        ctypes.byref(total))
        self.launches += 1
        _lib.check(rc, "wisp_ep_receive")
        return list(counts), list(pairs)

    def received(self, R: int):
        """Views of the compacted received rows: x [R,H], w [R,1], ids [R,1] and
        the output rows y [R,H] the local layer writes."""
        return self.x_recv[:R], self.w_recv[:R], self.ids_recv[:R], self.y_recv[:R]

    def send_back(self) -> None:
        _lib.check(_lib.lib().wisp_ep_return(self._h, self._stream()), "wisp_ep_return")
        self.launches += 1

    def combine(self, out: torch.Tensor, T: int, K: int) -> None:
        _lib.check(_lib.lib().wisp_ep_combine(self._h, int(T), int(K), out.data_ptr(), self._stream()),
                   "wisp_ep_combine")
        self.launches += 1

    def synchronize(self) -> None:
        """Wait for the device; raise if a wait of the group's kernels ran out."""
        _lib.check(_lib.lib().wisp_ep_sync(self._h), "expert-parallel exchange")

    def close(self) -> None:
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            _lib.lib().wisp_ep_group_destroy(h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class EPMoELayer:
    """One MoE layer sharded over the ranks of an expert-parallel group.

    ``cpu_w13_shard [E/P, 2I, H]`` and ``cpu_w2_shard [E/P, H, I]`` are this
    rank's experts (bf16 host masters, pinned here if they are not).
    ``cap_experts`` is this rank's slot count (``WISP_CAP_EXPERTS`` per GPU);
    ``mode`` is ``"paged"`` or ``"resident"``.  ``exchange`` is the group's
    :class:`EPExchange` (shared by the model's layers); without one the layer
    builds its own for calls of up to ``max_pairs`` pairs.  ``local``
    replaces the one-GPU layer that computes the received rows (tests)."""

    def __init__(self, cpu_w13_shard: torch.Tensor | None, cpu_w2_shard: torch.Tensor | None,
                 num_experts: int, cap_experts: int, mode: str = "paged", device=None,
                 layer_idx: int = 0, group=None, rank: int | None = None,
                 world_size: int | None = None, local=None, exchange=None, max_pairs: int = 512) -> None:
        self.group = group
        if exchange is not None:
            self.world, self.rank = exchange.world, exchange.rank
        else:
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
        self._own_exchange = exchange is None
        if exchange is None:
            exchange = EPExchange(self.hidden, max_pairs, self.device, group=group, rank=self.rank,
                                  world=self.world)
        self.exchange = exchange
        # the largest call this owner can receive: every source's pairs, one
        # expert per row; reserved now (a workspace that grows mid-run waits for
        # the device, and the receive size varies from call to call)
        reserve = getattr(local, "reserve", None)
        if reserve is not None and getattr(local, "hidden_size", 0):
            reserve(exchange.world * exchange.max_pairs, 1)
        self.last_counts: list[int] = []
        self.last_runs: list[tuple[int, int]] = []   # (first row, rows) of each local call of the last forward

    # ---- phases (forward runs them in order; tests may run them per rank) ----
    def begin(self, x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor):
        """Route this rank's pairs and store them into their owners."""
        T, K = int(topk_ids.shape[0]), int(topk_ids.shape[-1])
        if x.dtype != torch.bfloat16:
            raise TypeError("wisp_b200 expert parallelism moves bf16 hidden states; got %s" % x.dtype)
        x = x.contiguous()
        w = topk_weights.to(torch.float32).contiguous()
        ids = topk_ids if topk_ids.dtype in (torch.int32, torch.int64) else topk_ids.to(torch.int64)
        ids = ids.contiguous()
        self.exchange.dispatch(x, w, ids, self.experts_per_rank)
        return T, K

    def arrive(self):
        """Wait for every source; returns (rows per source, pairs per source)."""
        threshold = getattr(self.local, "class_threshold", None)
        counts, src_pairs = self.exchange.receive(threshold() if threshold is not None else 0)
        self.last_counts = counts
        return counts, src_pairs

    def compute(self, counts: list[int], src_pairs: list[int]) -> None:
        """This rank's experts on the rows it received (one expert per row),
        each source's rows in the numeric class of a one-GPU call of that
        source's size."""
        R = sum(counts)
        self.last_runs = []
        if not R:
            return
        x, w, ids, y = self.exchange.received(R)
        classify = getattr(self.local, "compute_class", None)
        if classify is None:
            self.last_runs = [(0, R)]
            self.local.forward(x, w, ids, out=y)
            return
        runs = []  # [class, first row, rows]: consecutive sources of one class
        row = 0
        for cnt, pairs in zip(counts, src_pairs):
            cls = classify(int(pairs))
            if cnt and runs and runs[-1][0] == cls:
                runs[-1][2] += cnt
            elif cnt:
                runs.append([cls, row, cnt])
            row += cnt
        self.last_runs = [(r0, n) for _, r0, n in runs]
        try:
            for cls, r0, n in runs:
                self.local.configure(compute_class=cls)
                self.local.forward(x[r0:r0 + n], w[r0:r0 + n], ids[r0:r0 + n], out=y[r0:r0 + n])
        finally:
            self.local.configure(compute_class="auto")

    def finish(self, T: int, K: int, out: torch.Tensor | None = None) -> torch.Tensor:
        """Return the weighted rows to their sources and sum each token's rows."""
        self.exchange.send_back()
        if out is None:
            out = torch.empty((T, self.exchange.hidden), dtype=torch.bfloat16, device=self.device)
        self.exchange.combine(out, T, K)
        return out

    # ---- the forward -------------------------------------------------------------
    def forward(self, x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """x [T,H] bf16, topk_weights [T,k], topk_ids [T,k] global expert ids;
        returns [T,H] bf16.  Collective: every rank of the group calls it."""
        T, K = self.begin(x, topk_weights, topk_ids)
        counts, src_pairs = self.arrive()
        self.compute(counts, src_pairs)
        return self.finish(T, K, out)

    def synchronize(self) -> None:
        self.local.synchronize()
        self.exchange.synchronize()

    def close(self) -> None:
        if hasattr(self.local, "close"):
            self.local.close()
        if self._own_exchange:
            self.exchange.close()


def shard_range(num_experts: int, rank: int, world: int) -> tuple[int, int]:
    """Experts owned by ``rank``: ``[lo, hi)``."""
    per = num_experts // world
    return rank * per, (rank + 1) * per


__all__ = ["EPExchange", "EPMoELayer", "shard_range"]
