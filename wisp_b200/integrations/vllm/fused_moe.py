"""B200 paged fused-MoE method patch: the drop-in for WiSP's vLLM plug-in.

Same surface and semantics as the reference module
(src/wisp/integrations/vllm/fused_moe.py):

* ``WISP_MODE`` = ``paged`` (default) | ``resident`` | ``copy`` with the
  legacy aliases ``day2b`` / ``day2a`` / ``day1``; unknown values warn and
  fall back to paged (fused_moe.py:76-92);
* ``WISP_CAP_EXPERTS``: unset -> ``min(E, 24)``, not an int -> ``E``, else
  clamped to ``[2, E]`` (fused_moe.py:95-118); ``install_wisp_moe(cap_experts=)``
  overrides it (fused_moe.py:843-847);
* ``install_wisp_moe(*, mode=None, cap_experts=None) -> bool`` patches
  ``UnquantizedFusedMoEMethod.create_weights``, ``process_weights_after_loading``
  and ``forward_cuda``, keeping the originals as ``_wisp_original_*``; it is
  idempotent through a class flag and a re-call only refreshes the runtime
  config (fused_moe.py:1245-1305); ``is_installed()`` (fused_moe.py:1308-1315);
* ``WispMoEState``: the per-layer paging state, attached as
  ``layer._wisp_state`` (fused_moe.py:126-490).

What changes is underneath: the LRU pager runs on the GPU (bit-exact with the
reference's ``ensure_resident``), page-in runs on a copy-engine stream, and the
expert compute is this package's sm_100a kernels behind the C ABI
(``include/wisp_b200.h``) instead of vLLM's ``fused_experts``.  The patch
targets the installed vLLM's method signatures
(``forward_cuda(layer, x, topk_weights, topk_ids, shared_experts,
shared_experts_input)``): routing arrives already computed.
"""
from __future__ import annotations

import ctypes
import logging
import os
from typing import Any

import torch

from wisp_b200 import _lib

logger = logging.getLogger("wisp_b200.integrations.vllm.fused_moe")

_PATCHED_FLAG = "_wisp_patched"


class _Mode:
    COPY = "copy"
    RESIDENT = "resident"
    PAGED = "paged"


_LEGACY_MODE_ALIASES = {"day1": _Mode.COPY, "day2a": _Mode.RESIDENT, "day2b": _Mode.PAGED}


def _resolve_mode() -> str:
    """``WISP_MODE`` -> mode (fused_moe.py:86-92)."""
    raw = os.environ.get("WISP_MODE", _Mode.PAGED).strip().lower()
    raw = _LEGACY_MODE_ALIASES.get(raw, raw)
    if raw not in (_Mode.COPY, _Mode.RESIDENT, _Mode.PAGED):
        logger.warning("WISP_MODE=%r unrecognised; defaulting to paged", raw)
        return _Mode.PAGED
    return raw


def _resolve_cap_experts(num_experts: int) -> int:
    """``WISP_CAP_EXPERTS`` -> paged-mode cap (fused_moe.py:95-118)."""
    raw = os.environ.get("WISP_CAP_EXPERTS")
    if raw is None:
        return min(num_experts, 24)
    try:
        cap = int(raw)
    except ValueError:
        logger.warning("WISP_CAP_EXPERTS=%r is not an int; using num_experts=%d", raw, num_experts)
        return num_experts
    return max(2, min(cap, num_experts))


class _DeviceBytes:
    """``__cuda_array_interface__`` over library-owned device memory, so torch
    can view the slot scratch and the expert map without copying."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {
            "shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3,
            "strides": None, "stream": None,
        }


def _device_view(ptr: int, nbytes: int, dtype: torch.dtype, shape, device) -> torch.Tensor:
    raw = torch.as_tensor(_DeviceBytes(ptr, nbytes), device=device)
    return raw.view(dtype).view(*shape)


def _pinned(t: torch.Tensor) -> torch.Tensor:
    t = t.contiguous()
    return t if t.is_pinned() else t.pin_memory()


class WispMoEState:
    """Per-layer paging state (fused_moe.py:126-490) backed by a C-ABI layer.

    ``cpu_w13 [E, 2I, H]`` / ``cpu_w2 [E, H, I]`` are the host masters (pinned
    here if they are not).  The bookkeeping fields of the reference
    (``slot_to_expert``, ``expert_to_slot``, ``lru_tick``, ``lru_clock``,
    ``stats_*``) are read back from the device on access.  Forward compute needs
    bf16 masters of those shapes; any other dtype/shape still pages (the
    reference's own unit tests page tiny fp32 experts)."""

    def __init__(self, cpu_w13: torch.Tensor, cpu_w2: torch.Tensor, cap_experts: int, mode: str,
                 device: torch.device, layer_idx: int) -> None:
        self.layer_idx = int(layer_idx)
        self.num_experts = int(cpu_w13.shape[0])
        self.mode = mode
        self.cpu_w13 = _pinned(cpu_w13)
        self.cpu_w2 = _pinned(cpu_w2)
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        E = self.num_experts
        b13 = self.cpu_w13[0].numel() * self.cpu_w13.element_size()
        b2 = self.cpu_w2[0].numel() * self.cpu_w2.element_size()
        hidden = inter = 0
        if (self.cpu_w13.dtype == torch.bfloat16 and self.cpu_w2.dtype == torch.bfloat16
                and self.cpu_w13.dim() == 3 and self.cpu_w2.dim() == 3
                and self.cpu_w13.shape[1] == 2 * self.cpu_w2.shape[2]
                and self.cpu_w13.shape[2] == self.cpu_w2.shape[1]
                and self.cpu_w2.shape[1] % 8 == 0 and self.cpu_w2.shape[2] % 8 == 0):
            hidden, inter = int(self.cpu_w2.shape[1]), int(self.cpu_w2.shape[2])
        self.hidden_size, self.intermediate_size = hidden, inter
        cmode = _lib.MODE_RESIDENT if mode == _Mode.RESIDENT else _lib.MODE_PAGED
        self._h = self._create_native(E, int(cap_experts), hidden, inter, b13, b2, cmode)
        self._b13, self._b2 = b13, b2
        self.tc_min_pairs = self._query(_lib.CFG_TC_MIN_PAIRS)
        self.stats_pred_hits = 0
        self.stats_pred_total = 0
        self._refresh_views()

    def _create_native(self, E, cap, hidden, inter, b13, b2, cmode):
        handle = ctypes.c_void_p()
        _lib.check(_lib.lib().wisp_layer_create(
            E, cap, hidden, inter, b13, b2, self.cpu_w13.data_ptr(), self.cpu_w2.data_ptr(),
            self.device.index, cmode, ctypes.byref(handle)), "wisp_layer_create")
        return handle

    # ---- lifetime ---------------------------------------------------------
    def close(self) -> None:
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            _lib.lib().wisp_layer_destroy(h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- views --------------------------------------------------------------
    def _refresh_views(self) -> None:
        p13, p2, pm = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        _lib.check(_lib.lib().wisp_layer_buffers(self._h, ctypes.byref(p13), ctypes.byref(p2),
                                                 ctypes.byref(pm)))
        cap = self._read(cap_only=True)
        self.cap_experts = cap
        self.scratch_w13 = _device_view(p13.value, cap * self._b13, self.cpu_w13.dtype,
                                        (cap, *self.cpu_w13.shape[1:]), self.device)
        self.scratch_w2 = _device_view(p2.value, cap * self._b2, self.cpu_w2.dtype,
                                       (cap, *self.cpu_w2.shape[1:]), self.device)
        self.expert_map_device = _device_view(pm.value, 4 * self.num_experts, torch.int32,
                                              (self.num_experts,), self.device)

    def _read(self, cap_only: bool = False):
        L = _lib.lib()
        cap = ctypes.c_int32()
        if cap_only:
            _lib.check(L.wisp_get_state(self._h, None, None, None, None, None, ctypes.byref(cap)))
            return cap.value
        c = self.cap_experts
        s2e = (ctypes.c_int32 * c)()
        tick = (ctypes.c_int64 * c)()
        clock = ctypes.c_int64()
        stats = (ctypes.c_int64 * 4)()
        _lib.check(L.wisp_get_state(self._h, s2e, tick, ctypes.byref(clock), stats, None,
                                    ctypes.byref(cap)))
        return list(s2e), list(tick), clock.value, list(stats)

    @property
    def slot_to_expert(self) -> list:
        return self._read()[0]

    @property
    def expert_to_slot(self) -> dict:
        return {e: s for s, e in enumerate(self._read()[0]) if e != -1}

    @property
    def lru_tick(self) -> list:
        return self._read()[1]

    @property
    def lru_clock(self) -> int:
        return self._read()[2]

    def stats(self) -> list:
        """``[forward, miss, hits, evict]``."""
        return self._read()[3]

    @property
    def last_unique_experts(self) -> set:
        """Unique experts of the last paged forward (fused_moe.py:1170-1176);
        a resident forward leaves it unchanged, as the reference's does."""
        buf = (ctypes.c_int32 * self.num_experts)()
        n = ctypes.c_int32(0)
        _lib.check(_lib.lib().wisp_get_last_unique_experts(self._h, buf, self.num_experts, ctypes.byref(n)),
                   "last_unique_experts")
        return set(buf[: n.value])

    def _stat(i):  # noqa: N805
        def get(self):
            return self._read()[3][i]

        def put(self, v):
            s = self._read()[3]
            s[i] = int(v)
            _lib.check(_lib.lib().wisp_set_stats(self._h, (ctypes.c_int64 * 4)(*s)))
        return property(get, put)

    stats_forward = _stat(0)
    stats_miss = _stat(1)
    stats_hits = _stat(2)
    stats_evict = _stat(3)
    del _stat

    # ---- reference methods --------------------------------------------------
    def prime_identity(self) -> None:
        """Resident mode: identity map and full copy (fused_moe.py:242-258)."""
        assert self.cap_experts == self.num_experts, "prime_identity requires cap == num_experts"
        _lib.check(_lib.lib().wisp_prime_identity(self._h, _lib.stream_ptr(
            torch.cuda.current_stream(self.device))), "prime_identity")

    def ensure_resident(self, needed_experts: torch.Tensor) -> None:
        """One LRU admission step with page-in (fused_moe.py:264-358); raises
        ``RuntimeError`` (mentioning sub-batch) when the set exceeds the cap."""
        ids = needed_experts.reshape(-1)
        if ids.device != self.device:
            ids = ids.to(self.device)
        if ids.dtype not in (torch.int32, torch.int64):
            ids = ids.to(torch.int64)
        ids = ids.contiguous()
        _lib.check(_lib.lib().wisp_ensure_resident(
            self._h, ids.data_ptr(), int(ids.dtype == torch.int64), ids.numel(),
            _lib.stream_ptr(torch.cuda.current_stream(self.device))), "ensure_resident")

    def pager_step(self, topk_ids: torch.Tensor):
        """Pager side of one forward (groups + LRU + page-in) without compute;
        returns the slot each (t, k) reads as a CPU int32 tensor."""
        ids = topk_ids
        if ids.dim() == 1:
            ids = ids.reshape(1, -1)
        ids = ids.to(self.device)
        if ids.dtype not in (torch.int32, torch.int64):
            ids = ids.to(torch.int64)
        ids = ids.contiguous()
        T, K = ids.shape
        slots = torch.empty(T, K, dtype=torch.int32)
        _lib.check(_lib.lib().wisp_pager_step(
            self._h, ids.data_ptr(), int(ids.dtype == torch.int64), T, K, slots.data_ptr(),
            _lib.stream_ptr(torch.cuda.current_stream(self.device))), "pager_step")
        return slots

    def reserve(self, num_tokens: int, top_k: int) -> None:
        """Size the per-call workspace for calls of up to ``num_tokens`` x
        ``top_k`` now (``wisp_layer_reserve``), so no later call grows it."""
        _lib.check(_lib.lib().wisp_layer_reserve(self._h, int(num_tokens), int(top_k)), "reserve")

    def prefetch_async(self, predicted_experts) -> None:
        """Speculative page-in of ``predicted_experts`` (fused_moe.py:360-433):
        loads the predicted experts that have no slot, in the order the set
        iterates, evicting by LRU among slots whose expert is neither predicted
        nor in :attr:`last_unique_experts`; a prediction larger than the room
        loads in part.  Runs on the layer's copy stream after its last forward;
        its next forward waits for the copies."""
        ids = [int(e) for e in predicted_experts]
        if not ids:
            return
        arr = (ctypes.c_int32 * len(ids))(*ids)
        _lib.check(_lib.lib().wisp_prefetch_async(self._h, arr, len(ids), None), "prefetch_async")

    def resize_cap(self, new_cap: int) -> None:
        """Hot resize at a drained barrier (fused_moe.py:439-490); refreshes the
        scratch views."""
        _lib.check(_lib.lib().wisp_resize_cap(self._h, int(new_cap), None), "resize_cap")
        self._refresh_views()

    # ---- forward --------------------------------------------------------------
    def forward(self, x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """Paged (or resident) MoE forward: pager + page-in + expert compute +
        routing-order combine.  x [T,H] bf16, topk_weights [T,k], topk_ids
        [T,k] (int32/int64) on this state's device; returns [T,H] bf16."""
        if self.hidden_size == 0:
            raise _lib.WispError(_lib.WISP_ERR_UNSUPPORTED,
                                 "forward needs bf16 w13 [E,2I,H] / w2 [E,H,I] masters")
        T = x.shape[0]
        K = topk_ids.shape[-1]
        x = x.contiguous()
        if x.dtype != torch.bfloat16:
            raise TypeError("wisp_b200 forward computes in bf16; got %s" % x.dtype)
        tw = topk_weights.to(torch.float32).contiguous()
        ids = topk_ids if topk_ids.dtype in (torch.int32, torch.int64) else topk_ids.to(torch.int64)
        ids = ids.contiguous()
        if out is None:
            out = torch.empty_like(x)
        _lib.check(_lib.lib().wisp_moe_forward(
            self._h, x.data_ptr(), tw.data_ptr(), ids.data_ptr(), int(ids.dtype == torch.int64),
            T, K, out.data_ptr(), _lib.stream_ptr(torch.cuda.current_stream(self.device))),
            "wisp_moe_forward")
        return out

    def forward_logits(self, x: torch.Tensor, router_logits: torch.Tensor, top_k: int,
                       renormalize: bool = True, out: torch.Tensor | None = None) -> torch.Tensor:
        """The forward from router logits: softmax top-k routing on the GPU
        (:func:`select_experts`, fused_moe.py:1054-1076), then :meth:`forward`."""
        w, ids = select_experts(router_logits, top_k, renormalize)
        return self.forward(x, w, ids, out=out)

    def synchronize(self) -> None:
        """Wait for this layer's queued forwards (kernels and page-ins) and raise
        the first error any of them hit (forwards return before their work runs)."""
        _lib.check(_lib.lib().wisp_layer_sync(self._h), "forward")

    def telemetry(self) -> dict:
        """Cumulative counters (synchronises): token groups run, misses, page-in
        bytes, unique experts read summed over groups, kernels launched."""
        info = (ctypes.c_int64 * 4)()
        _lib.check(_lib.lib().wisp_get_telemetry(self._h, info))
        n = ctypes.c_int64(0)
        _lib.check(_lib.lib().wisp_get_launch_count(self._h, ctypes.byref(n)))
        return {"groups": info[0], "misses": info[1], "pagein_bytes": info[2],
                "unique_experts": info[3], "kernel_launches": n.value}

    def _query(self, key: int) -> int:
        v = ctypes.c_int64(0)
        _lib.check(_lib.lib().wisp_layer_query(self._h, key, ctypes.byref(v)), "wisp_layer_query")
        return int(v.value)

    def compute_class(self, pairs: int) -> str:
        """``"tc"`` when a call of ``pairs`` (token, k) pairs runs its expert
        compute on the tensor cores, else ``"cuda"`` (the library's rule)."""
        h, i = self.hidden_size, self.intermediate_size
        if not (h > 0 and i > 0 and h % 256 == 0 and i % 128 == 0):
            return "cuda"
        return "tc" if pairs >= min(self.tc_min_pairs, _lib.PREFILL_MIN_PAIRS) else "cuda"

    def class_threshold(self) -> int:
        """Calls of at least this many (token, k) pairs compute on the tensor
        cores (0: every call on the CUDA-core kernels); the rule of
        :meth:`compute_class`."""
        h, i = self.hidden_size, self.intermediate_size
        if not (h > 0 and i > 0 and h % 256 == 0 and i % 128 == 0):
            return 0
        return min(self.tc_min_pairs, _lib.PREFILL_MIN_PAIRS)

    def configure(self, *, asynchronous: bool | None = None, wait_ns: int | None = None,
                  drop_pageins: int | None = None, tc_min_pairs: int | None = None,
                  compute_class: str | None = None) -> None:
        """Runtime knobs of the native layer (see ``wisp_layer_config``).

        ``asynchronous``: the single-launch forward (default for resident
        layers).  A paged layer defaults to the host-synchronous forward: a
        paged single-launch forward waits inside its kernel for page-in copies
        a host thread issues after the launch, so it suits only callers that
        queue no other device work while it pages in.  ``tc_min_pairs``: calls
        of at least this many (token, k) pairs compute on the tensor cores.
        ``compute_class``: ``"auto"`` (by call size), ``"cuda"`` or ``"tc"``
        for every call until changed."""
        L = _lib.lib()
        cls = None if compute_class is None else {"auto": 0, "cuda": 1, "tc": 2}[compute_class]
        for key, val in ((_lib.CFG_ASYNC, asynchronous), (_lib.CFG_WAIT_NS, wait_ns),
                         (_lib.CFG_DROP_PAGEINS, drop_pageins), (_lib.CFG_TC_MIN_PAIRS, tc_min_pairs),
                         (_lib.CFG_COMPUTE_CLASS, cls)):
            if val is not None:
                _lib.check(L.wisp_layer_config(self._h, key, int(val)), "configure")
        if tc_min_pairs is not None:
            self.tc_min_pairs = self._query(_lib.CFG_TC_MIN_PAIRS)


def select_experts(router_logits: torch.Tensor, top_k: int, renormalize: bool = True):
    """Softmax top-k routing on the GPU (``wisp_route_topk``): fp32 softmax
    over the experts, the ``top_k`` largest probabilities in descending order
    (ties to the lower id), renormalised to sum to one when ``renormalize`` --
    the Qwen3 / Mixtral routing of the reference's paged forward
    (fused_moe.py:1054-1076).  router_logits [T, E] fp32 or bf16 on a CUDA
    device; returns (topk_weights [T, k] fp32, topk_ids [T, k] int32)."""
    logits = router_logits.contiguous()
    if logits.dtype not in (torch.float32, torch.bfloat16):
        logits = logits.float()
    T, E = logits.shape
    w = torch.empty((T, top_k), dtype=torch.float32, device=logits.device)
    ids = torch.empty((T, top_k), dtype=torch.int32, device=logits.device)
    _lib.check(_lib.lib().wisp_route_topk(
        logits.data_ptr(), int(logits.dtype == torch.bfloat16), T, E, int(top_k), int(bool(renormalize)),
        w.data_ptr(), ids.data_ptr(), _lib.stream_ptr(torch.cuda.current_stream(logits.device))),
        "wisp_route_topk")
    return w, ids


# ---------------------------------------------------------------------------
# Runtime config and layer registry (fused_moe.py:497-526, 537-593)
# ---------------------------------------------------------------------------

_WISP_RUNTIME_CONFIG: dict[str, Any] = {"mode": _Mode.RESIDENT, "cap_experts_override": None}
_LAYER_STATES: list[WispMoEState] = []
_LAYER_BY_ID: dict[int, WispMoEState] = {}

# Cross-layer prefetch (off unless WISP_PREFETCH is set, as in the reference):
# the co-occurrence table (None: not loaded yet; False: disabled after a load
# failure) and the current decode step's observations, layer -> unique experts.
_COOCCUR_TABLE: Any = None
_CURRENT_STEP_OBS: dict[int, set] = {}


def _env_on(name: str) -> bool:
    return os.environ.get(name, "0").strip().lower() in ("1", "true", "yes")


def _maybe_load_cooccur():
    """The co-occurrence table: ``WISP_COOCCUR_PATH`` (a warm table in the
    reference's JSON schema) or a cold table when ``WISP_COOCCUR_ONLINE`` is
    set; ``None`` when neither is configured (fused_moe.py:596-631).  The
    table lives in the library's host C++ (``NativeCooccurTable``: the same
    counts and rankings as the reference's, at native speed)."""
    global _COOCCUR_TABLE
    if _COOCCUR_TABLE is not None:
        return _COOCCUR_TABLE or None
    path = os.environ.get("WISP_COOCCUR_PATH", "").strip()
    if not path and not _env_on("WISP_COOCCUR_ONLINE"):
        return None
    from .cooccur import NativeCooccurTable
    try:
        _COOCCUR_TABLE = (NativeCooccurTable.load(path) if path and os.path.isfile(path)
                          else NativeCooccurTable())
    except Exception as e:
        logger.warning("wisp.vllm: cooccur table could not be loaded (%s); prefetch disabled", e)
        _COOCCUR_TABLE = False
        return None
    return _COOCCUR_TABLE


def _cooccur_predict_top_k(target_layer: int, k: int) -> list:
    """Experts to prefetch into ``target_layer`` from this step's observations
    at earlier layers (fused_moe.py:634-652: normalised, decay 0.5)."""
    table = _COOCCUR_TABLE
    if not table or not _CURRENT_STEP_OBS:
        return []
    from .cooccur import predict_layer
    return predict_layer(table, _CURRENT_STEP_OBS, target_layer, k=k, normalize=True, decay=0.5,
                         only_prev_layer=False)


def _post_forward(state: WispMoEState, last_set: set) -> None:
    """After a paged forward: record its unique experts for this step, predict
    ``max(8, cap // 2)`` experts for the next layer and prefetch them; after
    the last layer, learn the step online (fused_moe.py:1170-1233)."""
    table = _maybe_load_cooccur() if _env_on("WISP_PREFETCH") else None
    if table is None or not last_set:
        return
    _CURRENT_STEP_OBS[state.layer_idx] = last_set
    nxt = state.layer_idx + 1
    if nxt < len(_LAYER_STATES):
        ns = _LAYER_STATES[nxt]
        predicted = _cooccur_predict_top_k(nxt, max(8, ns.cap_experts // 2))
        if predicted and ns.mode == _Mode.PAGED:
            try:
                ns.prefetch_async(set(predicted))
                ns.stats_pred_total += len(predicted)
            except Exception as e:
                logger.debug("wisp.vllm: prefetch_async failed: %s", e)
    if state.layer_idx == len(_LAYER_STATES) - 1:
        if _env_on("WISP_COOCCUR_ONLINE"):
            try:
                table.observe_step(_CURRENT_STEP_OBS)
            except Exception:
                pass
        _CURRENT_STEP_OBS.clear()


def resize_layer_caps(new_cap: int) -> int:
    n = 0
    for st in _LAYER_STATES:
        st.resize_cap(new_cap)
        n += 1
    return n


def current_layer_cap() -> int | None:
    return _LAYER_STATES[0].cap_experts if _LAYER_STATES else None


def num_registered_layers() -> int:
    return len(_LAYER_STATES)


def num_experts_per_layer() -> int | None:
    return _LAYER_STATES[0].num_experts if _LAYER_STATES else None


def expert_bytes_per_cap() -> int:
    return sum(st._b13 + st._b2 for st in _LAYER_STATES)


def snapshot_expert_stats(reset: bool = True) -> dict:
    """Counters summed over layers; ``ws`` = the largest unique-expert set of
    any layer's last paged forward (fused_moe.py:579-593)."""
    miss = hit = fwd = 0
    for s in _LAYER_STATES:
        f, m, h, _e = s.stats()
        miss, hit, fwd = miss + m, hit + h, fwd + f
    ws = max((len(s.last_unique_experts) for s in _LAYER_STATES), default=0)
    if reset:
        for s in _LAYER_STATES:
            s.stats_miss = 0
            s.stats_hits = 0
            s.stats_forward = 0
    return {"miss": miss, "hit": hit, "forward": fwd, "ws": ws}


# ---------------------------------------------------------------------------
# Patched methods
# ---------------------------------------------------------------------------


def _patched_create_weights(self, layer: torch.nn.Module, num_experts: int, hidden_size: int,
                            intermediate_size_per_partition: int, params_dtype: torch.dtype,
                            **extra_weight_attrs) -> None:
    """Allocate the MoE master weights on CPU (fused_moe.py:673-759) so loading
    never puts the full expert set in HBM; they are pinned after loading."""
    from vllm.model_executor.utils import set_weight_attrs

    if self.moe.has_bias:
        raise NotImplementedError("wisp.vllm: has_bias=True MoE checkpoints are not supported")
    up = 2 * intermediate_size_per_partition if self.moe.is_act_and_mul else intermediate_size_per_partition
    w13 = torch.nn.Parameter(torch.empty(num_experts, up, hidden_size, dtype=params_dtype,
                                         device="cpu"), requires_grad=False)
    layer.register_parameter("w13_weight", w13)
    set_weight_attrs(w13, extra_weight_attrs)
    layer._wisp_cpu_pin_w13 = w13.data
    w2 = torch.nn.Parameter(torch.empty(num_experts, hidden_size, intermediate_size_per_partition,
                                        dtype=params_dtype, device="cpu"), requires_grad=False)
    layer.register_parameter("w2_weight", w2)
    set_weight_attrs(w2, extra_weight_attrs)
    layer._wisp_cpu_pin_w2 = w2.data


def _patched_process_weights_after_loading(self, layer: torch.nn.Module) -> None:
    """Pin the masters and build the layer's ``WispMoEState``
    (fused_moe.py:762-927); the Parameters become 0-element placeholders."""
    if getattr(layer, "_wisp_state", None) is not None or getattr(layer, "_wisp_cpu_w13", None) is not None:
        return
    try:
        type(self)._wisp_original_process_weights_after_loading(self, layer)
    except Exception as e:  # kernel set-up of the replaced backend is not needed
        logger.debug("wisp.vllm: original process_weights_after_loading skipped (%s)", e)
    w13 = getattr(layer, "w13_weight", None)
    w2 = getattr(layer, "w2_weight", None)
    if w13 is None or w2 is None:
        return
    gpu = torch.device("cuda", torch.cuda.current_device())
    pin13 = getattr(layer, "_wisp_cpu_pin_w13", None)
    pin2 = getattr(layer, "_wisp_cpu_pin_w2", None)
    if pin13 is not None and pin2 is not None:
        cpu_w13, cpu_w2 = _pinned(pin13), _pinned(pin2)
    elif w13.device.type == "cuda" and w2.device.type == "cuda":
        cpu_w13, cpu_w2 = _pinned(w13.data.cpu()), _pinned(w2.data.cpu())
    elif w13.device.type == "cpu" and w2.device.type == "cpu":
        cpu_w13, cpu_w2 = _pinned(w13.data), _pinned(w2.data)
    else:
        return
    layer._wisp_cpu_pin_w13, layer._wisp_cpu_pin_w2 = cpu_w13, cpu_w2
    mode = _WISP_RUNTIME_CONFIG["mode"]
    if mode == _Mode.COPY:
        layer._wisp_cpu_w13, layer._wisp_cpu_w2 = cpu_w13, cpu_w2
        layer._wisp_state = None
        return
    E = int(cpu_w13.shape[0])
    override = _WISP_RUNTIME_CONFIG["cap_experts_override"]
    if mode == _Mode.RESIDENT:
        cap = E
    else:
        cap = override if override is not None else _resolve_cap_experts(E)
    state = WispMoEState(cpu_w13, cpu_w2, cap, mode, gpu, len(_LAYER_STATES))
    _LAYER_STATES.append(state)
    _LAYER_BY_ID[id(layer)] = state
    if mode == _Mode.RESIDENT:
        state.prime_identity()
    layer._wisp_state = state
    layer.w13_weight.data = torch.empty(0, dtype=cpu_w13.dtype, device=gpu)
    layer.w2_weight.data = torch.empty(0, dtype=cpu_w2.dtype, device=gpu)
    # hand the loader's cached device blocks back so the engine's memory
    # accounting sees only the slot scratch (fused_moe.py:906-916)
    torch.cuda.empty_cache()
    logger.info("wisp.vllm[%s]: layer init: num_experts=%d cap_experts=%d", mode, E, state.cap_experts)


def _apply_shared(shared_experts, shared_experts_input) -> None:
    if shared_experts is not None:
        from vllm.model_executor.layers.fused_moe.runner.shared_experts import SharedExpertsOrder
        shared_experts.apply(shared_experts_input, SharedExpertsOrder.MK_INTERNAL_OVERLAPPED)


def _patched_forward_cuda(self, layer: torch.nn.Module, x: torch.Tensor, topk_weights: torch.Tensor,
                          topk_ids: torch.Tensor, shared_experts=None, shared_experts_input=None):
    """Paged / resident / copy dispatch (fused_moe.py:930-987) on the installed
    vLLM's signature: routing is already computed by the runner."""
    state: WispMoEState | None = getattr(layer, "_wisp_state", None)
    if state is None and getattr(layer, "_wisp_cpu_w13", None) is not None:
        # copy mode: stage the full expert set for this forward only
        tmp = WispMoEState(layer._wisp_cpu_w13, layer._wisp_cpu_w2, layer._wisp_cpu_w13.shape[0],
                           _Mode.RESIDENT, x.device, -1)
        try:
            tmp.prime_identity()
            out = tmp.forward(x, topk_weights, topk_ids)
            torch.cuda.current_stream(x.device).synchronize()
        finally:
            tmp.close()
        _apply_shared(shared_experts, shared_experts_input)
        return out
    if state is None:
        return type(self)._wisp_original_forward_cuda(self, layer, x, topk_weights, topk_ids,
                                                      shared_experts, shared_experts_input)
    out = state.forward(x, topk_weights, topk_ids)
    if state.mode == _Mode.PAGED and _env_on("WISP_PREFETCH"):
        _post_forward(state, state.last_unique_experts)
    _apply_shared(shared_experts, shared_experts_input)
    return out


# ---------------------------------------------------------------------------
# Install
# ---------------------------------------------------------------------------


def _method_class():
    try:
        from vllm.model_executor.layers.fused_moe.unquantized_fused_moe_method import (
            UnquantizedFusedMoEMethod,
        )
    except ImportError as e:
        raise ImportError("wisp_b200.integrations.vllm requires vllm to be installed.") from e
    return UnquantizedFusedMoEMethod


def install_wisp_moe(*, mode: str | None = None, cap_experts: int | None = None, _cls=None) -> bool:
    """Idempotent install (fused_moe.py:1245-1305).  Returns True iff this call
    applied the patch; a re-call only refreshes the runtime config."""
    cls = _cls if _cls is not None else _method_class()
    _WISP_RUNTIME_CONFIG["mode"] = mode if mode is not None else _resolve_mode()
    _WISP_RUNTIME_CONFIG["cap_experts_override"] = cap_experts
    if getattr(cls, _PATCHED_FLAG, False):
        return False
    cls._wisp_original_create_weights = cls.create_weights
    cls._wisp_original_process_weights_after_loading = cls.process_weights_after_loading
    cls._wisp_original_forward_cuda = cls.forward_cuda
    cls.create_weights = _patched_create_weights
    cls.process_weights_after_loading = _patched_process_weights_after_loading
    cls.forward_cuda = _patched_forward_cuda
    setattr(cls, _PATCHED_FLAG, True)
    logger.info("wisp.vllm: patched %s (mode=%s cap_experts=%s)", cls.__name__,
                _WISP_RUNTIME_CONFIG["mode"], cap_experts)
    if _cls is None:
        # the block-quantised FP8 MoE path too, best effort (fused_moe.py:1297-1303)
        try:
            from .fused_moe_fp8 import install_wisp_fp8
            install_wisp_fp8()
        except Exception as e:
            logger.warning("wisp.vllm: FP8 MoE patch not applied (%s)", e)
    return True


def is_installed(_cls=None) -> bool:
    try:
        cls = _cls if _cls is not None else _method_class()
    except ImportError:
        return False
    return bool(getattr(cls, _PATCHED_FLAG, False))


__all__ = ["install_wisp_moe", "is_installed", "WispMoEState", "select_experts"]
