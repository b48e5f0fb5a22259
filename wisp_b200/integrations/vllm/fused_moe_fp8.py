"""Block-quantised FP8 MoE paging: the drop-in for the reference's FP8 patch.

Same surface and semantics as src/wisp/integrations/vllm/fused_moe_fp8.py:

* ``install_wisp_fp8() -> bool`` patches vLLM's ``Fp8MoEMethod``
  (``create_weights``, ``process_weights_after_loading``, ``apply``) for the
  block-quantised branch only (other FP8 layers keep vLLM's path), idempotent
  through a class flag, originals kept as ``_wisp_original_*``
  (fused_moe_fp8.py:362-390); ``is_fp8_installed()``; ``install_wisp_moe``
  applies it too, best effort.
* ``WispMoEStateFP8`` pages (weight, scale) pairs: float8_e4m3fn ``w13 [E,
  2I, H]`` / ``w2 [E, H, I]`` with their per-128x128-block fp32 scales
  (fused_moe_fp8.py:61-145), with the same LRU pager as the bf16 layer.
* ``WISP_CAP_EXPERTS``: unset or not an int -> ``min(E, 24)``, else clamped
  to ``[8, E]`` (fused_moe_fp8.py:48-58).

Underneath, the pager runs on the GPU, page-in moves the four tensors of an
expert on the layer's copy stream, and the W8A8 block-scaled compute (the
arithmetic of vLLM's block-FP8 fused_experts) runs in this package's kernels.
The weight masters are pinned in place (registered, not copied), so a
200 GB master set is never held twice -- the reference keeps them pageable
for that reason (fused_moe_fp8.py:221-228).  Targets the installed vLLM's
``apply(layer, x, topk_weights, topk_ids, shared_experts,
shared_experts_input)``: routing arrives already computed.
"""
from __future__ import annotations

import ctypes
import logging
import os

import torch

from wisp_b200 import _lib

from .fused_moe import WispMoEState, _apply_shared, _device_view, _Mode

logger = logging.getLogger("wisp_b200.integrations.vllm.fused_moe_fp8")

_PATCHED_FLAG = "_wisp_fp8_patched"
_FP8_LAYER_STATES: list["WispMoEStateFP8"] = []
BLOCK = 128


def _resolve_cap_experts(num_experts: int) -> int:
    """``WISP_CAP_EXPERTS`` for FP8 layers (fused_moe_fp8.py:48-58)."""
    raw = os.environ.get("WISP_CAP_EXPERTS")
    if raw is None:
        return min(num_experts, 24)
    try:
        cap = int(raw)
    except ValueError:
        return min(num_experts, 24)
    return max(8, min(cap, num_experts))


def _pin_in_place(t: torch.Tensor, keep: list) -> torch.Tensor:
    """Page-lock a contiguous CPU tensor where it lies (cudaHostRegister), so
    no second copy of a large master set is made; ``keep`` collects what to
    unregister at close."""
    t = t.contiguous()
    if t.is_pinned():
        return t
    rc = torch.cuda.cudart().cudaHostRegister(t.data_ptr(), t.numel() * t.element_size(), 0)
    if int(rc) != 0:
        return t.pin_memory()          # registration refused: fall back to a pinned copy
    keep.append(t)
    return t


class WispMoEStateFP8(WispMoEState):
    """Per-layer FP8 paging state (fused_moe_fp8.py:61-145) backed by a C-ABI
    layer; the pager, counters and methods are those of :class:`WispMoEState`.
    Extra views: ``scratch_s13`` / ``scratch_s2`` (the slots' block scales)."""

    def __init__(self, cpu_w13, cpu_w2, cpu_s13, cpu_s2, cap_experts: int, device, layer_idx: int,
                 mode: str = _Mode.PAGED) -> None:
        if cpu_w13.dtype != torch.float8_e4m3fn or cpu_w2.dtype != torch.float8_e4m3fn:
            raise TypeError("WispMoEStateFP8 pages float8_e4m3fn experts")
        self._registered: list = []
        w13 = _pin_in_place(cpu_w13, self._registered)
        w2 = _pin_in_place(cpu_w2, self._registered)
        self.cpu_s13 = cpu_s13.to(torch.float32).contiguous().pin_memory()
        self.cpu_s2 = cpu_s2.to(torch.float32).contiguous().pin_memory()
        super().__init__(w13, w2, cap_experts, mode, device, layer_idx)

    def _create_native(self, E, cap, hidden, inter, b13, b2, cmode):
        hidden, inter = int(self.cpu_w2.shape[1]), int(self.cpu_w2.shape[2])
        self.hidden_size, self.intermediate_size = hidden, inter
        handle = ctypes.c_void_p()
        _lib.check(_lib.lib().wisp_layer_create_fp8(
            E, cap, hidden, inter, BLOCK, BLOCK, self.cpu_w13.data_ptr(), self.cpu_w2.data_ptr(),
            self.cpu_s13.data_ptr(), self.cpu_s2.data_ptr(), self.device.index, cmode, ctypes.byref(handle)),
            "wisp_layer_create_fp8")
        return handle

    def _refresh_views(self) -> None:
        super()._refresh_views()
        p13, p2 = ctypes.c_void_p(), ctypes.c_void_p()
        _lib.check(_lib.lib().wisp_layer_scale_buffers(self._h, ctypes.byref(p13), ctypes.byref(p2)))
        cap = self.cap_experts
        s13, s2 = self.cpu_s13, self.cpu_s2
        self.scratch_s13 = _device_view(p13.value, cap * s13[0].numel() * 4, torch.float32,
                                        (cap, *s13.shape[1:]), self.device)
        self.scratch_s2 = _device_view(p2.value, cap * s2[0].numel() * 4, torch.float32,
                                       (cap, *s2.shape[1:]), self.device)

    def class_threshold(self) -> int:
        return 0                        # one compute class (the CUDA-core W8A8 kernels)

    def close(self) -> None:
        super().close()
        for t in getattr(self, "_registered", []):
            torch.cuda.cudart().cudaHostUnregister(t.data_ptr())
        self._registered = []


# ---------------------------------------------------------------------------
# Patched Fp8MoEMethod methods
# ---------------------------------------------------------------------------


def _patched_create_weights(self, layer, num_experts, hidden_size, intermediate_size_per_partition,
                            params_dtype, **extra_weight_attrs):
    """Block-quant FP8 masters on CPU (fused_moe_fp8.py:148-213): weights in
    float8_e4m3fn, per-block fp32 scales; other FP8 layers keep vLLM's."""
    if not getattr(self, "block_quant", False):
        return type(self)._wisp_original_create_weights(self, layer, num_experts, hidden_size,
                                                        intermediate_size_per_partition, params_dtype,
                                                        **extra_weight_attrs)
    from vllm.model_executor.utils import set_weight_attrs

    bn, bk = self.weight_block_size[0], self.weight_block_size[1]
    if intermediate_size_per_partition % bn:
        raise ValueError(f"intermediate size {intermediate_size_per_partition} is not divisible by block_n {bn}")
    layer.num_experts = num_experts
    layer.orig_dtype = params_dtype
    layer.weight_block_size = self.weight_block_size
    I, H = intermediate_size_per_partition, hidden_size
    f8 = torch.float8_e4m3fn
    params = {
        "w13_weight": torch.empty(num_experts, 2 * I, H, dtype=f8),
        "w2_weight": torch.empty(num_experts, H, I, dtype=f8),
        "w13_weight_scale_inv": torch.ones(num_experts, 2 * ((I + bn - 1) // bn), (H + bk - 1) // bk),
        "w2_weight_scale_inv": torch.ones(num_experts, (H + bn - 1) // bn, (I + bk - 1) // bk),
    }
    for name, t in params.items():
        p = torch.nn.Parameter(t, requires_grad=False)
        layer.register_parameter(name, p)
        set_weight_attrs(p, extra_weight_attrs)
    try:
        from vllm.model_executor.layers.fused_moe.layer import FusedMoeWeightScaleSupported
        for name in ("w13_weight_scale_inv", "w2_weight_scale_inv"):
            set_weight_attrs(getattr(layer, name), {"quant_method": FusedMoeWeightScaleSupported.BLOCK.value})
    except ImportError:
        pass
    layer.w13_input_scale = None
    layer.w2_input_scale = None


def _patched_process_weights_after_loading(self, layer) -> None:
    """Build the layer's ``WispMoEStateFP8`` from the CPU masters
    (fused_moe_fp8.py:216-269); the Parameters become 0-element placeholders."""
    if getattr(layer, "_wisp_fp8_state", None) is not None:
        return
    if not getattr(self, "block_quant", False):
        return type(self)._wisp_original_process_weights_after_loading(self, layer)
    cpu = [getattr(layer, n).data for n in ("w13_weight", "w2_weight", "w13_weight_scale_inv",
                                            "w2_weight_scale_inv")]
    cpu = [t.cpu() if t.device.type != "cpu" else t for t in cpu]
    gpu = torch.device("cuda", torch.cuda.current_device())
    E = int(cpu[0].shape[0])
    st = WispMoEStateFP8(cpu[0], cpu[1], cpu[2], cpu[3], _resolve_cap_experts(E), gpu, len(_FP8_LAYER_STATES))
    _FP8_LAYER_STATES.append(st)
    layer._wisp_fp8_state = st
    for n, t in zip(("w13_weight", "w2_weight", "w13_weight_scale_inv", "w2_weight_scale_inv"), cpu):
        getattr(layer, n).data = torch.empty(0, dtype=t.dtype, device=gpu)
    torch.cuda.empty_cache()
    logger.info("wisp.fp8: layer %d init num_experts=%d cap=%d", st.layer_idx, E, st.cap_experts)


def _patched_apply(self, layer, x, topk_weights, topk_ids, shared_experts=None, shared_experts_input=None):
    """The paged FP8 forward (fused_moe_fp8.py:272-359) on the installed
    vLLM's signature."""
    st = getattr(layer, "_wisp_fp8_state", None)
    if st is None:
        return type(self)._wisp_original_apply(self, layer, x, topk_weights, topk_ids, shared_experts,
                                               shared_experts_input)
    out = st.forward(x, topk_weights, topk_ids)
    _apply_shared(shared_experts, shared_experts_input)
    return out


def _method_class():
    from vllm.model_executor.layers.quantization.fp8 import Fp8MoEMethod
    return Fp8MoEMethod


def install_wisp_fp8(_cls=None) -> bool:
    """Patch Fp8MoEMethod's block-quant path; idempotent.  True iff this call
    applied the patch (fused_moe_fp8.py:362-379)."""
    try:
        cls = _cls if _cls is not None else _method_class()
    except ImportError as e:
        logger.warning("wisp.fp8: cannot import Fp8MoEMethod (%s); FP8 paging disabled", e)
        return False
    if getattr(cls, _PATCHED_FLAG, False):
        return False
    cls._wisp_original_create_weights = cls.create_weights
    cls._wisp_original_process_weights_after_loading = cls.process_weights_after_loading
    cls._wisp_original_apply = cls.apply
    cls.create_weights = _patched_create_weights
    cls.process_weights_after_loading = _patched_process_weights_after_loading
    cls.apply = _patched_apply
    setattr(cls, _PATCHED_FLAG, True)
    logger.info("wisp.fp8: patched %s (block-quant working-set paging)", cls.__name__)
    return True


def is_fp8_installed(_cls=None) -> bool:
    try:
        cls = _cls if _cls is not None else _method_class()
    except ImportError:
        return False
    return bool(getattr(cls, _PATCHED_FLAG, False))


__all__ = ["install_wisp_fp8", "is_fp8_installed", "WispMoEStateFP8"]
