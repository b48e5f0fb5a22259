"""vLLM shim: ``install_wisp_moe()`` / ``is_installed()``.

Same entry points as the reference's ``wisp.integrations.vllm``
(src/wisp/integrations/vllm/__init__.py:37-39)::

    from wisp_b200.integrations.vllm import install_wisp_moe
    install_wisp_moe()          # before vLLM builds the model

``WISP_MODE`` / ``WISP_CAP_EXPERTS`` keep their meaning; the paging, page-in
and expert compute run in this package's sm_100a kernels.
"""
from .fused_moe import WispMoEState, install_wisp_moe, is_installed
from .fused_moe_fp8 import WispMoEStateFP8, install_wisp_fp8, is_fp8_installed

__all__ = ["install_wisp_moe", "is_installed", "WispMoEState", "install_wisp_fp8", "is_fp8_installed",
           "WispMoEStateFP8"]
