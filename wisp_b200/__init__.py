"""wisp_b200: B200-native (sm_100a) paged fused-MoE layer.

The drop-in surface is ``wisp_b200.integrations.vllm`` (``install_wisp_moe``,
``is_installed``, ``WispMoEState``); the native library is
``wisp_b200/lib/libwisp_b200.so`` with the C ABI in ``include/wisp_b200.h``.
"""
__version__ = "0.1.0"
