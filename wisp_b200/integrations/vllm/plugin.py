"""``vllm.general_plugins`` entry point (src/wisp/integrations/vllm/plugin.py:47-124).

Register in a package's metadata as::

    [project.entry-points."vllm.general_plugins"]
    wisp_b200 = "wisp_b200.integrations.vllm.plugin:register"

vLLM calls it in every process it starts; it is idempotent.
``WISP_PLUGIN_DISABLE=1`` leaves the plug-in inert.  The live expert/KV
controller arm of the reference (``WISP_DYNAMIC``) is not part of this build:
with ``WISP_DYNAMIC=1`` a warning says so and paging runs with a static split.
"""
from __future__ import annotations

import logging
import os

logger = logging.getLogger(__name__)

_TRUE = ("1", "true", "yes", "on")


def register() -> None:
    if os.environ.get("WISP_PLUGIN_DISABLE", "0").strip().lower() in _TRUE:
        logger.info("wisp_b200.plugin: WISP_PLUGIN_DISABLE=1 - skipping patch")
        return
    try:
        from .fused_moe import install_wisp_moe, is_installed
    except ImportError as e:
        logger.warning("wisp_b200.plugin: import failed (%s); plug-in not installed", e)
        return
    if is_installed():
        return
    install_wisp_moe()
    logger.info("wisp_b200.plugin: patched vLLM (WISP_MODE=%s WISP_CAP_EXPERTS=%s)",
                os.environ.get("WISP_MODE", "paged"), os.environ.get("WISP_CAP_EXPERTS", "auto"))
    if os.environ.get("WISP_DYNAMIC", "0").strip().lower() in _TRUE:
        logger.error("wisp_b200.plugin: WISP_DYNAMIC=1 but the live expert/KV controller is not "
                     "part of this build; running with a static split")
