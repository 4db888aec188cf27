"""B200-native quantized MoE / decode-GEMM path for SGLang (sglang-restomod's hot path).

The package mirrors the reference plugin's surface for this path
(``sglang_restomod/__init__.py:24-53``, ``plugins.py``): importing it is
cheap; :func:`register` installs the selected components. The kernels live in
``libb200moe.so`` (C ABI in ``include/b200moe.h``), loaded on first use.
"""

from __future__ import annotations

__version__ = "0.1.0"


def register() -> None:
    """SGLang plugin entry point: install the components selected by
    ``SGLANG_RESTOMOD_COMPONENTS`` (see :mod:`.plugins`)."""
    from . import plugins

    plugins.load_enabled()
