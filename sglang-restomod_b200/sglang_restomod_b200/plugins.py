"""Which of this package's hooks get installed into SGLang.

A launch profile names components in ``SGLANG_RESTOMOD_COMPONENTS``
(comma-separated). The variable and the component names are the reference
plugin's (``sglang_restomod/plugins.py``), restricted to the quantized MoE
and decode-GEMM path built here, so a profile written for the reference
selects the B200 kernels unchanged; the reference's other components are
refused by name with a pointer to why.

Activation runs one component at a time through three steps - import its
module, find its ``register()``, call it - and the first step that does not
succeed decides the component's state in :mod:`.attest`. One component's
failure never stops the next (SGLang itself swallows plugin exceptions, so a
raise here would silently drop every component after it).
"""

from __future__ import annotations

import importlib
import logging
import os
from dataclasses import dataclass
from typing import Callable, Mapping, Sequence

from . import attest

logger = logging.getLogger(__name__)

ENV_COMPONENTS = "SGLANG_RESTOMOD_COMPONENTS"

_PKG = __name__.rsplit(".", 1)[0]


@dataclass(frozen=True)
class Component:
    name: str
    module: str
    description: str


COMPONENTS: dict[str, Component] = {
    c.name: c
    for c in (
        Component("fp8_moe", f"{_PKG}.quant.fp8_moe",
                  "block-FP8 fused MoE: Fp8MoEMethod -> B200 expert GEMMs"),
        Component("fp8_dense", f"{_PKG}.quant.fp8_dense",
                  "block-FP8 dense linear / decode GEMV: Fp8LinearMethod.apply"),
        Component("fp8_lm_head", f"{_PKG}.quant.fp8_lm_head",
                  "quantize the LM head to block FP8 after load (needs fp8_dense)"),
        Component("fp8_dense_quant", f"{_PKG}.quant.fp8_dense_quant",
                  "quantize admitted bf16 dense linears to block FP8 after load"),
        Component("moe_align_sm70", f"{_PKG}.moe.align",
                  "moe_align_block_size on the B200 kernel"),
        Component("fp4_moe", f"{_PKG}.quant.fp4_moe",
                  "NVFP4 fused MoE: prepare_moe_nvfp4 + moe_wna16_marlin_gemm + moe_sum_reduce"),
        Component("fp4_dense", f"{_PKG}.quant.fp4_dense",
                  "NVFP4 dense linear (W4A16)"),
    )
}

# Reference components that are not on this path (refused with that reason).
NOT_ON_THIS_PATH = frozenset({"attention_v100", "lsa_sm70", "sm70_marlin_v100", "ple_sm70",
                              "spec_sm70", "gdn_tilelang_sm70"})


class UnknownComponent(ValueError):
    """A selected name this package does not provide."""


def parse_selection(text: str) -> list[str]:
    """Names in ``text`` in first-seen order, blanks and repeats dropped."""
    return list(dict.fromkeys(part.strip() for part in text.split(",") if part.strip()))


def selection(env: Mapping[str, str] | None = None) -> list[str]:
    """The selected component names; unknown ones raise :class:`UnknownComponent`."""
    names = parse_selection((os.environ if env is None else env).get(ENV_COMPONENTS, ""))
    unknown = [n for n in names if n not in COMPONENTS]
    if not unknown:
        return names
    elsewhere = sorted(set(unknown) & NOT_ON_THIS_PATH)
    why = (f"; {', '.join(elsewhere)} is not part of the B200 MoE/GEMV path" if elsewhere else "")
    raise UnknownComponent(
        f"unknown component(s) in {ENV_COMPONENTS}: {', '.join(unknown)}{why} "
        f"(this package provides: {', '.join(sorted(COMPONENTS))})")


def is_enabled(name: str, env: Mapping[str, str] | None = None) -> bool:
    return name in selection(env)


def _describe(exc: BaseException) -> str:
    return f"{type(exc).__name__}: {exc}"


def activate(component: Component) -> bool:
    """Import and register one component; its outcome goes to the ledger.
    True when it registered (it may still have reported itself inactive)."""
    try:
        module = importlib.import_module(component.module)
    except Exception as exc:  # noqa: BLE001 - the next component still loads
        attest.record(component.name, False, "import failed: " + _describe(exc))
        logger.warning("component %s: import failed", component.name, exc_info=True)
        return False
    register: Callable[[], object] | None = getattr(module, "register", None)
    if not callable(register):
        attest.record(component.name, False, f"{component.module} defines no register()")
        return False
    try:
        register()
    except Exception as exc:  # noqa: BLE001
        attest.record(component.name, False, _describe(exc))
        logger.warning("component %s: register() raised", component.name, exc_info=True)
        return False
    attest.record(component.name, True)
    return True


def load_enabled(env: Mapping[str, str] | None = None) -> Sequence[str]:
    """Activate every selected component in order; return the ones that
    registered. The ledger is written to ``$SGLANG_RESTOMOD_ATTEST`` at the end."""
    names = selection(env)
    attest.set_selected(names)
    registered = [n for n in names if activate(COMPONENTS[n])]
    from . import census

    census.install_profile()  # only when SGLANG_B200_PROFILE asks for it
    attest.write()
    logger.info("sglang-restomod-b200: %d of %d selected components registered (%s)",
                len(registered), len(names), ", ".join(registered) or "none")
    return registered
