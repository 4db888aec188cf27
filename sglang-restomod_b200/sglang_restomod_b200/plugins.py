"""Component registry: which hooks this package installs into SGLang.

The selection variable and the component names are the reference's
(``sglang_restomod/plugins.py:26-104``), restricted to the quantized MoE and
decode-GEMM path this package implements, so an existing launch profile
(``SGLANG_RESTOMOD_COMPONENTS=fp8_moe,fp8_dense,...``) selects the B200
kernels unchanged. Components outside this path are refused by name.

Each selected component is imported and registered on its own: a failure is
recorded in :mod:`.attest` and does not stop the others (SGLang wraps plugin
loading in ``except Exception``, so a raise would silently drop everything).
"""

from __future__ import annotations

import importlib
import logging
import os
from dataclasses import dataclass
from typing import Mapping, Sequence

logger = logging.getLogger(__name__)

ENV_COMPONENTS = "SGLANG_RESTOMOD_COMPONENTS"


@dataclass(frozen=True)
class Component:
    name: str
    module: str
    description: str


_PKG = "sglang_restomod_b200"

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

# Names the reference also knows but that are outside this path.
OUT_OF_SCOPE = ("attention_v100", "lsa_sm70", "sm70_marlin_v100", "ple_sm70", "spec_sm70",
                "gdn_tilelang_sm70")


def selection(env: Mapping[str, str] | None = None) -> list[str]:
    """Selected component names, validated and de-duplicated (order kept)."""
    raw = (env if env is not None else os.environ).get(ENV_COMPONENTS, "")
    names: list[str] = []
    for item in raw.split(","):
        name = item.strip()
        if name and name not in names:
            names.append(name)
    unknown = [n for n in names if n not in COMPONENTS]
    if unknown:
        scoped = [n for n in unknown if n in OUT_OF_SCOPE]
        hint = f" ({', '.join(scoped)} is not part of the B200 MoE/GEMV path)" if scoped else ""
        raise ValueError(
            f"unknown component(s) in {ENV_COMPONENTS}: {', '.join(unknown)}{hint}; "
            f"known: {', '.join(sorted(COMPONENTS))}"
        )
    return names


def is_enabled(name: str, env: Mapping[str, str] | None = None) -> bool:
    return name in selection(env)


def load_enabled(env: Mapping[str, str] | None = None) -> Sequence[str]:
    """Import and register every selected component; return the loaded names."""
    from . import attest

    selected = selection(env)
    attest.set_selected(selected)
    loaded: list[str] = []
    for name in selected:
        comp = COMPONENTS[name]
        try:
            module = importlib.import_module(comp.module)
        except Exception as exc:  # noqa: BLE001 - isolate each component
            attest.inactive(name, f"import failed: {type(exc).__name__}: {exc}")
            logger.warning("component %s failed to import", name, exc_info=True)
            continue
        register = getattr(module, "register", None)
        if register is None:
            attest.inactive(name, f"imported {comp.module} but it has no register()")
            continue
        try:
            register()
        except Exception as exc:  # noqa: BLE001
            attest.record(name, False, f"{type(exc).__name__}: {exc}")
            logger.warning("component %s failed to register", name, exc_info=True)
            continue
        attest.record(name, True)
        loaded.append(name)
    recorded = attest.snapshot()["components"]
    for name in sorted(set(selected) - set(recorded)):
        attest.inactive(name, "selected but never registered")
    attest.write()
    logger.info("sglang-restomod-b200: %d/%d components active (%s)", len(loaded),
                len(selected), ", ".join(loaded) or "none")
    return loaded
