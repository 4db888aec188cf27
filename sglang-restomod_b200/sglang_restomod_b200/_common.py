"""Helpers shared by the components: mode switches, device check, and the
SGLang types they return (with stand-ins when SGLang is not importable, so the
components import and their host logic can be tested without it)."""

from __future__ import annotations

import os
from dataclasses import dataclass

MODES = ("auto", "on", "off")


def mode(env_name: str) -> str:
    """``auto`` (default), ``on`` or ``off``; anything else raises."""
    value = os.environ.get(env_name, "auto").strip().lower() or "auto"
    if value not in MODES:
        raise ValueError(f"{env_name} must be auto, on or off; got {value!r}")
    return value


def is_b200() -> bool:
    """True on an sm_100 device (B200)."""
    try:
        import torch

        return torch.cuda.is_available() and torch.cuda.get_device_capability() == (10, 0)
    except Exception:  # noqa: BLE001
        return False


def b200_ops():
    """``torch.ops.b200_moe``: the library's ops registered as torch custom ops
    (registration happens on the first call)."""
    import torch

    from . import torch_ops  # noqa: F401

    return torch.ops.b200_moe


def rebind_everywhere(attr: str, original, replacement) -> int:
    """Point every loaded module whose ``attr`` is ``original`` at
    ``replacement`` (modules that did ``from x import name`` before a hook was
    installed keep their own reference). Returns how many were rebound."""
    import sys

    count = 0
    for module in list(sys.modules.values()):
        if module is None:
            continue
        try:
            if getattr(module, attr, None) is original:
                setattr(module, attr, replacement)
                count += 1
        except Exception:  # noqa: BLE001 - half-imported or proxy modules
            continue
    return count


def library_loadable() -> bool:
    try:
        from . import _lib

        _lib.load()
        return True
    except Exception:  # noqa: BLE001
        return False


@dataclass
class CombineInput:
    """Stand-in for sglang's StandardCombineInput (only ``hidden_states``)."""

    hidden_states: object


def combine_input(hidden_states):
    try:
        from sglang.srt.layers.moe.token_dispatcher import StandardCombineInput

        return StandardCombineInput(hidden_states=hidden_states)
    except Exception:  # noqa: BLE001 - no sglang: plain result object
        return CombineInput(hidden_states=hidden_states)
