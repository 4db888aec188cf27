"""Which components are active, as a record observers can check.

Same states and JSON output as the reference's attestation
(``sglang_restomod/attest.py:40-194``): a selected component is *loaded*
(registered and in use), *failed* (its registration raised), or *inactive*
(registered but doing nothing, with the reason) - the third state is the one
a silent fallback would otherwise hide. ``SGLANG_RESTOMOD_ATTEST=<path>``
writes the record as JSON. Nothing here raises.
"""

from __future__ import annotations

import json
import logging
import os
import sys
import tempfile
from typing import Any

logger = logging.getLogger(__name__)

ENV_ATTEST = "SGLANG_RESTOMOD_ATTEST"

_EMPTY = {"selected": [], "components": {}, "loaded": [], "failed": [], "inactive": []}
_STATE: dict[str, Any] = json.loads(json.dumps(_EMPTY))


def reset() -> None:
    """Forget every record (tests)."""
    _STATE.clear()
    _STATE.update(json.loads(json.dumps(_EMPTY)))


def set_selected(names) -> None:
    _STATE["selected"] = list(names)


def _add(bucket: str, name: str) -> None:
    if name not in _STATE[bucket]:
        _STATE[bucket].append(name)


def _drop(bucket: str, name: str) -> None:
    if name in _STATE[bucket]:
        _STATE[bucket].remove(name)


def record(name: str, ok: bool, detail: str = "") -> None:
    """Outcome of one component's register(); keeps an earlier inactive reason."""
    previous = _STATE["components"].get(name) or {}
    entry: dict[str, Any] = {"ok": bool(ok)}
    if detail:
        entry["detail"] = detail
    elif previous.get("detail"):
        entry["detail"] = previous["detail"]
    _STATE["components"][name] = entry
    if ok:
        _add("loaded", name)
        _drop("failed", name)
    else:
        _add("failed", name)
        _drop("loaded", name)


def inactive(name: str, reason: Any) -> None:
    """The component registered but will do nothing (and why)."""
    try:
        text = str(reason)
    except Exception:  # noqa: BLE001 - observability must not raise
        text = "<unprintable reason>"
    try:
        entry = _STATE["components"].setdefault(name, {"ok": True})
        entry["detail"] = "registered, inactive: " + text
        _add("inactive", name)
        _add("loaded", name)
        _drop("failed", name)
    except Exception:  # noqa: BLE001
        logger.debug("attest.inactive failed for %s", name, exc_info=True)


def engine() -> dict[str, Any]:
    mod = sys.modules.get("sglang")
    return {
        "python": sys.version.split()[0],
        "path": getattr(mod, "__file__", None) if mod else None,
        "version": getattr(mod, "__version__", None) if mod else None,
    }


def snapshot() -> dict[str, Any]:
    out = {
        "engine": engine(),
        "selected": list(_STATE["selected"]),
        "loaded": list(_STATE["loaded"]),
        "failed": list(_STATE["failed"]),
        "inactive": list(_STATE["inactive"]),
        "components": {k: dict(v) for k, v in _STATE["components"].items()},
    }
    out["missing"] = [n for n in out["selected"] if n not in out["components"]]
    return out


def write(path: str | None = None) -> str | None:
    """Write the snapshot as JSON (atomically); None when no path is set."""
    target = path or os.environ.get(ENV_ATTEST)
    if not target:
        return None
    try:
        directory = os.path.dirname(os.path.abspath(target)) or "."
        fd, tmp = tempfile.mkstemp(prefix=".attest-", dir=directory)
        with os.fdopen(fd, "w") as fh:
            json.dump(snapshot(), fh, indent=2, sort_keys=True)
        os.replace(tmp, target)
        return target
    except Exception:  # noqa: BLE001 - an unwritable path must not stop a server
        logger.warning("could not write attestation to %s", target, exc_info=True)
        return None
