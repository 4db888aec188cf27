"""A ledger of what each selected component actually did.

SGLang loads plugins inside ``except Exception`` and its plugin log lines do
not always reach a server's log, so "the component is on" cannot be read off
the logs. Every selected component therefore ends in one of three states,
kept here per component:

``LOADED``    its ``register()`` returned and the component serves its path;
``INACTIVE``  it registered but steps aside (not a B200, library missing,
              upstream symbol absent, ...), with the reason - the state a
              silent fallback would otherwise hide;
``FAILED``    its import or ``register()`` raised (the message is kept).

A component may report INACTIVE from inside ``register()``; the successful
return that follows does not hide it. A failure overrides both.

Observers read :func:`snapshot` in-process, or the JSON file named by
``SGLANG_RESTOMOD_ATTEST``. The JSON keys (``selected``, ``loaded``,
``failed``, ``inactive``, ``missing``, ``components{name: {ok, detail}}``,
``engine``) are the reference plugin's attestation format
(``sglang_restomod/attest.py``), kept so existing verifiers read this file
unchanged; INACTIVE components count as loaded there, with an
``"registered, inactive: "`` detail. Nothing in this module raises.
"""

from __future__ import annotations

import enum
import json
import logging
import os
import sys
from dataclasses import dataclass, field

logger = logging.getLogger(__name__)

ENV_ATTEST = "SGLANG_RESTOMOD_ATTEST"
INACTIVE_PREFIX = "registered, inactive: "


class State(enum.Enum):
    LOADED = "loaded"
    INACTIVE = "inactive"
    FAILED = "failed"


@dataclass
class Entry:
    state: State
    detail: str = ""


@dataclass
class Ledger:
    selected: tuple[str, ...] = ()
    entries: dict[str, Entry] = field(default_factory=dict)

    def loaded(self, name: str, detail: str = "") -> None:
        """register() returned. An INACTIVE or FAILED state reported earlier
        stands; only the detail is filled in when none was given."""
        entry = self.entries.get(name)
        if entry is None:
            self.entries[name] = Entry(State.LOADED, detail)
        elif detail and not entry.detail:
            entry.detail = detail

    def inactive(self, name: str, reason: str) -> None:
        entry = self.entries.get(name)
        if entry is not None and entry.state is State.FAILED:
            return
        self.entries[name] = Entry(State.INACTIVE, reason)

    def failed(self, name: str, detail: str) -> None:
        self.entries[name] = Entry(State.FAILED, detail)

    def names_in(self, *states: State) -> list[str]:
        return [n for n, e in self.entries.items() if e.state in states]

    def as_json(self) -> dict:
        components = {}
        for name, entry in self.entries.items():
            detail = entry.detail
            if entry.state is State.INACTIVE:
                detail = INACTIVE_PREFIX + detail
            item = {"ok": entry.state is not State.FAILED}
            if detail:
                item["detail"] = detail
            components[name] = item
        return {
            "engine": _engine(),
            "selected": list(self.selected),
            "loaded": self.names_in(State.LOADED, State.INACTIVE),
            "failed": self.names_in(State.FAILED),
            "inactive": self.names_in(State.INACTIVE),
            "missing": [n for n in self.selected if n not in self.entries],
            "components": components,
        }


_LEDGER = Ledger()


def _text(value) -> str:
    try:
        return str(value)
    except Exception:  # noqa: BLE001 - a reason that cannot print is still a reason
        return "<unprintable reason>"


def _engine() -> dict:
    sglang = sys.modules.get("sglang")
    return {
        "python": sys.version.split()[0],
        "path": getattr(sglang, "__file__", None),
        "version": getattr(sglang, "__version__", None),
    }


def ledger() -> Ledger:
    return _LEDGER


def reset() -> None:
    """Start a new ledger (tests)."""
    global _LEDGER
    _LEDGER = Ledger()


def set_selected(names) -> None:
    _LEDGER.selected = tuple(names)


def record(name: str, ok: bool, detail: str = "") -> None:
    """Outcome of a component's import / register()."""
    try:
        if ok:
            _LEDGER.loaded(name, _text(detail) if detail else "")
        else:
            _LEDGER.failed(name, _text(detail))
    except Exception:  # noqa: BLE001
        logger.debug("attest.record failed for %s", name, exc_info=True)


def inactive(name: str, reason) -> None:
    """The component registered but will do nothing, and why."""
    try:
        _LEDGER.inactive(name, _text(reason))
    except Exception:  # noqa: BLE001
        logger.debug("attest.inactive failed for %s", name, exc_info=True)


def snapshot() -> dict:
    return _LEDGER.as_json()


def write(path: str | None = None) -> str | None:
    """Write the snapshot as JSON to ``path`` (default: $SGLANG_RESTOMOD_ATTEST),
    replacing the file in one rename; None when no path is set or it failed."""
    target = path or os.environ.get(ENV_ATTEST)
    if not target:
        return None
    partial = f"{target}.{os.getpid()}.partial"
    try:
        text = json.dumps(snapshot(), indent=2, sort_keys=True)
        with open(partial, "w") as fh:
            fh.write(text)
            fh.flush()
            os.fsync(fh.fileno())
        os.replace(partial, target)
        return target
    except Exception:  # noqa: BLE001 - an unwritable path must not stop a server
        logger.warning("could not write the attestation to %s", target, exc_info=True)
        try:
            os.unlink(partial)
        except OSError:
            pass
        return None
