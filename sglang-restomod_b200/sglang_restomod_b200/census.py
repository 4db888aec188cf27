"""Which kernel path served which shape, and an in-process profile window.

Census (``SGLANG_B200_CENSUS=1``): every call of the library's GEMM ops
through ``torch.ops.b200_moe`` is tallied by (op, kernel path, tile rows,
shape) - the path is the library's own decision, asked through
``b200_linear_path`` / ``b200_moe_path``, so the tally cannot drift from
what ran. :func:`report` returns one line per entry; the tally is logged
every ``SGLANG_B200_CENSUS_EVERY`` calls (default 1024) and at exit. In the
reference the same question ("which path serves which projection at which
batch size") is answered by the NVFP4 decode dispatcher's census
(``quant/sm70_fp4_moe/decode_gemv.py:66-104``); here it covers the FP8 and
NVFP4 MoE, dense and W8A8 calls alike. Calls replayed from a CUDA graph are
not seen (no Python runs); the census counts the captured call once.

Profile window (``SGLANG_B200_PROFILE=<steps>``, output
``SGLANG_B200_PROFILE_OUT``): :func:`install_profile` wraps SGLang's
``ModelRunner.forward`` so that `steps` forwards after the first run under
``torch.profiler`` (CUDA activity) and the kernel table is written once -
the in-process capture path the reference also uses (``overrides.py:
511-571``), since no external profiler can attach inside the serving
container. :class:`ProfileWindow` is the same window for any loop.

Neither raises into the caller: both are instruments, not control.
"""

from __future__ import annotations

import atexit
import ctypes
import logging
import os
from collections import Counter

logger = logging.getLogger(__name__)

ENV_CENSUS = "SGLANG_B200_CENSUS"
ENV_CENSUS_EVERY = "SGLANG_B200_CENSUS_EVERY"
ENV_PROFILE = "SGLANG_B200_PROFILE"
ENV_PROFILE_OUT = "SGLANG_B200_PROFILE_OUT"

_TALLY: Counter = Counter()
_calls = 0
_enabled = os.environ.get(ENV_CENSUS, "") == "1"
_every = max(1, int(os.environ.get(ENV_CENSUS_EVERY, "1024") or 1024))
_atexit_set = False


def enable(on: bool = True) -> None:
    """Switch the census on or off in-process (tests, benchmarks)."""
    global _enabled
    _enabled = bool(on)


def enabled() -> bool:
    return _enabled


def reset() -> None:
    global _calls
    _TALLY.clear()
    _calls = 0


def _path_name(code: int, rows: int, parts: int = 1) -> str:
    from . import _lib

    if code == _lib.PATH_TCGEN05:
        return "tcgen05" + (f"/k{parts}" if parts > 1 else "")
    if code == _lib.PATH_STREAM:
        return f"stream/{rows}rows"
    return "invalid"


def _record(key: tuple) -> None:
    global _calls, _atexit_set
    _TALLY[key] += 1
    _calls += 1
    if not _atexit_set:
        atexit.register(lambda: logger.info("%s", report()))
        _atexit_set = True
    if _calls % _every == 0:
        logger.info("%s", report())


def note_linear(op: str, m: int, n: int, k: int) -> None:
    """A dense call (W8A16 linear or GEMV) of m rows against [n, k]."""
    if not _enabled:
        return
    try:
        from . import _lib

        rows, parts = ctypes.c_int32(0), ctypes.c_int32(1)
        code = _lib.load().b200_linear_path(m, n, k, ctypes.byref(rows), ctypes.byref(parts))
        _record((op, _path_name(code, rows.value, parts.value), f"m={m}", f"n={n}", f"k={k}"))
    except Exception:  # noqa: BLE001 - an instrument never breaks the call
        logger.debug("census failed", exc_info=True)


def note_moe(op: str, quant: int, tokens: int, routes: int, experts: int, block: int,
             groups: int, n: int, k: int) -> None:
    """A routed call: `routes` routes over `experts` experts in blocks of `block`."""
    if not _enabled:
        return
    try:
        from . import _lib

        rows = ctypes.c_int32(0)
        code = _lib.load().b200_moe_path(quant, block, groups, ctypes.byref(rows))
        _record((op, _path_name(code, rows.value), f"q={quant}", f"tokens={tokens}",
                 f"routes/expert={routes / max(experts, 1):.1f}", f"block={block}", f"n={n}",
                 f"k={k}"))
    except Exception:  # noqa: BLE001
        logger.debug("census failed", exc_info=True)


def note(op: str, *shape) -> None:
    """Any other op (W8A8, routing, exchange): tallied by its shape only."""
    if not _enabled:
        return
    try:
        _record((op, "-", *[str(s) for s in shape]))
    except Exception:  # noqa: BLE001
        logger.debug("census failed", exc_info=True)


def tally() -> dict:
    return dict(_TALLY)


def report() -> str:
    rows = ", ".join(f"{' '.join(key)} x{count}" for key, count in sorted(_TALLY.items()))
    return f"b200 census ({_calls} calls): {rows or '<none>'}"


class ProfileWindow:
    """Profiles `steps` steps of a loop after its first one (the warm-up,
    e.g. graph capture) with torch.profiler and writes the CUDA kernel table
    to `path` once. Call :meth:`before` ahead of and :meth:`step` after every
    step."""

    def __init__(self, steps: int, path: str, row_limit: int = 40):
        self.steps = int(steps)
        self.path = path
        self.row_limit = row_limit
        self.seen = 0
        self.prof = None
        self.written = False

    def before(self) -> None:
        if self.written or self.prof is not None or self.seen != 1:
            return
        try:
            import torch

            self.prof = torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA])
            self.prof.__enter__()
        except Exception:  # noqa: BLE001
            logger.warning("b200 profile window could not start", exc_info=True)
            self.prof = None
            self.written = True

    def step(self) -> None:
        self.seen += 1
        if self.prof is None or self.seen <= self.steps:
            return
        prof, self.prof = self.prof, None
        self.written = True
        try:
            import torch

            torch.cuda.synchronize()
            prof.__exit__(None, None, None)
            table = prof.key_averages().table(sort_by="cuda_time_total", row_limit=self.row_limit)
            with open(self.path, "w") as fh:
                fh.write(table)
            logger.info("b200 profile window written to %s", self.path)
        except Exception:  # noqa: BLE001
            logger.warning("b200 profile window could not be written", exc_info=True)


def install_profile(runner_cls=None) -> bool:
    """Wrap ``ModelRunner.forward`` with a :class:`ProfileWindow` when
    ``SGLANG_B200_PROFILE`` is a positive step count. False when unset,
    invalid or already installed."""
    text = os.environ.get(ENV_PROFILE, "").strip()
    try:
        steps = int(text) if text else 0
    except ValueError:
        logger.warning("ignoring %s=%r (not a step count)", ENV_PROFILE, text)
        return False
    if steps <= 0:
        return False
    if runner_cls is None:
        try:
            from sglang.srt.model_executor.model_runner import ModelRunner as runner_cls
        except Exception:  # noqa: BLE001
            return False
    original = runner_cls.forward
    if getattr(original, "_b200_profile", False):
        return False
    import torch

    device = torch.cuda.current_device() if torch.cuda.is_available() else 0
    window = ProfileWindow(steps, os.environ.get(ENV_PROFILE_OUT,
                                                 f"/tmp/b200_profile_{device}.txt"))

    def forward(self, *args, **kwargs):
        window.before()
        result = original(self, *args, **kwargs)
        window.step()
        return result

    forward._b200_profile = True
    runner_cls.forward = forward
    return True
