"""Tracing for the node and coordinator runtimes.

* ``nvtx(name)`` - a context manager that pushes an NVTX range around a host phase (a training step, a
  push, a swap, each merge phase), so an Nsight Systems timeline or an ``ncu --nvtx`` filter lines GPU
  work up with the phase that launched it. A no-op without CUDA or with ``DT_NVTX=0``. Ranges opened
  while a CUDA graph is being captured are not replayed with the graph; the per-step ranges are opened
  around the replay.
* ``setup_logging()`` - an environment filter in the style of the reference's ``RUST_LOG``
  (coordinator/src/main.rs:43-48, node/cli/src/main.rs:126-131): ``DT_LOG=info`` or
  ``DT_LOG=warning,distrain_b200.parallel=debug`` (a default level, then per-logger levels).
* ``PhaseTimer`` - wall-clock timers of the named phases of one operation, logged at debug level and
  returned as a dict (the reference times merge phases, aggregation.rs:162,346-381, and checkpoint
  swaps, continuous.rs:460,498-501, the same way).
"""
from __future__ import annotations

import contextlib
import logging
import os
import time
from typing import Dict, Optional

_nvtx_mod = None
_nvtx_state = None  # None = undecided, False = off


def _nvtx():
    global _nvtx_mod, _nvtx_state
    if _nvtx_state is None:
        _nvtx_state = False
        if os.environ.get("DT_NVTX", "1") != "0":
            try:
                import torch
                if torch.cuda.is_available():
                    import torch.cuda.nvtx as nv
                    nv.range_push("dt")
                    nv.range_pop()
                    _nvtx_mod, _nvtx_state = nv, True
            except Exception:
                _nvtx_state = False
    return _nvtx_mod if _nvtx_state else None


@contextlib.contextmanager
def nvtx(name: str):
    nv = _nvtx()
    if nv is None:
        yield
        return
    nv.range_push(name)
    try:
        yield
    finally:
        nv.range_pop()


def setup_logging(spec: Optional[str] = None, stream=None):
    """Configure logging from ``spec`` (default: the DT_LOG environment variable, else "warning")."""
    spec = spec if spec is not None else os.environ.get("DT_LOG", "warning")
    default = logging.WARNING
    per = {}
    for part in [p.strip() for p in spec.split(",") if p.strip()]:
        if "=" in part:
            name, lvl = part.split("=", 1)
            per[name.strip()] = lvl.strip().upper()
        else:
            default = getattr(logging, part.upper(), logging.WARNING)
    root = logging.getLogger()
    # one handler of ours at a time, on the stream of the latest call (stderr by default)
    for old in [h for h in root.handlers if getattr(h, "_dt", False)]:
        root.removeHandler(old)
    h = logging.StreamHandler(stream)
    h.setFormatter(logging.Formatter("%(asctime)s %(levelname)s %(name)s: %(message)s"))
    h._dt = True
    root.addHandler(h)
    root.setLevel(default)
    for name, lvl in per.items():
        logging.getLogger(name).setLevel(getattr(logging, lvl, logging.INFO))


class PhaseTimer:
    """``with t.phase("apply"): ...`` accumulates wall seconds per phase; ``t.report()`` logs them."""

    def __init__(self, what: str, logger: Optional[logging.Logger] = None):
        self.what = what
        self.log = logger or logging.getLogger("distrain_b200")
        self.t0 = time.perf_counter()
        self.phases: Dict[str, float] = {}

    @contextlib.contextmanager
    def phase(self, name: str):
        t = time.perf_counter()
        with nvtx(f"{self.what}/{name}"):
            try:
                yield
            finally:
                self.phases[name] = self.phases.get(name, 0.0) + time.perf_counter() - t

    def report(self, **extra) -> Dict[str, float]:
        out = {k: round(v * 1e3, 3) for k, v in self.phases.items()}
        out["total_ms"] = round((time.perf_counter() - self.t0) * 1e3, 3)
        if self.log.isEnabledFor(logging.DEBUG):
            self.log.debug("%s %s %s", self.what, " ".join(f"{k}={v}" for k, v in out.items()),
                           " ".join(f"{k}={v}" for k, v in extra.items()))
        return out
