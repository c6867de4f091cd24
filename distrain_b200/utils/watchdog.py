"""Step watchdog (reference node/cli/src/trainer.rs:1098-1163): a training step that makes no progress for
max(6 x the expected step time, 300 s) is reported as hung instead of waiting forever.

The reference runs each round in a task under a timeout and returns ``TrainingFailure::GpuHung``. Here a
monitor thread watches a progress counter that the training loop bumps with ``beat()``; when it stalls
past the limit the thread calls ``on_timeout(seconds_stalled)`` once (the node records the failure and
stops its side threads; the process is left to its supervisor - device-side waits in this library are
bounded, so a stall means a host-side or driver problem)."""
from __future__ import annotations

import logging
import threading
import time
from typing import Callable, Optional

log = logging.getLogger("distrain_b200.watchdog")


def watchdog_limit(expected_step_secs: float, steps: int = 1, factor: float = 6.0, floor: float = 300.0) -> float:
    """The reference's limit: factor x the expected time of `steps` steps, at least `floor` seconds."""
    return max(steps * max(expected_step_secs, 0.0) * factor, floor)


class StepWatchdog:
    def __init__(self, limit_secs: float, on_timeout: Optional[Callable[[float], None]] = None,
                 poll_secs: float = 1.0):
        self.limit = float(limit_secs)
        self.on_timeout = on_timeout
        self.poll = min(poll_secs, max(self.limit / 10.0, 0.01))
        self.last = time.monotonic()
        self.fired = False
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()

    def beat(self):
        self.last = time.monotonic()

    def _run(self):
        while not self._stop.wait(self.poll):
            stalled = time.monotonic() - self.last
            if stalled > self.limit and not self.fired:
                self.fired = True
                log.error("training step stalled for %.0f s (limit %.0f s)", stalled, self.limit)
                if self.on_timeout is not None:
                    self.on_timeout(stalled)

    def close(self):
        self._stop.set()
        self._thread.join(timeout=5)
