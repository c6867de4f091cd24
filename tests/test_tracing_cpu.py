"""Tracing helpers: the DT_LOG-style filter, phase timers, NVTX ranges as no-ops without CUDA."""
import io
import logging

from distrain_b200.utils.tracing import PhaseTimer, nvtx, setup_logging


def test_log_filter_default_and_per_logger():
    buf = io.StringIO()
    setup_logging("warning,distrain_b200.inbox=debug", stream=buf)
    logging.getLogger("distrain_b200.inbox").debug("swap seen")
    logging.getLogger("distrain_b200.coordinator").info("hidden")
    logging.getLogger("other").warning("shown")
    out = buf.getvalue()
    assert "swap seen" in out and "shown" in out and "hidden" not in out
    setup_logging("warning")


def test_phase_timer_and_nvtx():
    t = PhaseTimer("merge", logging.getLogger("distrain_b200.test"))
    with t.phase("plan"):
        with nvtx("inner"):
            pass
    with t.phase("apply"):
        pass
    with t.phase("apply"):
        pass
    r = t.report(version=3)
    assert set(r) == {"plan", "apply", "total_ms"} and r["total_ms"] >= r["plan"] >= 0
