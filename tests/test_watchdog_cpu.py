"""Step watchdog: fires once when the progress counter stalls past the limit, never while steps beat."""
import time

from distrain_b200.utils.watchdog import StepWatchdog, watchdog_limit


def test_limit_rule():
    assert watchdog_limit(0.1, steps=50) == 300.0
    assert watchdog_limit(2.0, steps=50) == 600.0


def test_fires_once_on_stall_and_not_while_beating():
    fired = []
    wd = StepWatchdog(0.3, on_timeout=fired.append, poll_secs=0.02)
    for _ in range(20):  # 0.4 s of regular progress
        time.sleep(0.02)
        wd.beat()
    assert not fired
    time.sleep(0.6)
    wd.close()
    assert len(fired) == 1 and fired[0] > 0.3
