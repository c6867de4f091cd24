"""Prometheus text exposition with the reference's metric names (coordinator/src/metrics.rs:46-107),
plus the device-side merge figures of the in-box data plane."""
from __future__ import annotations

import threading


class Metrics:
    _FIELDS = [
        ("checkpoint_version", "gauge", "Current checkpoint version.", "{}"),
        ("delta_pushes_total", "counter", "Total delta push requests.", "{}"),
        ("delta_pushes_accepted", "counter", "Accepted delta pushes.", "{}"),
        ("delta_pushes_rejected", "counter", "Rejected delta pushes.", "{}"),
        ("aggregations_total", "counter", "Total aggregation runs.", "{}"),
        ("aggregations_failed", "counter", "Failed aggregation runs.", "{}"),
        ("accumulator_contributions", "gauge", "Current contributions in accumulator.", "{}"),
        ("active_nodes", "gauge", "Number of active nodes.", "{}"),
        ("registered_nodes", "gauge", "Total registered nodes.", "{}"),
        ("last_aggregation_seconds", "gauge", "Duration of last aggregation.", "{:.4f}"),
        ("last_outer_delta_norm", "gauge", "Delta norm of last aggregation.", "{:.6f}"),
    ]
    _EXTRA = [
        ("merge_device_ms", "gauge", "Device time of the last in-box merge (pull + apply + broadcast).", "{:.3f}"),
        ("merge_pulled_bytes", "gauge", "Compressed payload bytes read over NVLink by the last merge.", "{}"),
    ]

    def __init__(self):
        self._lock = threading.Lock()
        for name, *_ in self._FIELDS + self._EXTRA:
            if name != "last_aggregation_seconds":
                setattr(self, name, 0)
        self.last_aggregation_secs = 0.0
        self.last_outer_delta_norm = 0.0
        self.merge_device_ms = 0.0

    def render(self) -> str:
        out = []
        for name, typ, help_, fmt in self._FIELDS + self._EXTRA:
            v = getattr(self, "last_aggregation_secs" if name == "last_aggregation_seconds" else name)
            out.append(f"# HELP distrain_{name} {help_}\n# TYPE distrain_{name} {typ}\ndistrain_{name} "
                       f"{fmt.format(v)}\n")
        return "\n".join(out)
