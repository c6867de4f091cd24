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


class MetricsServer:
    """Serves ``GET /metrics`` (Prometheus text) and ``GET /health`` for a ``Metrics`` object on the native
    HTTP server (the in-box coordinator's equivalent of the coordinator service's /metrics route)."""

    def __init__(self, metrics: Metrics, host: str = "0.0.0.0", port: int = 0, threads: int = 2):
        import ctypes
        from ..utils import native
        self.metrics = metrics
        handler_t = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_void_p,
                                     ctypes.c_longlong, ctypes.c_void_p)
        L = native.rt()
        native.register("dtr_http_start", [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_longlong, handler_t,
                                           ctypes.c_void_p], ctypes.c_void_p)
        native.register("dtr_http_port", [ctypes.c_void_p], ctypes.c_int)
        native.register("dtr_http_stop", [ctypes.c_void_p], None)
        native.register("dtr_http_respond", [ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_void_p,
                                             ctypes.c_longlong], None)
        self._L = L

        def on_request(ctx, method, path, body, blen, resp):
            p = path.decode().split("?", 1)[0]
            if p == "/metrics":
                with self.metrics._lock:
                    out = self.metrics.render().encode()
                status, ctype = 200, b"text/plain; version=0.0.4"
            elif p == "/health":
                status, ctype, out = 200, b"text/plain", b"ok"
            else:
                status, ctype, out = 404, b"text/plain", b"not found"
            L.dtr_http_respond(resp, status, ctype, out, len(out))

        self._cb = handler_t(on_request)
        self.handle = L.dtr_http_start(host.encode(), port, threads, 1 << 16, self._cb, None)
        if not self.handle:
            raise RuntimeError(f"metrics server: cannot bind {host}:{port}")
        self.port = L.dtr_http_port(self.handle)

    def stop(self):
        if self.handle:
            self._L.dtr_http_stop(self.handle)
            self.handle = None
