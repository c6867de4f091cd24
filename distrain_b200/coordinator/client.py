"""Node-side HTTP client of the coordinator API (reference node/cli/src/client.rs:7-164).

Persistent keep-alive connection per thread; ``heartbeat_sync`` uses a 2 s timeout like the
reference's blocking heartbeat (client.rs:110-135)."""
from __future__ import annotations

import http.client
import json
import threading
import urllib.parse
from typing import Optional

from .. import protocol as P


class CoordinatorError(RuntimeError):
    pass


class CoordinatorClient:
    def __init__(self, base_url: str, timeout: float = 30.0):
        u = urllib.parse.urlparse(base_url)
        self.scheme, self.host, self.timeout = u.scheme or "http", u.netloc, timeout
        self._tls = threading.local()

    def _conn(self, timeout=None):
        c = getattr(self._tls, "c", None)
        if c is None or (timeout is not None and c.timeout != timeout):
            cls = http.client.HTTPSConnection if self.scheme == "https" else http.client.HTTPConnection
            c = cls(self.host, timeout=timeout or self.timeout)
            self._tls.c = c
        return c

    def request(self, method: str, path: str, body: Optional[bytes] = None, ctype="application/json", timeout=None):
        for attempt in range(2):
            c = self._conn(timeout)
            try:
                hdrs = {"Content-Type": ctype} if body is not None else {}
                c.request(method, path, body=body, headers=hdrs)
                r = c.getresponse()
                data = r.read()
                return r.status, data
            except (http.client.HTTPException, ConnectionError, OSError):
                self._tls.c = None
                if attempt == 1:
                    raise
        raise CoordinatorError("unreachable")

    def _json(self, method, path, obj=None, timeout=None):
        st, data = self.request(method, path, json.dumps(obj).encode() if obj is not None else None, timeout=timeout)
        if st != 200:
            raise CoordinatorError(f"{method} {path}: HTTP {st}: {data[:200]!r}")
        return json.loads(data)

    def register(self, req: P.RegisterRequest) -> P.RegisterResponse:
        return P.RegisterResponse.from_dict(self._json("POST", "/nodes/register", req.to_dict()))

    def push_delta(self, push: P.DeltaPush) -> P.DeltaPushResponse:
        return P.DeltaPushResponse.from_dict(self._json("POST", "/delta", push.to_dict()))

    def get_latest_checkpoint(self) -> P.CheckpointInfo:
        return P.CheckpointInfo.from_dict(self._json("GET", "/checkpoint/latest"))

    def heartbeat(self, req: P.HeartbeatRequest) -> P.HeartbeatResponse:
        return P.HeartbeatResponse.from_dict(self._json("POST", "/heartbeat", req.to_dict()))

    def heartbeat_sync(self, req: P.HeartbeatRequest) -> P.HeartbeatResponse:
        return P.HeartbeatResponse.from_dict(self._json("POST", "/heartbeat", req.to_dict(), timeout=2.0))

    def get_config(self) -> dict:
        return self._json("GET", "/config")

    def get_status(self) -> P.TrainingStatus:
        return P.TrainingStatus.from_dict(self._json("GET", "/status"))

    def health(self) -> bool:
        try:
            return self._json("GET", "/health").get("status") == "ok"
        except Exception:
            return False

    def metrics(self) -> str:
        st, data = self.request("GET", "/metrics")
        return data.decode()

    def upload(self, key: str, data: bytes):
        st, _ = self.request("PUT", f"/upload/{key}", data, ctype="application/octet-stream")
        if st != 200:
            raise CoordinatorError(f"upload {key}: HTTP {st}")

    def download(self, key: str) -> bytes:
        st, data = self.request("GET", f"/download/{key}")
        if st != 200:
            raise CoordinatorError(f"download {key}: HTTP {st}")
        return data
