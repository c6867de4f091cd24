"""Object store behind the checkpoint / delta / data key layout (reference core/shared/src/storage.rs).

* ``FsStore``  - the default in-box store: a directory tree (``root/bucket/key``) with atomic writes.
* ``S3Store``  - S3 / R2 / MinIO over HTTP with AWS Signature V4 (path-style addressing like the
  reference's client, storage.rs:20-44), retries with 2^n s backoff (storage.rs:57-90) and
  multipart upload above 100 MB (storage.rs:93-172).
Both expose put/get/exists/delete/list_keys/get_json/put_json/download_to_file/upload_from_file.
"""
from __future__ import annotations

import datetime as _dt
import hashlib
import hmac
import http.client
import json
import os
import tempfile
import time
import urllib.parse
from typing import List, Optional
from xml.etree import ElementTree

from ..config import StorageConfig

MULTIPART_THRESHOLD = 100 * 1024 * 1024
PART_SIZE = 64 * 1024 * 1024


class StorageError(RuntimeError):
    pass


class ObjectStore:
    def put(self, key: str, data: bytes) -> None: ...
    def get(self, key: str) -> bytes: ...
    def exists(self, key: str) -> bool: ...
    def delete(self, key: str) -> None: ...
    def list_keys(self, prefix: str) -> List[str]: ...

    def get_json(self, key: str):
        return json.loads(self.get(key))

    def put_json(self, key: str, obj) -> None:
        self.put(key, json.dumps(obj).encode())

    def download_to_file(self, key: str, path: str) -> None:
        data = self.get(key)
        tmp = path + ".tmp"
        with open(tmp, "wb") as f:
            f.write(data)
        os.replace(tmp, path)

    def upload_from_file(self, path: str, key: str) -> None:
        with open(path, "rb") as f:
            self.put(key, f.read())

    def ensure_bucket(self) -> None:
        pass


class FsStore(ObjectStore):
    def __init__(self, root: str, bucket: str = "distrain-training"):
        self.base = os.path.join(root, bucket)
        os.makedirs(self.base, exist_ok=True)

    def _path(self, key: str) -> str:
        key = key.lstrip("/")
        p = os.path.normpath(os.path.join(self.base, key))
        if not p.startswith(os.path.normpath(self.base)):
            raise StorageError(f"key escapes the bucket: {key}")
        return p

    def put(self, key, data):
        p = self._path(key)
        os.makedirs(os.path.dirname(p), exist_ok=True)
        fd, tmp = tempfile.mkstemp(dir=os.path.dirname(p), prefix=".put-")
        with os.fdopen(fd, "wb") as f:
            f.write(data)
        os.replace(tmp, p)

    def get(self, key):
        try:
            with open(self._path(key), "rb") as f:
                return f.read()
        except FileNotFoundError:
            raise StorageError(f"no such key: {key}") from None

    def exists(self, key):
        return os.path.exists(self._path(key))

    def delete(self, key):
        try:
            os.remove(self._path(key))
        except FileNotFoundError:
            pass

    def list_keys(self, prefix):
        out = []
        for dp, _, files in os.walk(self.base):
            for f in files:
                if f.startswith(".put-"):
                    continue
                k = os.path.relpath(os.path.join(dp, f), self.base).replace(os.sep, "/")
                if k.startswith(prefix):
                    out.append(k)
        return sorted(out)


# ─────────────────────────────── S3 (SigV4) ───────────────────────────────
def _sha256(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


def _hmac(key: bytes, msg: str) -> bytes:
    return hmac.new(key, msg.encode(), hashlib.sha256).digest()


def sigv4_headers(method: str, host: str, path: str, query: dict, headers: dict, payload: bytes, access_key: str,
                  secret_key: str, region: str, service: str = "s3", now: Optional[_dt.datetime] = None,
                  unsigned_payload: bool = False) -> dict:
    """AWS Signature Version 4: returns headers (incl. Authorization) to send."""
    now = now or _dt.datetime.now(_dt.timezone.utc)
    amz_date = now.strftime("%Y%m%dT%H%M%SZ")
    datestamp = now.strftime("%Y%m%d")
    phash = "UNSIGNED-PAYLOAD" if unsigned_payload else _sha256(payload)
    h = {k.lower(): str(v).strip() for k, v in headers.items()}
    h["host"] = host
    h["x-amz-date"] = amz_date
    if service == "s3":
        h["x-amz-content-sha256"] = phash
    signed = sorted(h)
    canon_headers = "".join(f"{k}:{h[k]}\n" for k in signed)
    canon_query = "&".join(f"{urllib.parse.quote(str(k), safe='-_.~')}={urllib.parse.quote(str(v), safe='-_.~')}"
                           for k, v in sorted(query.items()))
    canon_uri = urllib.parse.quote(path, safe="/-_.~")
    creq = "\n".join([method, canon_uri, canon_query, canon_headers, ";".join(signed), phash])
    scope = f"{datestamp}/{region}/{service}/aws4_request"
    sts = "\n".join(["AWS4-HMAC-SHA256", amz_date, scope, _sha256(creq.encode())])
    k = _hmac(("AWS4" + secret_key).encode(), datestamp)
    k = _hmac(k, region)
    k = _hmac(k, service)
    k = _hmac(k, "aws4_request")
    sig = hmac.new(k, sts.encode(), hashlib.sha256).hexdigest()
    out = dict(h)
    out["authorization"] = (f"AWS4-HMAC-SHA256 Credential={access_key}/{scope}, SignedHeaders={';'.join(signed)}, "
                            f"Signature={sig}")
    return out


class S3Store(ObjectStore):
    def __init__(self, cfg: StorageConfig, retries: int = 5):
        self.cfg = cfg
        u = urllib.parse.urlparse(cfg.endpoint)
        self.scheme, self.host = u.scheme or "http", u.netloc
        self.region = cfg.region if cfg.region and cfg.region != "auto" else "us-east-1"
        self.retries = retries

    def _request(self, method, key, query=None, body=b"", extra=None, ok=(200, 204)):
        path = f"/{self.cfg.bucket}" + (f"/{key}" if key else "")
        query = query or {}
        last = None
        for attempt in range(self.retries):
            try:
                hdrs = sigv4_headers(method, self.host, path, query, extra or {}, body, self.cfg.access_key_id,
                                     self.cfg.secret_access_key, self.region)
                conn_cls = http.client.HTTPSConnection if self.scheme == "https" else http.client.HTTPConnection
                conn = conn_cls(self.host, timeout=300)
                qs = "&".join(f"{urllib.parse.quote(str(k), safe='-_.~')}={urllib.parse.quote(str(v), safe='-_.~')}"
                              for k, v in sorted(query.items()))
                conn.request(method, urllib.parse.quote(path, safe="/-_.~") + (f"?{qs}" if qs else ""), body=body,
                             headers=hdrs)
                r = conn.getresponse()
                data = r.read()
                if r.status in ok:
                    return r, data
                if r.status == 404:
                    raise StorageError(f"{method} {key}: 404")
                last = StorageError(f"{method} {key}: HTTP {r.status} {data[:200]!r}")
            except StorageError:
                raise
            except Exception as e:  # network error -> retry
                last = e
            time.sleep(2 ** attempt if attempt < self.retries - 1 else 0)
        raise StorageError(f"{method} {key} failed after {self.retries} attempts: {last}")

    def put(self, key, data):
        if len(data) > MULTIPART_THRESHOLD:
            return self._put_multipart(key, data)
        self._request("PUT", key, body=data)

    def _put_multipart(self, key, data):
        _, resp = self._request("POST", key, query={"uploads": ""})
        upload_id = ElementTree.fromstring(resp).find("{*}UploadId").text
        etags = []
        for i in range(0, len(data), PART_SIZE):
            n = i // PART_SIZE + 1
            r, _ = self._request("PUT", key, query={"partNumber": n, "uploadId": upload_id},
                                 body=data[i:i + PART_SIZE])
            etags.append((n, r.getheader("ETag")))
        xml = "<CompleteMultipartUpload>" + "".join(
            f"<Part><PartNumber>{n}</PartNumber><ETag>{e}</ETag></Part>" for n, e in etags) + \
            "</CompleteMultipartUpload>"
        self._request("POST", key, query={"uploadId": upload_id}, body=xml.encode())

    def get(self, key):
        return self._request("GET", key)[1]

    def exists(self, key):
        try:
            self._request("HEAD", key)
            return True
        except StorageError:
            return False

    def delete(self, key):
        self._request("DELETE", key, ok=(200, 204, 404))

    def list_keys(self, prefix):
        keys, token = [], None
        while True:
            q = {"list-type": "2", "prefix": prefix}
            if token:
                q["continuation-token"] = token
            _, data = self._request("GET", "", query=q)
            root = ElementTree.fromstring(data)
            keys += [e.find("{*}Key").text for e in root.findall("{*}Contents")]
            t = root.find("{*}NextContinuationToken")
            if t is None or not t.text:
                break
            token = t.text
        return keys

    def ensure_bucket(self):
        try:
            self._request("HEAD", "")
        except StorageError:
            self._request("PUT", "")


def open_store(url_or_cfg, env=None) -> ObjectStore:
    """``file:///path`` / plain path -> FsStore; StorageConfig / http(s) endpoint -> S3Store.

    An endpoint string takes its bucket, region and credentials from the R2_* environment (``env``, or
    the process environment), as the coordinator does, and overrides only the endpoint."""
    if isinstance(url_or_cfg, StorageConfig):
        if url_or_cfg.endpoint.startswith("file://"):
            return FsStore(url_or_cfg.endpoint[len("file://"):], url_or_cfg.bucket)
        return S3Store(url_or_cfg)
    s = str(url_or_cfg)
    if s.startswith("http://") or s.startswith("https://"):
        from ..config import CoordinatorConfig
        cfg = CoordinatorConfig.from_env(env).storage
        cfg.endpoint = s
        return S3Store(cfg)
    if s.startswith("file://"):
        s = s[len("file://"):]
    return FsStore(s)
