"""S3 object store: AWS Signature Version 4 against AWS's published example, and S3Store end to end
against an in-process S3 endpoint that re-derives every request's signature from the request as it
arrived on the wire (path, query, headers, body) and implements PUT / GET / HEAD / DELETE, ListObjectsV2
with continuation tokens, and multipart uploads."""
import datetime as dt
import hashlib
import http.server
import threading
import urllib.parse

import pytest

from distrain_b200.config import StorageConfig
from distrain_b200.utils import storage as S


def test_sigv4_matches_the_published_aws_example():
    h = S.sigv4_headers("GET", "iam.amazonaws.com", "/", {"Action": "ListUsers", "Version": "2010-05-08"},
                        {"Content-Type": "application/x-www-form-urlencoded; charset=utf-8"}, b"", "AKIDEXAMPLE",
                        "wJalrXUtnFEMI/K7MDENG+bPxRfiCYEXAMPLEKEY", "us-east-1", service="iam",
                        now=dt.datetime(2015, 8, 30, 12, 36, 0, tzinfo=dt.timezone.utc))
    assert h["authorization"] == ("AWS4-HMAC-SHA256 Credential=AKIDEXAMPLE/20150830/us-east-1/iam/aws4_request, "
                                  "SignedHeaders=content-type;host;x-amz-date, "
                                  "Signature=5d672d79c15b13162d9279b0855cfba6789a8edb4c82c400e06b5924a6f2b5d7")


class _FakeS3(http.server.BaseHTTPRequestHandler):
    objects, uploads, bad_sigs, requests = {}, {}, [], []
    access, secret, page = "AKID", "SECRET", 2

    def log_message(self, *a):
        pass

    def _verify(self, body: bytes):
        u = urllib.parse.urlsplit(self.path)
        query = dict(urllib.parse.parse_qsl(u.query, keep_blank_values=True))
        auth = self.headers["authorization"]
        signed = auth.split("SignedHeaders=")[1].split(",")[0].split(";")
        extra = {k: self.headers[k] for k in signed if k not in ("host", "x-amz-date", "x-amz-content-sha256")}
        when = dt.datetime.strptime(self.headers["x-amz-date"], "%Y%m%dT%H%M%SZ").replace(tzinfo=dt.timezone.utc)
        want = S.sigv4_headers(self.command, self.headers["host"], urllib.parse.unquote(u.path), query, extra, body,
                               self.access, self.secret, "us-east-1", now=when)["authorization"]
        if want != auth or self.headers["x-amz-content-sha256"] != hashlib.sha256(body).hexdigest():
            self.bad_sigs.append(self.path)
        self.requests.append((self.command, u.path, query))
        return urllib.parse.unquote(u.path).split("/", 2), query

    def _reply(self, code, data=b"", headers=()):
        self.send_response(code)
        for k, v in headers:
            self.send_header(k, v)
        self.send_header("Content-Length", str(len(data)))
        self.end_headers()
        if self.command != "HEAD":
            self.wfile.write(data)

    def _body(self):
        n = int(self.headers.get("Content-Length", 0) or 0)
        return self.rfile.read(n) if n else b""

    def do_PUT(self):
        body = self._body()
        (_, _, key), q = self._verify(body)
        if "partNumber" in q:
            self.uploads[q["uploadId"]][int(q["partNumber"])] = body
            return self._reply(200, headers=[("ETag", f'"{hashlib.md5(body).hexdigest()}"')])
        self.objects[key] = body
        self._reply(200)

    def do_POST(self):
        body = self._body()
        (_, _, key), q = self._verify(body)
        if "uploads" in q:
            uid = f"u{len(self.uploads)}"
            self.uploads[uid] = {}
            xml = f"<InitiateMultipartUploadResult><UploadId>{uid}</UploadId></InitiateMultipartUploadResult>"
            return self._reply(200, xml.encode())
        parts = self.uploads.pop(q["uploadId"])
        self.objects[key] = b"".join(parts[i] for i in sorted(parts))
        self._reply(200, b"<CompleteMultipartUploadResult/>")

    def do_GET(self):
        parts, q = self._verify(b"")
        if q.get("list-type") == "2":
            keys = sorted(k for k in self.objects if k.startswith(q.get("prefix", "")))
            start = int(q.get("continuation-token", "0"))
            page = keys[start:start + self.page]
            more = start + self.page < len(keys)
            xml = "<ListBucketResult>" + "".join(f"<Contents><Key>{k}</Key></Contents>" for k in page) + (
                f"<NextContinuationToken>{start + self.page}</NextContinuationToken>" if more else "") + \
                "</ListBucketResult>"
            return self._reply(200, xml.encode())
        key = parts[2]
        if key not in self.objects:
            return self._reply(404)
        self._reply(200, self.objects[key])

    def do_HEAD(self):
        parts, _ = self._verify(b"")
        key = parts[2] if len(parts) > 2 else ""
        self._reply(200 if (not key or key in self.objects) else 404)

    def do_DELETE(self):
        (_, _, key), _ = self._verify(b"")
        self.objects.pop(key, None)
        self._reply(204)


@pytest.fixture
def s3(monkeypatch):
    srv = http.server.ThreadingHTTPServer(("127.0.0.1", 0), _FakeS3)
    t = threading.Thread(target=srv.serve_forever, daemon=True)
    t.start()
    _FakeS3.objects.clear(), _FakeS3.uploads.clear(), _FakeS3.bad_sigs.clear(), _FakeS3.requests.clear()
    monkeypatch.setattr(S, "MULTIPART_THRESHOLD", 1000)
    monkeypatch.setattr(S, "PART_SIZE", 400)
    cfg = StorageConfig(endpoint=f"http://127.0.0.1:{srv.server_address[1]}", bucket="bkt", access_key_id="AKID",
                        secret_access_key="SECRET", region="us-east-1")
    yield S.S3Store(cfg, retries=2)
    srv.shutdown()


def test_s3store_end_to_end_with_signed_requests(s3):
    s3.put("checkpoints/v1/model.safetensors", b"weights")
    s3.put("deltas/v1/node a_1.delta.zst", b"x" * 10)      # a space in the key: URI encoding on both sides
    big = bytes(range(256)) * 11                             # 2816 bytes: multipart in 400-byte parts
    s3.put("deltas/v1/big.delta.zst", big)
    assert s3.get("checkpoints/v1/model.safetensors") == b"weights"
    assert s3.get("deltas/v1/big.delta.zst") == big
    assert ("POST", "/bkt/deltas/v1/big.delta.zst", {"uploads": ""}) in _FakeS3.requests
    assert s3.exists("deltas/v1/node a_1.delta.zst") and not s3.exists("nope")
    keys = s3.list_keys("deltas/")                           # 2 per page: follows the continuation token
    assert keys == ["deltas/v1/big.delta.zst", "deltas/v1/node a_1.delta.zst"]
    s3.delete("deltas/v1/big.delta.zst")
    assert s3.list_keys("deltas/") == ["deltas/v1/node a_1.delta.zst"]
    with pytest.raises(S.StorageError):
        s3.get("deltas/v1/big.delta.zst")
    assert not _FakeS3.bad_sigs, _FakeS3.bad_sigs


def test_open_store_endpoint_uses_r2_environment(monkeypatch):
    """An S3 endpoint given as a string (a node's checkpoint store) signs with the R2_* credentials and
    writes into the R2_BUCKET bucket, not the built-in defaults."""
    srv = http.server.ThreadingHTTPServer(("127.0.0.1", 0), _FakeS3)
    t = threading.Thread(target=srv.serve_forever, daemon=True)
    t.start()
    try:
        _FakeS3.objects.clear(), _FakeS3.bad_sigs.clear(), _FakeS3.requests.clear()
        monkeypatch.setattr(_FakeS3, "access", "AKIDOTHER")
        monkeypatch.setattr(_FakeS3, "secret", "OTHERSECRET")
        env = {"R2_ACCESS_KEY_ID": "AKIDOTHER", "R2_SECRET_ACCESS_KEY": "OTHERSECRET", "R2_BUCKET": "runbucket",
               "R2_REGION": "us-east-1", "R2_ENDPOINT": "http://unused.invalid"}
        store = S.open_store(f"http://127.0.0.1:{srv.server_address[1]}", env=env)
        store.put("checkpoints/v3/model.safetensors", b"w3")
        assert store.get("checkpoints/v3/model.safetensors") == b"w3"
        assert ("PUT", "/runbucket/checkpoints/v3/model.safetensors", {}) in _FakeS3.requests
        assert not _FakeS3.bad_sigs, _FakeS3.bad_sigs
    finally:
        srv.shutdown()
