"""SigV4 signing against the AWS documentation's example, and the S3 client (get / range / put /
head / paginated list / localize) against a local fake S3 server that checks every signature."""

import datetime
import hashlib
import hmac
import os
import threading
import urllib.parse
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

import pytest

from marin_experiments_b200.utils import s3

AK, SK = "AKIDEXAMPLE", "wJalrXUtnFEMI/K7MDENG+bPxRfiCYEXAMPLEKEY"


def test_signing_key_and_signature_match_published_example():
    assert s3.signing_key(SK, "20120215", "us-east-1", "iam").hex() == \
        "f4780e2d9f65fa895f9c67b32ce1baf0b0d8a43505a000a1a9e090d414db404d"
    hdrs = s3.sign("GET", "https://iam.amazonaws.com/?Action=ListUsers&Version=2010-05-08", access_key=AK,
                   secret_key=SK, region="us-east-1", service="iam",
                   headers={"content-type": "application/x-www-form-urlencoded; charset=utf-8"},
                   when=datetime.datetime(2015, 8, 30, 12, 36, 0, tzinfo=datetime.timezone.utc))
    assert hdrs["Authorization"].endswith(
        "SignedHeaders=content-type;host;x-amz-date, "
        "Signature=5d672d79c15b13162d9279b0855cfba6789a8edb4c82c400e06b5924a6f2b5d7")


class _FakeS3(BaseHTTPRequestHandler):
    objects: dict = {}
    page = 2

    def log_message(self, *a):
        pass

    def _check_sig(self, body: bytes) -> bool:
        auth = self.headers.get("Authorization", "")
        signed = auth.split("SignedHeaders=")[1].split(",")[0].split(";")
        hdrs = {h: self.headers[h] for h in signed}
        url = f"http://{self.headers['host']}{self.path}"
        when = datetime.datetime.strptime(self.headers["x-amz-date"], "%Y%m%dT%H%M%SZ").replace(
            tzinfo=datetime.timezone.utc)
        want = s3.sign(self.command, url, access_key=AK, secret_key=SK, region="us-east-1", payload=body,
                       headers={k: v for k, v in hdrs.items() if k not in ("host", "x-amz-date", "x-amz-content-sha256")},
                       when=when)
        return hmac.compare_digest(want["Authorization"], auth) and \
            self.headers["x-amz-content-sha256"] == hashlib.sha256(body).hexdigest()

    def _key(self):
        p = urllib.parse.urlparse(self.path)
        parts = urllib.parse.unquote(p.path).lstrip("/").split("/", 1)
        return parts[0], (parts[1] if len(parts) > 1 else ""), dict(urllib.parse.parse_qsl(p.query))

    def _reply(self, code, body=b"", headers=None):
        self.send_response(code)
        for k, v in (headers or {}).items():
            self.send_header(k, v)
        self.send_header("Content-Length", str(len(body)))
        self.end_headers()
        if self.command != "HEAD":
            self.wfile.write(body)

    def do_PUT(self):
        body = self.rfile.read(int(self.headers.get("Content-Length", 0)))
        if not self._check_sig(body):
            return self._reply(403, b"bad signature")
        b, k, _ = self._key()
        self.objects[(b, k)] = body
        self._reply(200)

    def do_HEAD(self):
        if not self._check_sig(b""):
            return self._reply(403)
        b, k, _ = self._key()
        if (b, k) not in self.objects:
            return self._reply(404)
        self.send_response(200)
        self.send_header("Content-Length", str(len(self.objects[(b, k)])))
        self.end_headers()

    def do_GET(self):
        if not self._check_sig(b""):
            return self._reply(403, b"bad signature")
        b, k, q = self._key()
        if q.get("list-type") == "2":
            keys = sorted(kk for bb, kk in self.objects if bb == b and kk.startswith(q.get("prefix", "")))
            start = int(q.get("continuation-token", "0"))
            chunk = keys[start: start + self.page]
            more = start + self.page < len(keys)
            xml = "<ListBucketResult xmlns='http://s3.amazonaws.com/doc/2006-03-01/'>" + "".join(
                f"<Contents><Key>{kk}</Key><Size>{len(self.objects[(b, kk)])}</Size></Contents>" for kk in chunk) + \
                f"<IsTruncated>{'true' if more else 'false'}</IsTruncated>" + \
                (f"<NextContinuationToken>{start + self.page}</NextContinuationToken>" if more else "") + \
                "</ListBucketResult>"
            return self._reply(200, xml.encode())
        data = self.objects.get((b, k))
        if data is None:
            return self._reply(404, b"NoSuchKey")
        rng = self.headers.get("Range")
        if rng:
            lo, hi = (int(x) for x in rng.split("=")[1].split("-"))
            return self._reply(206, data[lo: hi + 1])
        self._reply(200, data)


@pytest.fixture()
def server():
    _FakeS3.objects = {}
    srv = ThreadingHTTPServer(("127.0.0.1", 0), _FakeS3)
    t = threading.Thread(target=srv.serve_forever, daemon=True)
    t.start()
    yield f"http://127.0.0.1:{srv.server_address[1]}"
    srv.shutdown()


def test_client_roundtrip_and_localize(server, tmp_path):
    c = s3.S3Client(server, access_key=AK, secret_key=SK, region="us-east-1", retries=0)
    files = {"cache/train/shard_ledger.json": b'{"is_finished": true}', "cache/train/input_ids/data/c/0": b"x" * 100,
             "cache/train/input_ids/offsets/c/0": b"y" * 7, "other/z": b"z"}
    for k, v in files.items():
        c.put("bkt", k, v)
    assert c.get("bkt", "cache/train/input_ids/data/c/0", byte_range=(10, 20)) == b"x" * 10
    assert c.head("bkt", "other/z")["size"] == 1
    assert sorted(o["key"] for o in c.list("bkt", "cache/")) == sorted(k for k in files if k.startswith("cache/"))
    with pytest.raises(s3.S3Error, match="404"):
        c.get("bkt", "missing")
    bad = s3.S3Client(server, access_key=AK, secret_key="wrong", region="us-east-1", retries=0)
    with pytest.raises(s3.S3Error, match="403"):
        bad.get("bkt", "other/z")
    out = s3.localize("s3://bkt/cache/train", str(tmp_path / "train"), client=c)
    assert open(os.path.join(out, "shard_ledger.json"), "rb").read() == files["cache/train/shard_ledger.json"]
    assert open(os.path.join(out, "input_ids", "data", "c", "0"), "rb").read() == b"x" * 100
    assert os.path.exists(os.path.join(out, ".localized"))
