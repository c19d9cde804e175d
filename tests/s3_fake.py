"""A local fake S3 server for CPU tests: path-style GET (with Range), PUT, HEAD and paginated
ListObjectsV2; every request's SigV4 signature is recomputed and checked."""

import datetime
import hashlib
import hmac
import threading
import urllib.parse
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

from marin_experiments_b200.utils import s3

AK, SK = "AKIDEXAMPLE", "wJalrXUtnFEMI/K7MDENG+bPxRfiCYEXAMPLEKEY"


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


def start_server():
    _FakeS3.objects = {}
    srv = ThreadingHTTPServer(("127.0.0.1", 0), _FakeS3)
    t = threading.Thread(target=srv.serve_forever, daemon=True)
    t.start()
    return f"http://127.0.0.1:{srv.server_address[1]}", srv
