"""S3-compatible object storage: AWS Signature Version 4 signing and a small client.

The reference reads tokenized caches and writes checkpoints on S3-compatible stores (R2,
CoreWeave object storage) through tensorstore and s3fs (megagpt-speedrun/cw_patch.py:1-260,
megagpt-speedrun/data.py:296-330). Its post-mortem of a silent multi-hour data-loader stall -- an
S3 GET with no read timeout -- is why every request here has a connect / read timeout and bounded
retries, and why ``localize`` mirrors a prefix to local disk once so training never reads remote
objects in its hot loop.

* ``sign``: SigV4 headers for one request (canonical request -> string to sign -> HMAC-SHA256
  signing-key chain ``AWS4<secret> / date / region / service / aws4_request``), from the AWS
  specification;
* ``S3Client``: ``get`` (optionally a byte range), ``put``, ``head``, ``list`` (ListObjectsV2 with
  continuation), path-style or virtual-hosted addressing (``utils.objstore.s3_spec``);
* ``localize(url, local_dir)``: download every object under an ``s3://bucket/prefix`` into a local
  directory (a marker file makes it idempotent), e.g. a TreeCache split for ``data.treecache``.

Credentials come from ``AWS_ACCESS_KEY_ID`` / ``AWS_SECRET_ACCESS_KEY`` (and ``AWS_SESSION_TOKEN``),
the endpoint from ``AWS_ENDPOINT_URL``, the region from ``AWS_DEFAULT_REGION`` (``auto`` for R2).
"""

from __future__ import annotations

import datetime
import hashlib
import hmac
import os
import time
import urllib.parse
import xml.etree.ElementTree as ET

EMPTY_SHA256 = hashlib.sha256(b"").hexdigest()


def _hmac(key: bytes, msg: str) -> bytes:
    return hmac.new(key, msg.encode(), hashlib.sha256).digest()


def signing_key(secret: str, date: str, region: str, service: str) -> bytes:
    k = _hmac(("AWS4" + secret).encode(), date)
    k = _hmac(k, region)
    k = _hmac(k, service)
    return _hmac(k, "aws4_request")


def _uri_encode(s: str, keep_slash: bool) -> str:
    return urllib.parse.quote(s, safe="/~" if keep_slash else "~")


def canonical_request(method: str, path: str, query: dict[str, str], headers: dict[str, str],
                      payload_hash: str) -> tuple[str, str]:
    """(canonical request, signed header list)."""
    q = "&".join(f"{_uri_encode(k, False)}={_uri_encode(v, False)}" for k, v in sorted(query.items()))
    h = {k.lower().strip(): " ".join(str(v).strip().split()) for k, v in headers.items()}
    names = sorted(h)
    ch = "".join(f"{n}:{h[n]}\n" for n in names)
    signed = ";".join(names)
    return "\n".join([method, _uri_encode(path, True) or "/", q, ch, signed, payload_hash]), signed


def sign(method: str, url: str, *, access_key: str, secret_key: str, region: str, service: str = "s3",
         payload: bytes = b"", headers: dict | None = None, when: datetime.datetime | None = None,
         session_token: str | None = None, unsigned_payload: bool = False) -> dict[str, str]:
    """Headers (``Authorization``, ``x-amz-date``, ``x-amz-content-sha256``, ``host``, and the
    caller's) that authenticate ``method url`` with SigV4."""
    u = urllib.parse.urlparse(url)
    when = when or datetime.datetime.now(datetime.timezone.utc)
    amz_date = when.strftime("%Y%m%dT%H%M%SZ")
    date = amz_date[:8]
    payload_hash = "UNSIGNED-PAYLOAD" if unsigned_payload else hashlib.sha256(payload).hexdigest()
    hdrs = dict(headers or {})
    hdrs["host"] = u.netloc
    hdrs["x-amz-date"] = amz_date
    if service == "s3":
        hdrs["x-amz-content-sha256"] = payload_hash
    if session_token:
        hdrs["x-amz-security-token"] = session_token
    query = dict(urllib.parse.parse_qsl(u.query, keep_blank_values=True))
    creq, signed = canonical_request(method, urllib.parse.unquote(u.path) or "/", query, hdrs, payload_hash)
    scope = f"{date}/{region}/{service}/aws4_request"
    sts = "\n".join(["AWS4-HMAC-SHA256", amz_date, scope, hashlib.sha256(creq.encode()).hexdigest()])
    sig = hmac.new(signing_key(secret_key, date, region, service), sts.encode(), hashlib.sha256).hexdigest()
    hdrs["Authorization"] = f"AWS4-HMAC-SHA256 Credential={access_key}/{scope}, SignedHeaders={signed}, Signature={sig}"
    return hdrs


class S3Error(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"S3 {status}: {msg}")
        self.status = status


class S3Client:
    def __init__(self, endpoint: str | None = None, *, access_key: str | None = None, secret_key: str | None = None,
                 region: str | None = None, virtual_hosted: bool = False, session_token: str | None = None,
                 timeout: tuple[float, float] = (10.0, 60.0), retries: int = 3):
        env = os.environ
        self.endpoint = (endpoint or env.get("AWS_ENDPOINT_URL") or "https://s3.amazonaws.com").rstrip("/")
        if "://" not in self.endpoint:
            self.endpoint = "https://" + self.endpoint
        self.access_key = access_key or env.get("AWS_ACCESS_KEY_ID", "")
        self.secret_key = secret_key or env.get("AWS_SECRET_ACCESS_KEY", "")
        self.session_token = session_token or env.get("AWS_SESSION_TOKEN")
        self.region = region or env.get("AWS_DEFAULT_REGION") or env.get("AWS_REGION") or "us-east-1"
        self.virtual_hosted = virtual_hosted
        self.timeout, self.retries = timeout, retries

    def url(self, bucket: str, key: str = "", query: dict | None = None) -> str:
        ep = urllib.parse.urlparse(self.endpoint)
        k = _uri_encode(key, True)
        base = f"{ep.scheme}://{bucket}.{ep.netloc}/{k}" if self.virtual_hosted else f"{self.endpoint}/{bucket}/{k}"
        if query:
            base += "?" + urllib.parse.urlencode(sorted(query.items()), quote_via=urllib.parse.quote)
        return base

    def _request(self, method: str, url: str, data: bytes = b"", headers: dict | None = None):
        import requests

        last = None
        for attempt in range(self.retries + 1):
            hdrs = sign(method, url, access_key=self.access_key, secret_key=self.secret_key, region=self.region,
                        payload=data, headers=headers, session_token=self.session_token)
            try:
                r = requests.request(method, url, data=data or None, headers=hdrs, timeout=self.timeout)
            except requests.RequestException as e:  # connection / timeout: retried
                last = e
            else:
                if r.status_code < 500 and r.status_code != 429:
                    if r.status_code >= 400:
                        raise S3Error(r.status_code, r.text[:300])
                    return r
                last = S3Error(r.status_code, r.text[:300])
            time.sleep(min(8.0, 0.25 * 2 ** attempt))
        raise last

    def get(self, bucket: str, key: str, byte_range: tuple[int, int] | None = None) -> bytes:
        """The object, or bytes ``[start, end)`` of it."""
        h = {"Range": f"bytes={byte_range[0]}-{byte_range[1] - 1}"} if byte_range else None
        return self._request("GET", self.url(bucket, key), headers=h).content

    def put(self, bucket: str, key: str, data: bytes) -> None:
        self._request("PUT", self.url(bucket, key), data=data)

    def head(self, bucket: str, key: str) -> dict:
        r = self._request("HEAD", self.url(bucket, key))
        return {"size": int(r.headers.get("Content-Length", 0)), "etag": r.headers.get("ETag")}

    def list(self, bucket: str, prefix: str = "") -> list[dict]:
        """Every object under ``prefix``: ``[{"key", "size"}]`` (ListObjectsV2 pages followed)."""
        out, token = [], None
        while True:
            q = {"list-type": "2", "prefix": prefix}
            if token:
                q["continuation-token"] = token
            root = ET.fromstring(self._request("GET", self.url(bucket, "", q)).content)
            ns = root.tag[: root.tag.index("}") + 1] if root.tag.startswith("{") else ""
            for c in root.findall(f"{ns}Contents"):
                out.append({"key": c.findtext(f"{ns}Key"), "size": int(c.findtext(f"{ns}Size") or 0)})
            if (root.findtext(f"{ns}IsTruncated") or "false").lower() != "true":
                return out
            token = root.findtext(f"{ns}NextContinuationToken")


def split_url(url: str) -> tuple[str, str]:
    p = urllib.parse.urlparse(url)
    if p.scheme != "s3":
        raise ValueError(f"not an s3 URL: {url!r}")
    return p.netloc, p.path.lstrip("/")


def localize(url: str, local_dir: str, client: S3Client | None = None, marker: str = ".localized") -> str:
    """Mirror every object under ``s3://bucket/prefix`` into ``local_dir`` (relative layout kept);
    a finished mirror leaves ``marker`` and is not fetched again."""
    if os.path.exists(os.path.join(local_dir, marker)):
        return local_dir
    client = client or S3Client()
    bucket, prefix = split_url(url)
    prefix = prefix.rstrip("/") + "/" if prefix else ""
    os.makedirs(local_dir, exist_ok=True)
    for obj in client.list(bucket, prefix):
        rel = obj["key"][len(prefix):]
        if not rel or rel.endswith("/"):
            continue
        dst = os.path.join(local_dir, *rel.split("/"))
        os.makedirs(os.path.dirname(dst), exist_ok=True)
        tmp = dst + ".part"
        with open(tmp, "wb") as f:
            f.write(client.get(bucket, obj["key"]))
        os.replace(tmp, dst)
    with open(os.path.join(local_dir, marker), "w") as f:
        f.write("ok\n")
    return local_dir


def mirror_prefix(src: S3Client, src_url: str, dst: S3Client, dst_url: str, *, workers: int = 32) -> dict:
    """Copy every object under ``src_url`` to the same relative key under ``dst_url`` (two stores,
    or two places in one), ``workers`` objects at a time: the caches are many objects of about a
    megabyte, so the copy is latency-bound and wants many requests in flight. An object already at
    the destination with the same size is skipped, so an interrupted mirror resumes where it
    stopped. Returns ``{"objects", "copied", "skipped", "bytes"}`` (bytes copied)."""
    from concurrent.futures import ThreadPoolExecutor

    sb, sp = split_url(src_url)
    db, dp = split_url(dst_url)
    sp = sp.rstrip("/") + "/" if sp else ""
    dp = dp.rstrip("/") + "/" if dp else ""
    have = {o["key"][len(dp):]: o["size"] for o in dst.list(db, dp)}
    todo, skipped = [], 0
    for o in src.list(sb, sp):
        rel = o["key"][len(sp):]
        if not rel or rel.endswith("/"):
            continue
        if have.get(rel) == o["size"]:
            skipped += 1
        else:
            todo.append((o["key"], rel, o["size"]))

    def copy(item):
        key, rel, size = item
        data = src.get(sb, key)
        if len(data) != size:
            raise S3Error(0, f"{key}: read {len(data)} bytes, listed {size}")
        dst.put(db, dp + rel, data)
        return size

    with ThreadPoolExecutor(max_workers=max(1, workers)) as ex:
        copied = sum(ex.map(copy, todo))
    return {"objects": len(todo) + skipped, "copied": len(todo), "skipped": skipped, "bytes": copied}
