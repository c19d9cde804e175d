"""Object-store addressing (megagpt-speedrun/cw_patch.py:1-260): S3 URLs under path-style or
virtual-hosted addressing.

Path style puts the bucket in the path (``{endpoint}/{bucket}/{key}``); some S3-compatible stores
accept only virtual-hosted addressing (``{scheme}://{bucket}.{host}/{key}``). ``s3_spec(url)``
returns the addressing to use: virtual-hosted when ``S3_VIRTUAL_HOSTED`` (or the reference's
``LEVANTER_S3_VIRTUAL_HOSTED``) is truthy and an ``AWS_ENDPOINT_URL`` is set, else path style with
the configured endpoint. ``storage_options`` turns it into keyword arguments for an fsspec-style
S3 filesystem. There is no network here; these helpers only compute addresses.
"""

from __future__ import annotations

import os
import urllib.parse


def _truthy(name: str) -> bool:
    return os.environ.get(name, "").strip().lower() in ("1", "true", "yes")


def virtual_hosted_enabled() -> bool:
    return _truthy("S3_VIRTUAL_HOSTED") or _truthy("LEVANTER_S3_VIRTUAL_HOSTED")


def s3_spec(url: str, env: dict | None = None) -> dict:
    """``{"bucket", "key", "endpoint", "addressing", "region"}`` for an ``s3://bucket/key`` URL."""
    env = os.environ if env is None else env
    p = urllib.parse.urlparse(url)
    if p.scheme != "s3":
        raise ValueError(f"not an s3 URL: {url!r}")
    bucket, key = p.netloc, p.path.lstrip("/")
    endpoint = env.get("AWS_ENDPOINT_URL")
    region = env.get("AWS_DEFAULT_REGION") or env.get("AWS_REGION")
    vh = (env.get("S3_VIRTUAL_HOSTED", "") or env.get("LEVANTER_S3_VIRTUAL_HOSTED", "")).strip().lower() in (
        "1", "true", "yes")
    if endpoint and vh:
        ep = urllib.parse.urlparse(endpoint if "://" in endpoint else "https://" + endpoint)
        return {"bucket": "", "key": key, "endpoint": f"{ep.scheme}://{bucket}.{ep.netloc}",
                "addressing": "virtual", "region": region, "object_url": f"{ep.scheme}://{bucket}.{ep.netloc}/{key}"}
    spec = {"bucket": bucket, "key": key, "endpoint": endpoint, "addressing": "path", "region": region}
    spec["object_url"] = f"{endpoint.rstrip('/')}/{bucket}/{key}" if endpoint else f"s3://{bucket}/{key}"
    return spec


def storage_options(url: str, env: dict | None = None) -> dict:
    s = s3_spec(url, env)
    opts: dict = {}
    client: dict = {}
    if s["endpoint"]:
        client["endpoint_url"] = s["endpoint"]
    if s["region"]:
        client["region_name"] = s["region"]
    if client:
        opts["client_kwargs"] = client
    if s["addressing"] == "virtual":
        opts["config_kwargs"] = {"s3": {"addressing_style": "virtual"}}
    return opts
