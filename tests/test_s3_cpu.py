"""SigV4 signing against the AWS documentation's example, and the S3 client (get / range / put /
head / paginated list / localize) against a local fake S3 server that checks every signature."""

import datetime
import os

import pytest

from marin_experiments_b200.utils import s3
from s3_fake import AK, SK, start_server


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


@pytest.fixture()
def server():
    url, srv = start_server()
    yield url
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
