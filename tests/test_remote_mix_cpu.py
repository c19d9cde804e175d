"""Object-store mixtures: TreeCache splits under an S3 prefix (one with assistant masks) are mirrored
through the signed client, converted to native shards once, and served by the block mixture."""

import os

import numpy as np
import pytest

from marin_experiments_b200.data import remote
from marin_experiments_b200.data.treecache import write_tree_cache
from marin_experiments_b200.utils import s3
from s3_fake import AK, SK, start_server


@pytest.fixture()
def client():
    url, srv = start_server()
    yield s3.S3Client(url, access_key=AK, secret_key=SK, region="us-east-1", retries=0)
    srv.shutdown()


def _upload(c, local_dir, bucket, key_prefix):
    for dirpath, _, files in os.walk(local_dir):
        for f in files:
            p = os.path.join(dirpath, f)
            rel = os.path.relpath(p, local_dir).replace(os.sep, "/")
            with open(p, "rb") as fh:
                c.put(bucket, f"{key_prefix}/{rel}", fh.read())


def test_remote_mix_materializes_and_serves(client, tmp_path):
    rng = np.random.default_rng(0)
    web = [{"input_ids": rng.integers(1, 500, size=rng.integers(20, 90)).astype(np.int32)} for _ in range(40)]
    chat = []
    for _ in range(30):
        n = int(rng.integers(16, 64))
        chat.append({"input_ids": rng.integers(1, 500, size=n).astype(np.int32),
                     "assistant_masks": (np.arange(n) >= n // 2).astype(np.int8)})
    write_tree_cache(str(tmp_path / "src_web"), web)
    write_tree_cache(str(tmp_path / "src_chat"), chat, fields=("input_ids", "assistant_masks"))
    _upload(client, str(tmp_path / "src_web"), "bkt", "root/tokenized/web-abc/train")
    _upload(client, str(tmp_path / "src_chat"), "bkt", "root/tokenized/chat-def/train")

    mix = remote.RemoteMix("t", {"web": ("tokenized/web-abc", 3.0), "chat": ("tokenized/chat-def", 1.0)},
                           smoke={"web": ("tokenized/web-abc", 1.0)})
    local = str(tmp_path / "local")
    cfg = remote.data_config(mix, local, prefix="s3://bkt/root", client=client, seed=3)
    assert cfg.source == "mixture" and cfg.seed == 3
    assert [(n, w) for n, _, w in cfg.components] == [("web", 3.0), ("chat", 1.0)]
    import json

    meta = json.load(open(os.path.join(local, "native", "chat", "meta.json")))
    assert meta["num_docs"] == 30 and meta["format"] == "chat"
    assert meta["num_tokens"] == sum(len(r["input_ids"]) for r in chat)
    web_tokens = np.fromfile(os.path.join(local, "native", "web", "tokens-00000.bin"), dtype="<u4")
    assert np.array_equal(web_tokens, np.concatenate([r["input_ids"] for r in web]))

    # finished components are neither fetched nor converted again (a dead client proves it)
    class Dead:
        def list(self, *a, **k):
            raise AssertionError("fetched again")

    again = remote.data_config(mix, local, prefix="s3://bkt/root", client=Dead())
    assert again.components == cfg.components
    assert [n for n, _, _ in remote.data_config(mix, local, prefix="s3://bkt/root", client=Dead(),
                                                only=["chat"]).components] == ["chat"]
    assert [c for c, _, _ in remote.data_config(mix, local, prefix="s3://bkt/root", client=Dead(),
                                                smoke=True).components] == ["web"]
    with pytest.raises(ValueError, match="none of"):
        mix.table(only=["nope"])

    rt = pytest.importorskip("marin_experiments_b200.runtime")
    try:
        rt.rt()
    except Exception as e:  # the native runtime is built by the package build step
        pytest.skip(f"native runtime unavailable: {e}")
    from marin_experiments_b200.data.loader import build_dataset

    ds = build_dataset(cfg, 32, 512)
    assert ds.seq_len() == 32


def test_named_mixtures_and_prefix():
    assert set(remote.MIXES) == {"nemotron", "nemotron-full", "sft-chat"}
    assert list(remote.NEMOTRON.table(smoke=True)) == ["nemotron_cc/hq_actual"]
    assert abs(sum(w for _, w in remote.SFT_CHAT.components.values()) - 1.0) < 1e-9
    old = os.environ.pop("MXK_CORPUS_PREFIX", None)
    try:
        with pytest.raises(ValueError, match="prefix"):
            remote.materialize(remote.NEMOTRON, "/nonexistent")
    finally:
        if old is not None:
            os.environ["MXK_CORPUS_PREFIX"] = old


def test_mirror_between_stores(client, tmp_path):
    """Components copied smallest first, resumable by size, with a manifest and a byte cap."""
    sizes = {"a": 5, "b": 2, "c": 9}
    mix = remote.RemoteMix("m", {k: (f"tokenized/{k}-h", 1.0) for k in sizes})
    for k, n in sizes.items():
        for i in range(n):
            client.put("src", f"root/tokenized/{k}-h/train/chunk-{i}.bin", bytes([i]) * (100 + i))
        client.put("src", f"root/tokenized/{k}-h/validation/x.bin", b"not copied")
    man = remote.mirror_mix(mix, "s3://src/root", "s3://dst/mirror", client, client, max_bytes=2 * 101 * 5 + 600)
    assert list(man["components"]) == ["b", "a"]  # smallest first; c would pass the cap
    got = {o["key"] for o in client.list("dst", "mirror/")}
    assert "mirror/tokenized/b-h/train/chunk-1.bin" in got and not any("validation" in k for k in got)
    assert client.get("dst", "mirror/tokenized/a-h/train/chunk-3.bin") == bytes([3]) * 103
    # resume: finished components are skipped, the rest is copied; a damaged object is copied again
    client.put("dst", "mirror/tokenized/c-h/train/chunk-0.bin", b"short")
    st = s3.mirror_prefix(client, "s3://src/root/tokenized/c-h/train", client, "s3://dst/mirror/tokenized/c-h/train",
                          workers=4)
    assert st == {"objects": 9, "copied": 9, "skipped": 0, "bytes": sum(100 + i for i in range(9))}
    again = s3.mirror_prefix(client, "s3://src/root/tokenized/c-h/train", client,
                             "s3://dst/mirror/tokenized/c-h/train")
    assert again["copied"] == 0 and again["skipped"] == 9
    man = remote.mirror_mix(mix, "s3://src/root", "s3://dst/mirror", client, client)
    assert list(man["components"]) == ["b", "a", "c"] and man["components"]["c"]["objects"] == 9
    import json

    assert json.loads(client.get("dst", "mirror/MANIFEST.json")) == man


def test_remote_source_resolves_when_the_dataset_is_built(client, tmp_path, monkeypatch):
    """``DataConfig(source="remote", mix=...)`` names a mixture; the mirror happens in build_dataset."""
    rng = np.random.default_rng(1)
    rows = [{"input_ids": rng.integers(1, 500, size=rng.integers(40, 90)).astype(np.int32)} for _ in range(30)]
    write_tree_cache(str(tmp_path / "src"), rows)
    _upload(client, str(tmp_path / "src"), "bkt", "root/tokenized/tiny-1/train")
    monkeypatch.setitem(remote.MIXES, "tiny", remote.RemoteMix("tiny", {"t": ("tokenized/tiny-1", 1.0)}))
    for k, v in {"MXK_CORPUS_PREFIX": "s3://bkt/root", "AWS_ENDPOINT_URL": client.endpoint, "AWS_ACCESS_KEY_ID": AK,
                 "AWS_SECRET_ACCESS_KEY": SK, "AWS_DEFAULT_REGION": "us-east-1"}.items():
        monkeypatch.setenv(k, v)
    rt = pytest.importorskip("marin_experiments_b200.runtime")
    try:
        rt.rt()
    except Exception as e:
        pytest.skip(f"native runtime unavailable: {e}")
    from marin_experiments_b200.config import DataConfig
    from marin_experiments_b200.data.loader import build_dataset

    ds = build_dataset(DataConfig(source="remote", mix="tiny", cache_dir=str(tmp_path / "local")), 32, 512)
    assert ds.seq_len() == 32 and os.path.exists(tmp_path / "local" / "native" / "t" / "meta.json")
    with pytest.raises(ValueError, match="unknown remote mixture"):
        build_dataset(DataConfig(source="remote", mix="nope"), 32, 512)
