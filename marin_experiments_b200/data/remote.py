"""Pretraining mixtures over tokenized caches in object storage (megagpt-speedrun/data.py:100-240).

The reference trains from named components, each a TreeCache split (``shard_ledger.json`` plus
jagged ``input_ids``) under an S3-compatible prefix, sampled with per-component weights; smoke runs
use one component, ``only`` restricts a mixture to the components already mirrored, and the read
path is kept off the network during training by localizing the caches first
(megagpt-speedrun/data.py:244-330 explains why). Here:

* ``RemoteMix(name, components={component: (relative path, weight)}, prefix, smoke)``;
* ``materialize(mix, local_root)`` mirrors each component's ``<prefix>/<rel>/<split>`` to local disk
  once (``utils.s3.localize``), converts its rows to the native loader's shards
  (``data.treecache.to_native_cache``) and returns ``{component: native cache dir}``; finished
  components are reused;
* ``data_config(mix, local_root)`` is the ``DataConfig(source="mixture")`` over them;
* ``mirror_mix(mix, src_prefix, dst_prefix)`` copies the components' caches from one object store to
  another (megagpt-speedrun/mirror_to_cw.py: a cluster-local copy of the caches): components are
  sized first and copied smallest first, so a run can start on the first finished one; objects move
  many at a time and an object already present with the same size is skipped; after each component
  ``MANIFEST.json`` at the destination root lists the finished ones (a later run skips them), and
  ``max_bytes`` stops before a component that would pass the cap.

The component tables below follow the reference's named mixtures (component names and weights);
their prefix defaults to ``MXK_CORPUS_PREFIX`` (the object-store root that holds ``tokenized/``).
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field

from ..config import DataConfig


@dataclass(frozen=True)
class RemoteMix:
    name: str
    components: dict = field(default_factory=dict)  # component -> (relative path under prefix, weight)
    smoke: dict = field(default_factory=dict)  # the one-component smoke variant
    split: str = "train"

    def table(self, smoke: bool = False, only: list[str] | None = None) -> dict:
        t = dict(self.smoke if smoke and self.smoke else self.components)
        if only:
            t = {k: v for k, v in t.items() if k in only}
            if not t:
                raise ValueError(f"{self.name}: none of {only} in {list(self.components)}")
        return t


# Component tables: relative cache roots (their content hashes included, so the same object-store
# caches are read) and sampling weights. The quality-tilted mixture of the reference's object-store
# runs (megagpt-speedrun/data.py:139-150):
NEMOTRON = RemoteMix(
    "nemotron",
    {"nemotron_cc/hq_actual": ("tokenized/nemotron_cc/hq_actual-5af4cc", 2.0),
     "nemotron_cc/medium_high": ("tokenized/nemotron_cc/medium_high-d21701", 1.5),
     "nemotron_cc/medium_low": ("tokenized/nemotron_cc/medium_low-5b94a4", 1.0),
     "nemotron_cc/low_actual": ("tokenized/nemotron_cc/low_actual-cb3f2c", 0.5),
     "nemotron_cc/low_synth": ("tokenized/nemotron_cc/low_synth-3c57b3", 0.4),
     "starcoderdata": ("tokenized/starcoderdata-12f018", 0.5),
     "proofpile_2": ("tokenized/proofpile_2-5ba7ac", 0.2)},
    smoke={"nemotron_cc/hq_actual": ("tokenized/nemotron_cc/hq_actual-5af4cc", 1.0)})
# The size-proportional full mixture (megagpt-speedrun/data.py:52-62):
NEMOTRON_FULL = RemoteMix(
    "nemotron-full",
    {"nemotron_cc/hq_actual": ("tokenized/nemotron_cc/hq_actual-5af4cc", 0.91351),
     "nemotron_cc/hq_synth": ("tokenized/nemotron_cc/hq_synth-3525e2", 2.72),
     "nemotron_cc/medium_high": ("tokenized/nemotron_cc/medium_high-d21701", 0.82471),
     "nemotron_cc/medium": ("tokenized/nemotron_cc/medium-d86506", 3.38),
     "nemotron_cc/medium_low": ("tokenized/nemotron_cc/medium_low-0fdb07", 1.54),
     "nemotron_cc/low_actual": ("tokenized/nemotron_cc/low_actual-cb3f2c", 0.70123),
     "nemotron_cc/low_synth": ("tokenized/nemotron_cc/low_synth-3c57b3", 0.62771),
     "starcoderdata": ("tokenized/starcoderdata-12f018", 0.25),
     "proofpile_2": ("tokenized/proofpile_2-4a35c7", 0.055)})
# Chat SFT cooldown (assistant-only loss masks ride along as ``assistant_masks``;
# megagpt-speedrun/data.py:272-283):
SFT_CHAT = RemoteMix("sft-chat", {"tulu3": ("tokenized/megagpt_sft_v2/tulu3", 0.5),
                                  "smoltalk": ("tokenized/megagpt_sft_v2/smoltalk", 0.4),
                                  "ot_agent": ("tokenized/megagpt_sft_v2/ot_agent", 0.1)})
MIXES = {m.name: m for m in (NEMOTRON, NEMOTRON_FULL, SFT_CHAT)}


def _prefix(prefix: str | None) -> str:
    p = prefix or os.environ.get("MXK_CORPUS_PREFIX")
    if not p:
        raise ValueError("no object-store prefix: pass prefix= or set MXK_CORPUS_PREFIX (s3://bucket/root)")
    return p.rstrip("/")


def materialize(mix: RemoteMix, local_root: str, *, prefix: str | None = None, client=None, smoke: bool = False,
                only: list[str] | None = None, eos_id: int | None = None, vocab_size: int | None = None) -> dict:
    """``{component: native cache dir}`` for the mixture's components, fetched and converted once."""
    from ..utils.s3 import localize
    from .tokenize import is_complete
    from .treecache import to_native_cache

    root = _prefix(prefix)
    out = {}
    for comp, (rel, _) in mix.table(smoke, only).items():
        native = os.path.join(local_root, "native", comp)
        if not is_complete(native):
            tc_dir = localize(f"{root}/{rel}/{mix.split}", os.path.join(local_root, "treecache", comp, mix.split),
                              client=client)
            to_native_cache(tc_dir, native, eos_id=eos_id, vocab_size=vocab_size)
        out[comp] = native
    return out


def data_config(mix: RemoteMix, local_root: str, *, seed: int = 0, smoke: bool = False, only: list[str] | None = None,
                **kw) -> DataConfig:
    caches = materialize(mix, local_root, smoke=smoke, only=only, **kw)
    table = mix.table(smoke, only)
    return DataConfig(source="mixture", components=tuple((c, caches[c], float(table[c][1])) for c in caches),
                      seed=seed)


def mirror_mix(mix: RemoteMix, src_prefix: str, dst_prefix: str, src_client=None, dst_client=None, *,
               only: list[str] | None = None, max_bytes: int = 0, workers: int = 32) -> dict:
    """Copy ``mix``'s component caches (their ``split``) between object stores; returns the manifest."""
    import json

    from ..utils import s3

    src = src_client or s3.S3Client()
    dst = dst_client or s3.S3Client()
    sroot, droot = src_prefix.rstrip("/"), dst_prefix.rstrip("/")
    db, dkey = s3.split_url(droot)
    man_key = (dkey + "/" if dkey else "") + "MANIFEST.json"
    try:
        manifest = json.loads(dst.get(db, man_key))
    except s3.S3Error as e:
        if e.status != 404:
            raise
        manifest = {"mix": mix.name, "split": mix.split, "components": {}}
    sizes = {}
    for comp, (rel, _w) in mix.table(only=only).items():
        if comp in manifest["components"]:
            continue
        b, k = s3.split_url(f"{sroot}/{rel}/{mix.split}")
        sizes[comp] = sum(o["size"] for o in src.list(b, k.rstrip("/") + "/"))
    total = sum(c["bytes"] for c in manifest["components"].values())
    for comp in sorted(sizes, key=lambda c: (sizes[c], c)):
        if max_bytes and total + sizes[comp] > max_bytes:
            break
        rel = mix.components.get(comp, mix.smoke.get(comp))[0]
        st = s3.mirror_prefix(src, f"{sroot}/{rel}/{mix.split}", dst, f"{droot}/{rel}/{mix.split}", workers=workers)
        manifest["components"][comp] = {"rel": rel, "bytes": sizes[comp], "objects": st["objects"]}
        total += sizes[comp]
        dst.put(db, man_key, json.dumps(manifest, indent=1).encode())
    return manifest
