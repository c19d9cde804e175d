"""Reference-layout (Levanter tree) checkpoints and the zarr array IO under them."""

import json
import os

import numpy as np
import pytest
import torch

from marin_experiments_b200.utils import zarr_io

MOE = dict(vocab_size=512, hidden_dim=128, intermediate_dim=128, shared_expert_intermediate_dim=256, num_experts=4,
           num_experts_per_token=2, num_layers=2, num_heads=2, num_kv_heads=1, head_dim=64, max_seq_len=64,
           sliding_window=64, capacity_factor=2.0)


@pytest.mark.parametrize("zstd", [False, True])
@pytest.mark.parametrize("shape,chunks,dtype", [((10, 7), (4, 7), np.float32), ((5,), None, np.int64),
                                                ((), None, np.int32), ((3, 5, 2), (2, 2, 2), np.float16)])
def test_zarr_v3_roundtrip(tmp_path, shape, chunks, dtype, zstd):
    a = (np.arange(int(np.prod(shape))).reshape(shape) * 3 - 7).astype(dtype)
    p = str(tmp_path / "arr")
    zarr_io.write_array(p, a, chunks=chunks, zstd=zstd)
    meta = json.load(open(os.path.join(p, "zarr.json")))
    assert meta["zarr_format"] == 3 and meta["node_type"] == "array" and meta["shape"] == list(shape)
    b = zarr_io.read_array(p)
    assert b.dtype == a.dtype and b.shape == a.shape and (b == a).all()


def test_zarr_v2_read(tmp_path):
    """A zarr v2 array as the tensorstore ``zarr`` driver lays it out: ``.zarray`` + ``<i>.<j>`` chunks."""
    import pyarrow as pa

    a = np.arange(30, dtype="<f4").reshape(5, 6)
    p = tmp_path / "v2"
    p.mkdir()
    meta = {"zarr_format": 2, "shape": [5, 6], "chunks": [2, 4], "dtype": "<f4", "compressor": {"id": "zstd"},
            "fill_value": 0, "order": "C", "filters": None}
    (p / ".zarray").write_text(json.dumps(meta))
    codec = pa.Codec("zstd")
    for i in range(3):
        for j in range(2):
            blk = np.zeros((2, 4), dtype="<f4")
            sub = a[2 * i: 2 * i + 2, 4 * j: 4 * j + 4]
            blk[: sub.shape[0], : sub.shape[1]] = sub
            (p / f"{i}.{j}").write_bytes(codec.compress(blk.tobytes(), asbytes=True))
    assert (zarr_io.read_array(str(p)) == a).all()


def _trainer(seed=0, ema=None):
    from marin_experiments_b200.config import GrugModelConfig, GrugRunConfig, GrugTrainerConfig, TrainerConfig
    from marin_experiments_b200.optim import GrugMoeAdamHConfig
    from marin_experiments_b200.train.trainer import Trainer

    run = GrugRunConfig(model=GrugModelConfig(**MOE), optimizer=GrugMoeAdamHConfig(warmup=0.0),
                        trainer=GrugTrainerConfig(trainer=TrainerConfig(num_train_steps=10, seed=seed), ema_beta=ema))
    return Trainer(run, device="cpu")


def test_reference_layout_export_and_import(tmp_path):
    from marin_experiments_b200.train.checkpoint import scan_checkpoint_root
    from marin_experiments_b200.train.levanter_ckpt import load_levanter, save_levanter

    tr = _trainer(ema=0.9)
    g = torch.Generator().manual_seed(0)
    for _ in range(2):
        tr.train_step({"tokens": torch.randint(0, 512, (2, 64), generator=g)})
    path = str(tmp_path / "step-2")
    save_levanter(tr, path)
    # the reference's names and [in, out] layouts (megagpt-speedrun/model.py:234-720)
    d, h, hd, e, i, si = 128, 2, 64, 4, 128, 256
    expect = {"params/blocks/0/attn/w_q": (d, h * hd), "params/blocks/0/attn/w_k": (d, hd),
              "params/blocks/0/attn/w_o": (h * hd, d), "params/blocks/0/attn/attn_gate": (d, h),
              "params/blocks/1/mlp/router": (d, e), "params/blocks/1/mlp/expert_mlp/w_gate_up": (e, d, 2 * i),
              "params/blocks/1/mlp/expert_mlp/w_down": (e, i, d), "params/blocks/0/shared/w_gate": (d, si),
              "params/blocks/0/shared/w_down": (si, d), "params/blocks/0/rms_attn/weight": (d,),
              "params/blocks/0/attn_gated_norm/w_down": (d, 128), "params/token_embed": (512, d),
              "params/output_proj": (d, 512), "params/final_gated_norm/w_up": (128, d),
              "ema_params/blocks/1/mlp/router_threshold": (), "pending_qb_betas": (2, e), "step": ()}
    for p, shp in expect.items():
        assert tuple(zarr_io.read_meta(os.path.join(path, p))["shape"]) == shp, p
    assert int(zarr_io.read_array(os.path.join(path, "step"))) == 2
    assert [s for s, _, _ in scan_checkpoint_root(str(tmp_path))] == [2]
    # gate columns first in the routed experts' fused weight: column j < I is expert gate unit j
    from marin_experiments_b200.ops.layout import blocked_rows_to_gate_up

    wgu = zarr_io.read_array(os.path.join(path, "params/blocks/1/mlp/expert_mlp/w_gate_up"))
    ours = tr.store.master_view([x for x in tr.store.infos if x.name == "blocks.1.mlp.w_gate_up"][0])
    gate, _ = blocked_rows_to_gate_up(ours)
    assert np.allclose(wgu[:, :, :i], gate.transpose(1, 2).numpy())
    fresh = _trainer(seed=5, ema=0.9)
    assert not torch.equal(fresh.store.master, tr.store.master)
    assert load_levanter(fresh, path) == 2 and fresh.step == 2
    assert torch.equal(fresh.store.master, tr.store.master)
    assert torch.equal(fresh.ema, tr.ema)
    assert torch.equal(fresh.pending_qb, tr.pending_qb)


def test_import_reports_missing_leaf(tmp_path):
    from marin_experiments_b200.train.levanter_ckpt import load_levanter, save_levanter

    tr = _trainer()
    path = str(tmp_path / "step-0")
    save_levanter(tr, path, zstd=False)
    import shutil

    shutil.rmtree(os.path.join(path, "params", "blocks", "1", "attn", "w_v"))
    with pytest.raises(KeyError, match="blocks/1/attn/w_v"):
        load_levanter(_trainer(seed=1), path)


def test_tree_cache_roundtrip_and_native_conversion(tmp_path):
    """A TreeCache split (ledger + jagged input_ids / assistant_masks) reads back row by row and
    converts to native loader shards that serve the same tokens."""
    from marin_experiments_b200.data.loader import open_cache
    from marin_experiments_b200.data.treecache import TreeCache, to_native_cache, write_tree_cache

    g = np.random.default_rng(0)
    rows = []
    for i in range(40):
        n = int(g.integers(5, 60))
        ids = g.integers(0, 1000, n).astype(np.int32)
        ids[-1] = 999  # end of document
        rows.append({"input_ids": ids, "assistant_masks": (g.random(n) > 0.5).astype(np.int32)})
    root = str(tmp_path / "cache" / "train")
    ledger = write_tree_cache(root, rows, fields=("input_ids", "assistant_masks"))
    assert ledger["is_finished"] and ledger["total_num_rows"] == 40
    tc = TreeCache(root)
    assert len(tc) == 40 and set(tc.fields) == {"input_ids", "assistant_masks"}
    for i in (0, 17, 39):
        assert (tc[i]["input_ids"] == rows[i]["input_ids"]).all()
        assert (tc[i]["assistant_masks"] == rows[i]["assistant_masks"]).all()
    native = str(tmp_path / "native")
    meta = to_native_cache(root, native, eos_id=999, vocab_size=1000, shard_tokens=300)
    assert len(meta["shards"]) > 1 and meta["num_docs"] == 40 and all("mask" in s for s in meta["shards"])
    flat = np.concatenate([np.fromfile(os.path.join(native, s["tokens"]), dtype="<u4") for s in meta["shards"]])
    assert (flat == np.concatenate([r["input_ids"] for r in rows])).all()
    ds = open_cache(native, 16, seed=0, shuffle=False)
    assert ds.size() > 0
