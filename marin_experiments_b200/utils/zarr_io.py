"""Zarr arrays on a local filesystem: the on-disk array format of Levanter checkpoints and token
caches (written there through tensorstore; megagpt-speedrun/checkpointing.py:28-158 restores them,
megagpt-speedrun/probe_cwobject.py:40 lists the ``zarr.json`` files of a cache).

Neither zarr nor tensorstore is a dependency here, so this module implements the parts of the two
published formats that those files use:

* zarr v3 -- an array directory holds ``zarr.json`` (``zarr_format: 3``, ``node_type: "array"``,
  ``shape``, ``data_type``, a ``regular`` chunk grid, ``default`` chunk-key encoding, ``codecs``)
  and one file per chunk at ``c/<i>/<j>/...``; codecs ``bytes`` (little endian) optionally
  followed by ``zstd`` (and, on read, a trailing ``crc32c`` checksum, not verified); missing chunks
  read as the fill value;
* zarr v2 (read only) -- ``.zarray`` (``zarr_format: 2``, ``dtype`` as a NumPy type string,
  ``compressor`` null or ``{"id": "zstd"}``, ``dimension_separator`` "." or "/"), chunk files
  ``<i>.<j>`` -- the layout of older tensorstore ``zarr`` driver checkpoints.

Chunks are read and written whole; edge chunks are stored full size (zarr's rule) and clipped on
read. zstd frames are produced and decoded by pyarrow's codec.
"""

from __future__ import annotations

import itertools
import json
import os

import numpy as np

_V3_TYPES = {
    "bool": np.bool_, "int8": np.int8, "int16": np.int16, "int32": np.int32, "int64": np.int64,
    "uint8": np.uint8, "uint16": np.uint16, "uint32": np.uint32, "uint64": np.uint64,
    "float16": np.float16, "float32": np.float32, "float64": np.float64,
}


def _v3_name(dtype) -> str:
    dt = np.dtype(dtype)
    if dt.name == "bfloat16" or str(dt) == "bfloat16":
        return "bfloat16"
    for k, v in _V3_TYPES.items():
        if np.dtype(v) == dt:
            return k
    raise TypeError(f"no zarr v3 data type for {dt}")


def _zstd():
    import pyarrow as pa

    return pa.Codec("zstd")


def _chunk_indices(shape, chunks):
    return itertools.product(*[range(max(1, -(-s // c))) for s, c in zip(shape, chunks)])


def write_array(path: str, arr: np.ndarray, *, chunks: tuple[int, ...] | None = None, zstd: bool = True,
                attributes: dict | None = None, raw_dtype: str | None = None) -> None:
    """Write ``arr`` as a zarr v3 array directory at ``path``. ``raw_dtype`` names the stored data
    type when ``arr`` holds its bytes under another NumPy type (``"bfloat16"`` from a uint16 view)."""
    arr = np.asarray(arr, order="C")  # (keeps 0-d arrays 0-d, unlike ascontiguousarray)
    shape = tuple(int(s) for s in arr.shape)
    if chunks is None:
        chunks = _default_chunks(shape, arr.itemsize)
    chunks = tuple(int(c) for c in chunks)
    codecs = [{"name": "bytes", "configuration": {"endian": "little"}}]
    if zstd:
        codecs.append({"name": "zstd", "configuration": {"level": 3, "checksum": False}})
    meta = {
        "zarr_format": 3, "node_type": "array", "shape": list(shape),
        "data_type": raw_dtype or _v3_name(arr.dtype),
        "chunk_grid": {"name": "regular", "configuration": {"chunk_shape": list(chunks)}},
        "chunk_key_encoding": {"name": "default", "configuration": {"separator": "/"}},
        "fill_value": 0, "codecs": codecs, "attributes": dict(attributes or {}),
    }
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "zarr.json"), "w") as f:
        json.dump(meta, f, indent=2)
    codec = _zstd() if zstd else None
    for idx in _chunk_indices(shape, chunks):
        sl = tuple(slice(i * c, min((i + 1) * c, s)) for i, c, s in zip(idx, chunks, shape))
        block = arr[sl] if shape else arr
        if shape and block.shape != chunks:  # edge chunk: stored full size, zero-filled
            full = np.zeros(chunks, dtype=arr.dtype)
            full[tuple(slice(0, b) for b in block.shape)] = block
            block = full
        data = np.asarray(block, order="C").astype(block.dtype.newbyteorder("<"), copy=False).tobytes()
        if codec is not None:
            data = codec.compress(data, asbytes=True)
        key = os.path.join(path, "c", *[str(i) for i in idx]) if shape else os.path.join(path, "c")
        os.makedirs(os.path.dirname(key), exist_ok=True)
        with open(key, "wb") as f:
            f.write(data)


def _default_chunks(shape, itemsize: int, target: int = 64 << 20) -> tuple[int, ...]:
    """Whole rows, at most ``target`` bytes per chunk (one chunk for small arrays)."""
    if not shape:
        return ()
    row = itemsize * int(np.prod(shape[1:])) if len(shape) > 1 else itemsize
    rows = max(1, min(shape[0], target // max(1, row)))
    return (rows,) + tuple(shape[1:])


def read_meta(path: str) -> dict:
    v3 = os.path.join(path, "zarr.json")
    if os.path.exists(v3):
        with open(v3) as f:
            return json.load(f)
    v2 = os.path.join(path, ".zarray")
    if os.path.exists(v2):
        with open(v2) as f:
            return json.load(f)
    raise FileNotFoundError(f"{path}: no zarr.json or .zarray")


def is_array(path: str) -> bool:
    return os.path.exists(os.path.join(path, "zarr.json")) or os.path.exists(os.path.join(path, ".zarray"))


def read_array(path: str) -> np.ndarray:
    """Read a zarr v3 or v2 array directory. bfloat16 arrays come back as uint16 holding the bits
    (``np.ndarray.view`` them into the framework's bf16 tensors)."""
    meta = read_meta(path)
    if meta.get("zarr_format") == 3:
        return _read_v3(path, meta)
    if meta.get("zarr_format") == 2:
        return _read_v2(path, meta)
    raise ValueError(f"{path}: unsupported zarr format {meta.get('zarr_format')}")


def _read_v3(path, meta):
    if meta.get("node_type") != "array":
        raise ValueError(f"{path}: not an array node")
    name = meta["data_type"]
    dtype = np.dtype(np.uint16) if name == "bfloat16" else np.dtype(_V3_TYPES[name])
    shape = tuple(meta["shape"])
    grid = meta["chunk_grid"]
    if grid.get("name") != "regular":
        raise ValueError(f"{path}: chunk grid {grid.get('name')!r} is not supported")
    chunks = tuple(grid["configuration"]["chunk_shape"])
    enc = meta.get("chunk_key_encoding", {"name": "default"})
    sep = enc.get("configuration", {}).get("separator", "/")
    prefix = ["c"] if enc.get("name", "default") == "default" else []
    endian, zstd, crc = "little", False, False
    for c in meta.get("codecs", []):
        if c["name"] == "bytes":
            endian = c.get("configuration", {}).get("endian", "little")
        elif c["name"] == "zstd":
            zstd = True
        elif c["name"] == "crc32c":  # a 4-byte checksum appended after the other codecs
            crc = True
        else:
            raise ValueError(f"{path}: codec {c['name']!r} is not supported")
    dt = dtype.newbyteorder("<" if endian == "little" else ">")
    fill = meta.get("fill_value", 0)
    out = np.full(shape, 0 if fill is None or isinstance(fill, str) else fill, dtype=dtype)
    codec = _zstd() if zstd else None
    for idx in _chunk_indices(shape, chunks):
        parts = prefix + [str(i) for i in idx]
        key = os.path.join(path, *parts) if sep == "/" else os.path.join(path, sep.join(parts))
        if not shape:
            key = os.path.join(path, "c")
        if not os.path.exists(key):
            continue
        with open(key, "rb") as f:
            data = f.read()
        if crc:
            data = data[:-4]
        if codec is not None:
            data = codec.decompress(data, decompressed_size=int(np.prod(chunks or (1,))) * dtype.itemsize,
                                    asbytes=True)
        block = np.frombuffer(data, dtype=dt).astype(dtype).reshape(chunks)
        if not shape:
            out[()] = block.reshape(())
            continue
        sl = tuple(slice(i * c, min((i + 1) * c, s)) for i, c, s in zip(idx, chunks, shape))
        out[sl] = block[tuple(slice(0, x.stop - x.start) for x in sl)]
    return out


def _read_v2(path, meta):
    dtype = np.dtype(meta["dtype"])
    if dtype.str.endswith("V2") or meta["dtype"] in ("bfloat16", "<V2"):
        dtype = np.dtype("<u2")
    shape = tuple(meta["shape"])
    chunks = tuple(meta["chunks"])
    comp = meta.get("compressor")
    if comp is not None and comp.get("id") != "zstd":
        raise ValueError(f"{path}: compressor {comp.get('id')!r} is not supported")
    sep = meta.get("dimension_separator", ".")
    order = meta.get("order", "C")
    fill = meta.get("fill_value", 0)
    out = np.full(shape, 0 if fill is None else fill, dtype=dtype.newbyteorder("="))
    codec = _zstd() if comp is not None else None
    for idx in _chunk_indices(shape, chunks):
        key = os.path.join(path, sep.join(str(i) for i in idx) if shape else "0")
        if not os.path.exists(key):
            continue
        with open(key, "rb") as f:
            data = f.read()
        if codec is not None:
            data = codec.decompress(data, decompressed_size=int(np.prod(chunks or (1,))) * dtype.itemsize,
                                    asbytes=True)
        block = np.frombuffer(data, dtype=dtype).reshape(chunks, order=order)
        if not shape:
            out[()] = block.reshape(())
            continue
        sl = tuple(slice(i * c, min((i + 1) * c, s)) for i, c, s in zip(idx, chunks, shape))
        out[sl] = block[tuple(slice(0, x.stop - x.start) for x in sl)]
    return out
