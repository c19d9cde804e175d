"""Checkpoints: layout, save policy, restore search and weights-only initialisation.

Layout (one directory per checkpoint, ``<base>/step-<N>``, megagpt-speedrun/SUMMARY.md:12-13):

* ``metadata.json`` -- ``{"step": N, "timestamp": ..., "is_temporary": ...}``, written LAST, after
  every writer rank finished; a directory without it is not a checkpoint (the restore search keys on
  it exactly like megagpt-speedrun/checkpointing.py:42-78).
* ``manifest.json`` -- every array leaf: file, dtype, local and global shape, first index along the
  leading (expert) axis for expert-parallel shards, and CRC-32C of every 16 MiB piece.
* one raw little-endian file per leaf, named by its state path: ``params/blocks/0/attn/w_qkv.bin``,
  ``opt_state/m/...``, ``opt_state/v/...``, ``ema_params/...``; expert shards add their leading-axis
  range (``w_gate_up.e0-8.bin``). Scalars (``step``, optimizer counters) live in ``state.json``.

State paths mirror the reference train state ``(step, params, opt_state, ema_params,
pending_qb_betas)`` (megagpt-speedrun/train.py:310-317). Restore also accepts the legacy layout
whose paths carry a ``train_state/`` prefix (megagpt-speedrun/checkpointing.py:142-158).

Saving copies each flat fp32 buffer to page-locked host memory once (a few large device-to-host
copies), then writes all leaves from those host views with the native parallel writer in a
background thread, so training continues during the file IO. Replicated leaves are written by rank 0;
expert shards by the ranks of the first data-parallel replica. Every writer leaves
``rank-NNNNN.json`` with its part of the manifest; rank 0 merges them and writes ``metadata.json``.

Policy (levanter ``CheckpointerConfig`` fields, megagpt-speedrun/launch.py:152-165): a rolling
*temporary* checkpoint every ``save_interval_s`` seconds of wall clock, of which the newest
``keep_last_temporary_checkpoints`` are kept; *permanent* checkpoints at steps matching a ``keep``
policy ``{"every": N}``; a final one at the end of training.
"""

from __future__ import annotations

import datetime
import json
import os
import shutil
import threading
import time
from dataclasses import dataclass, field

import torch

from ..runtime import rt

PIECE = 16 << 20
FORMAT = "mxk-ckpt-1"


class CorruptCheckpointError(FileNotFoundError):
    """A leaf's bytes do not match its recorded CRC (treated like a missing checkpoint, so the
    restore search falls back to an older one)."""


# ------------------------------------------------------------------------------ state mapping
def _leaf_path(name: str) -> str:
    return name.replace(".", "/")


@dataclass
class _Leaf:
    key: str
    buf: torch.Tensor  # flat fp32 buffer (host or device) the leaf lives in
    offset: int
    numel: int
    shape: tuple
    global_shape: tuple
    axis0_start: int
    sharded: bool


def flat_buffers(trainer) -> dict[str, torch.Tensor]:
    """State-path prefix -> flat fp32 buffer laid out like ``trainer.store``."""
    out = {"params": trainer.store.master}
    opt = trainer.opt
    inner = getattr(opt, "inner", opt)
    out["opt_state/m"] = inner.m
    out["opt_state/v"] = inner.v
    if trainer.ema is not None:
        out["ema_params"] = trainer.ema
    if inner is not opt:  # delayed-gradient wrapper state
        out["opt_state/delayed/last_update"] = opt.last_update
        for k in ("v_ema", "m_raw"):
            if getattr(opt, k, None) is not None:
                out[f"opt_state/delayed/{k}"] = getattr(opt, k)
        for k in ("grad_ring", "param_ring"):
            ring = getattr(opt, k, None)
            if ring is not None:
                for i in range(ring.shape[0]):
                    out[f"opt_state/delayed/{k}/{i}"] = ring[i]
    return out


def scalar_state(trainer) -> dict:
    opt = trainer.opt
    inner = getattr(opt, "inner", opt)
    st = {"step": int(trainer.step), "opt_step": int(inner.step_count)}
    if inner is not opt:
        st["delayed_t"] = int(opt.t)
    return st


def load_scalar_state(trainer, st: dict) -> None:
    opt = trainer.opt
    inner = getattr(opt, "inner", opt)
    trainer.step = int(st["step"])
    inner.step_count = int(st.get("opt_step", st["step"]))
    if inner is not opt and "delayed_t" in st:
        opt.t = int(st["delayed_t"])


def _opt_shard(trainer):
    inner = getattr(trainer.opt, "inner", trainer.opt)
    return getattr(inner, "shard", None)


def _leaves(trainer, buffers: dict[str, torch.Tensor], ep_size: int, ep_rank: int) -> list[_Leaf]:
    out = []
    gname = getattr(trainer.model, "global_name", lambda n: n)
    n_store = trainer.store.numel
    shard = _opt_shard(trainer)
    local_lo = getattr(trainer.store, "expert_start", None)
    for prefix, buf in buffers.items():
        if buf.numel() != n_store:
            # optimizer state kept only for this rank's flat ranges (ZeRO): one leaf per range, at its
            # packed position in the moment buffer. Ranges inside the expert region hold this
            # expert-parallel rank's own experts, so their leaf is named per expert-parallel rank.
            pos = 0
            for lo, hi in shard:
                if hi <= lo:  # a rank whose range is empty (its span belongs to another rank's matrix)
                    continue
                key = f"{prefix}/__flat__"
                if local_lo is not None and lo >= local_lo and ep_size > 1:
                    key = f"{prefix}/__flat_ep{ep_rank}__"
                out.append(_Leaf(key, buf, pos, hi - lo, (hi - lo,), (n_store,), lo, True))
                pos += hi - lo
            continue
        for info in trainer.store.infos:
            sharded = info.sharded_over == "expert" and ep_size > 1
            gshape = tuple(info.shape)
            start = 0
            if sharded:
                e_loc = info.shape[0]
                gshape = (e_loc * ep_size,) + tuple(info.shape[1:])
                start = ep_rank * e_loc
            out.append(_Leaf(f"{prefix}/{_leaf_path(gname(info.name))}", buf, info.offset, info.numel, tuple(info.shape),
                             gshape, start, sharded))
    return out


def _file_of(leaf: _Leaf) -> str:
    if leaf.sharded:
        return f"{leaf.key}.e{leaf.axis0_start}-{leaf.axis0_start + leaf.shape[0]}.bin"
    return f"{leaf.key}.bin"


# ------------------------------------------------------------------------------------- save
class _PinnedPool:
    """Reusable page-locked host copies of the flat buffers (allocated once per shape)."""

    def __init__(self):
        self.bufs: dict[str, torch.Tensor] = {}

    def host(self, name: str, t: torch.Tensor) -> torch.Tensor:
        h = self.bufs.get(name)
        if h is None or h.numel() != t.numel():
            h = torch.empty(t.numel(), dtype=t.dtype, pin_memory=t.is_cuda)
            self.bufs[name] = h
        return h


def _dist_info(trainer):
    d = trainer.dist
    if d is None:
        return 0, 1, 1, 0
    return d.rank, d.world, d.ep_size, d.ep_rank


class SaveHandle:
    def __init__(self, thread: threading.Thread | None, box: dict):
        self.thread, self.box = thread, box

    def wait(self) -> None:
        if self.thread is not None:
            self.thread.join()
            self.thread = None
        if self.box.get("error") is not None:
            err, self.box["error"] = self.box["error"], None
            raise err


def save_checkpoint(trainer, path: str, *, step: int | None = None, temporary: bool = False,
                    pool: _PinnedPool | None = None, background: bool = False, threads: int = 8,
                    part_timeout_s: float = 600.0) -> SaveHandle:
    """Write the train state to ``path`` (a ``step-N`` directory)."""
    rank, world, ep_size, ep_rank = _dist_info(trainer)
    step = int(trainer.step if step is None else step)
    pool = pool or _PinnedPool()
    writers = list(range(ep_size)) if ep_size > 1 else [0]
    if _opt_shard(trainer) is not None:
        writers = list(range(world))
    if rank not in writers:
        return SaveHandle(None, {})
    buffers = flat_buffers(trainer)
    leaves = [lf for lf in _leaves(trainer, buffers, ep_size, ep_rank) if lf.sharded or rank == 0]
    # one device-to-host copy per flat buffer
    host = {}
    for name, buf in buffers.items():
        if any(lf.buf is buf for lf in leaves):
            h = pool.host(name, buf)
            h.copy_(buf.detach().reshape(-1), non_blocking=True)
            host[name] = h
    extra = {}
    if rank == 0 and trainer.pending_qb is not None:
        extra["pending_qb_betas"] = trainer.pending_qb.detach().float().cpu().contiguous()
    if buffers["params"].is_cuda:
        torch.cuda.current_stream().synchronize()
    by_buf = {id(b): n for n, b in buffers.items()}
    files, views, entries = [], [], {}
    for lf in leaves:
        h = host[by_buf[id(lf.buf)]]
        files.append(_file_of(lf))
        views.append(h[lf.offset: lf.offset + lf.numel].view(torch.uint8))
        entries[lf.key] = {"file": files[-1], "dtype": "float32", "shape": list(lf.shape),
                           "global_shape": list(lf.global_shape), "axis0_start": lf.axis0_start}
    for k, t in extra.items():
        files.append(f"{k}.bin")
        views.append(t.reshape(-1).view(torch.uint8))
        entries[k] = {"file": files[-1], "dtype": "float32", "shape": list(t.shape), "global_shape": list(t.shape),
                      "axis0_start": 0}
    scalars = scalar_state(trainer)
    scalars["step"] = step
    box: dict = {"error": None}

    def work():
        try:
            os.makedirs(path, exist_ok=True)
            for f in set(os.path.dirname(f) for f in files):
                os.makedirs(os.path.join(path, f), exist_ok=True)
            crcs = rt().write_files([os.path.join(path, f) for f in files], views, threads, False, PIECE)
            for (key, e), c in zip(entries.items(), crcs):
                e["crc32c"] = [int(x) for x in c]
                e["piece"] = PIECE
            part = os.path.join(path, f"rank-{rank:05d}.json")
            with open(part + ".tmp", "w") as f:
                json.dump(entries, f)
            os.replace(part + ".tmp", part)
            if rank != 0:
                return
            merged: dict[str, list] = {}
            deadline = time.monotonic() + part_timeout_s
            for r in writers:
                pr = os.path.join(path, f"rank-{r:05d}.json")
                while not os.path.exists(pr):
                    if time.monotonic() > deadline:
                        raise TimeoutError(f"checkpoint {path}: rank {r} did not finish writing")
                    time.sleep(0.05)
                with open(pr) as f:
                    for k, e in json.load(f).items():
                        merged.setdefault(k, []).append(e)
            manifest = {"format": FORMAT, "world_size": world, "ep_size": ep_size, "leaves": merged}
            with open(os.path.join(path, "manifest.json"), "w") as f:
                json.dump(manifest, f)
            with open(os.path.join(path, "state.json"), "w") as f:
                json.dump(scalars, f)
            meta = {"step": step, "timestamp": datetime.datetime.now(datetime.timezone.utc).isoformat(),
                    "is_temporary": bool(temporary)}
            with open(os.path.join(path, "metadata.json.tmp"), "w") as f:
                json.dump(meta, f)
            os.replace(os.path.join(path, "metadata.json.tmp"), os.path.join(path, "metadata.json"))
        except BaseException as e:  # surfaced by SaveHandle.wait()
            box["error"] = e

    if background:
        th = threading.Thread(target=work, name="checkpoint-writer", daemon=True)
        th.start()
        return SaveHandle(th, box)
    work()
    h = SaveHandle(None, box)
    h.wait()
    return h


# ------------------------------------------------------------------------------------- load
def _read_manifest(path: str) -> dict:
    mp = os.path.join(path, "manifest.json")
    if not os.path.exists(mp) or not os.path.exists(os.path.join(path, "metadata.json")):
        raise FileNotFoundError(f"no complete checkpoint at {path}")
    with open(mp) as f:
        return json.load(f)


def _read_partial(path: str, entries: list[dict], start: int, rows: int, row_elems: int, out: torch.Tensor) -> None:
    """Fill rows [start, start+rows) of a leading-axis-sharded leaf from whichever shard files
    overlap them (restore under a different expert-parallel size)."""
    import numpy as np

    done = 0
    for e in entries:
        e0, e1 = e["axis0_start"], e["axis0_start"] + e["shape"][0]
        lo, hi = max(e0, start), min(e1, start + rows)
        if lo >= hi:
            continue
        arr = np.fromfile(os.path.join(path, e["file"]), dtype="<f4", count=(hi - lo) * row_elems,
                          offset=(lo - e0) * row_elems * 4)
        out[(lo - start) * row_elems: (hi - start) * row_elems].copy_(torch.from_numpy(arr))
        done += hi - lo
    if done != rows:
        raise FileNotFoundError(f"expert rows [{start}, {start + rows}) not covered by the checkpoint shards")


def load_checkpoint(trainer, path: str, *, allow_partial: bool = False, params_only: bool = False,
                    threads: int = 8) -> int:
    """Load ``path`` into ``trainer``; returns the checkpoint step."""
    man = _read_manifest(path)
    leaves_meta: dict[str, list] = man["leaves"]
    pfx = "train_state/" if any(k.startswith("train_state/") for k in leaves_meta) else ""
    rank, world, ep_size, ep_rank = _dist_info(trainer)
    buffers = flat_buffers(trainer)
    if params_only:
        buffers = {k: v for k, v in buffers.items() if k in ("params", "ema_params")}
    pool = _PinnedPool()
    host = {n: pool.host(n, b) for n, b in buffers.items()}
    for n, b in buffers.items():
        host[n].copy_(b.detach().reshape(-1))  # keep values of leaves that stay missing (allow_partial)
    by_buf = {id(b): n for n, b in buffers.items()}
    files, views, expect = [], [], []
    for lf in _leaves(trainer, buffers, ep_size, ep_rank):
        ents = leaves_meta.get(pfx + lf.key)
        if ents is None:
            if params_only and lf.key.startswith("ema_params/"):
                continue
            if allow_partial:
                continue
            raise FileNotFoundError(f"{path}: missing leaf {lf.key}")
        dst = host[by_buf[id(lf.buf)]][lf.offset: lf.offset + lf.numel]
        exact = [e for e in ents if e["axis0_start"] == lf.axis0_start and tuple(e["shape"]) == lf.shape]
        if exact:
            files.append(os.path.join(path, exact[0]["file"]))
            views.append(dst.view(torch.uint8))
            expect.append(exact[0])
        else:
            if tuple(ents[0]["global_shape"]) != lf.global_shape:
                raise ValueError(f"{lf.key}: checkpoint shape {ents[0]['global_shape']} != {list(lf.global_shape)}")
            row = lf.numel // lf.shape[0]
            _read_partial(path, ents, lf.axis0_start, lf.shape[0], row, dst)
    try:
        crcs = rt().read_files(files, views, threads, PIECE)
    except ValueError as e:
        if "FileNotFound" in str(e):
            raise FileNotFoundError(str(e)) from e
        raise
    for f, e, c in zip(files, expect, crcs):
        if "crc32c" in e and [int(x) for x in c] != e["crc32c"]:
            raise CorruptCheckpointError(f"checksum mismatch in {f}")
    for n, b in buffers.items():
        b.copy_(host[n].view(b.shape).to(b.device))
    trainer.store.sync_compute()
    qb = leaves_meta.get(pfx + "pending_qb_betas")
    if qb and trainer.pending_qb is not None and not params_only:
        import numpy as np

        arr = np.fromfile(os.path.join(path, qb[0]["file"]), dtype="<f4").reshape(qb[0]["shape"])
        trainer.pending_qb.copy_(torch.from_numpy(arr))
    with open(os.path.join(path, "metadata.json")) as f:
        step = int(json.load(f)["step"])
    if not params_only:
        sp = os.path.join(path, "state.json")
        if os.path.exists(sp):
            with open(sp) as f:
                load_scalar_state(trainer, json.load(f))
        else:
            trainer.step = step
    return step


# --------------------------------------------------------------------------- restore search
def scan_checkpoint_root(root: str) -> list[tuple[int, str, str]]:
    """(step, timestamp, path) of every complete checkpoint directly under ``root`` (and ``root``
    itself), like megagpt-speedrun/checkpointing.py:42-78."""
    if not os.path.isdir(root):
        return []
    cands = [os.path.join(root, d) for d in sorted(os.listdir(root)) if os.path.isdir(os.path.join(root, d))]
    cands.append(root)
    out = []
    for c in cands:
        mp = os.path.join(c, "metadata.json")
        if not os.path.exists(mp):
            continue
        try:
            with open(mp) as f:
                meta = json.load(f)
        except (OSError, ValueError):
            continue
        try:
            step = int(meta.get("step"))
        except (TypeError, ValueError):
            step = -1
        ts = meta.get("timestamp")
        out.append((step, "" if ts is None else str(ts), c))
    return out


def checkpoint_candidates(search_paths) -> list[str]:
    """Every checkpoint under the search roots, newest (step, then timestamp) first, followed by
    the roots themselves."""
    cands = []
    for p in search_paths:
        cands += scan_checkpoint_root(p)
    cands.sort(key=lambda t: (t[0], t[1]), reverse=True)
    ordered = [c for _, _, c in cands]
    for p in search_paths:
        if p not in ordered:
            ordered.append(p)
    return ordered


def restore_from_checkpoint(trainer, search_paths, *, load_checkpoint_setting: bool | None = None,
                            allow_partial: bool = False, load_fn=load_checkpoint) -> str | None:
    """Newest-first restore with fallback to older checkpoints on ``FileNotFoundError``
    (megagpt-speedrun/checkpointing.py:81-139). Returns the path loaded, or ``None`` when starting
    from scratch; raises when ``load_checkpoint_setting`` is True and nothing loads."""
    search_paths = [p for p in (search_paths or []) if p]
    if not search_paths:
        if load_checkpoint_setting:
            raise FileNotFoundError("load_checkpoint=True but no checkpoint search paths are configured")
        return None
    if load_checkpoint_setting is False:
        return None
    cands = checkpoint_candidates(search_paths)
    last = None
    for c in cands:
        try:
            load_fn(trainer, c, allow_partial=allow_partial)
            return c
        except FileNotFoundError as e:
            last = e
    if load_checkpoint_setting:
        raise FileNotFoundError(f"could not load a checkpoint from {search_paths}; tried {cands}") from last
    return None


def initialize_from(trainer, path: str) -> str:
    """Weights-only graft: parameters (and EMA when saved) from the newest checkpoint under
    ``path``; the step restarts at 0 with fresh optimizer state (megagpt-speedrun/train.py:594-609)."""
    for c in checkpoint_candidates([path]):
        try:
            load_checkpoint(trainer, c, params_only=True)
        except FileNotFoundError:
            continue
        trainer.step = 0
        return c
    raise FileNotFoundError(f"no checkpoint to initialize from under {path}")


# ------------------------------------------------------------------------------ save policy
class Checkpointer:
    """Temporary (time-based, rolling) and permanent (step-policy) checkpoints."""

    def __init__(self, cfg, *, run_id: str | None = None, clock=time.monotonic, background: bool = True):
        base = cfg.base_path
        if cfg.append_run_id_to_base_path and run_id:
            base = os.path.join(base, run_id)
        self.cfg = cfg
        self.base = base
        self.tmp_base = cfg.temporary_base_path or base
        if cfg.temporary_base_path and cfg.append_run_id_to_base_path and run_id:
            self.tmp_base = os.path.join(cfg.temporary_base_path, run_id)
        self.clock = clock
        self.last_save = clock()
        self.background = background
        self.pool = _PinnedPool()
        self.pending: SaveHandle | None = None
        self.saved: list[tuple[int, str, bool]] = []

    def search_paths(self) -> list[str]:
        return [p for p in dict.fromkeys([self.base, self.tmp_base])]

    def is_permanent_step(self, step: int) -> bool:
        for pol in self.cfg.keep or ():
            every = int(pol.get("every", 0))
            until = pol.get("until")
            if every > 0 and step % every == 0 and (until is None or step <= int(until)):
                return True
        return False

    def _decide(self, trainer, step: int, force: bool) -> int:
        """0 = no save, 1 = temporary, 2 = permanent (rank 0 decides; broadcast to all ranks)."""
        dec = 0
        if self.is_permanent_step(step) or force:
            dec = 2
        elif self.clock() - self.last_save >= self.cfg.save_interval_s:
            dec = 1
        d = trainer.dist
        if d is not None and d.world > 1:
            import torch.distributed as tdist

            t = torch.tensor([dec], dtype=torch.int32, device=trainer.device if trainer.device.type == "cuda" else "cpu")
            tdist.broadcast(t, src=0)
            dec = int(t.item())
        return dec

    def on_step(self, trainer, step: int, force: bool = False) -> None:
        dec = self._decide(trainer, step, force)
        if dec:
            self.save(trainer, step, temporary=(dec == 1))

    def save(self, trainer, step: int, temporary: bool) -> None:
        self.wait()
        self.rank = _dist_info(trainer)[0]
        root = self.tmp_base if temporary else self.base
        path = os.path.join(root, f"step-{step}")
        self.pending = save_checkpoint(trainer, path, step=step, temporary=temporary, pool=self.pool,
                                       background=self.background)
        self.saved.append((step, path, temporary))
        self.last_save = self.clock()

    def wait(self) -> None:
        if self.pending is not None:
            h, self.pending = self.pending, None
            h.wait()
            self._cleanup()

    def on_end(self, trainer) -> None:
        if self.cfg.save_final and not any(s == trainer.step for s, _, _ in self.saved):
            self.save(trainer, trainer.step, temporary=False)
        self.wait()

    def _cleanup(self) -> None:
        """Delete temporary checkpoints beyond the newest ``keep_last_temporary_checkpoints``."""
        keep = self.cfg.keep_last_temporary_checkpoints
        if getattr(self, "rank", 0) != 0:
            return
        if keep is None or not os.path.isdir(self.tmp_base):
            return
        temps = []
        for step, _, path in scan_checkpoint_root(self.tmp_base):
            try:
                with open(os.path.join(path, "metadata.json")) as f:
                    if json.load(f).get("is_temporary"):
                        temps.append((step, path))
            except (OSError, ValueError):
                continue
        temps.sort(reverse=True)
        for _, path in temps[keep:]:
            shutil.rmtree(path, ignore_errors=True)
