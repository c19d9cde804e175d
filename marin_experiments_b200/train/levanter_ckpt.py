"""Checkpoints in the reference's tree layout: the leaves of its train state as zarr arrays.

The reference saves its ``GrugTrainState`` (``step``, ``params``, ``opt_state``, ``ema_params``,
``pending_qb_betas``; megagpt-speedrun/train.py:310-317) with Levanter's checkpointer: one array
per pytree leaf, under a directory per path component, plus ``metadata.json`` written last
(megagpt-speedrun/checkpointing.py:42-78 keys the restore search on it). This module writes and
reads that tree for everything except the optimizer state, whose layout is optax's:

* ``params/...`` and ``ema_params/...`` in the reference's names and layouts
  (megagpt-speedrun/model.py:234-720): matrices ``[in, out]`` (this framework stores ``[out, in]``),
  ``w_q`` / ``w_k`` / ``w_v`` as three leaves (one fused ``w_qkv`` here), the routed experts'
  ``w_gate_up [E, D, 2I]`` with all gate columns first (block-interleaved rows here, see
  ``ops.layout``), the shared expert's ``w_gate`` / ``w_up`` / ``w_down``, ``blocks/<i>/...`` per layer;
* ``step`` (int32 scalar) and ``pending_qb_betas [layers, E]`` (fp32).

Arrays are zarr v3 (``utils.zarr_io``). A checkpoint written here restores a ``Trainer`` with the
same weights (``load_levanter``); ``save_levanter`` exports one. The optimizer moments restart at
zero on import, as in a weights-only initialisation. Expert-parallel shards are exported by a
process that holds every expert (restore the sharded checkpoint into one process first).
"""

from __future__ import annotations

import json
import os
import time

import numpy as np
import torch

from ..ops.layout import blocked_rows_to_gate_up, from_reference_gate_up, gate_up_to_blocked_rows, to_reference_gate_up
from ..utils import zarr_io


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def _module_of(model, name: str):
    mods = dict(model.named_modules())
    return mods.get(name.rsplit(".", 1)[0])


def _norm_path(prefix: str) -> tuple[str, str]:
    """Our ``<x>_norm`` NormPair prefix -> the reference's (RMSNorm path, GatedNorm path)."""
    table = {"attn_norm": ("rms_attn", "attn_gated_norm"), "mlp_norm": ("rms_mlp", "mlp_gated_norm"),
             "embed_norm": ("embed_norm", "embed_gated_norm"), "final_norm": ("final_norm", "final_gated_norm")}
    return table[prefix]


def to_reference_tree(model, values: dict[str, torch.Tensor]) -> dict[str, np.ndarray]:
    """Our parameters (name -> tensor in this framework's layout) -> the reference's leaves
    (path -> fp32 array in its layout)."""
    out: dict[str, np.ndarray] = {}
    for name, t in values.items():
        parts = name.split(".")
        if parts[0] == "blocks":
            base, rest = f"blocks/{parts[1]}", parts[2:]
        else:
            base, rest = "", parts
        pre = (base + "/") if base else ""
        head = rest[0]
        leaf = rest[-1]
        if head in ("attn_norm", "mlp_norm", "embed_norm", "final_norm"):
            rms, gated = _norm_path(head)
            if rest[1] == "rms":
                out[f"{pre}{rms}/weight"] = _np(t)
            else:  # gated.w_down [r, D] / gated.w_up [D, r] -> [D, r] / [r, D]
                out[f"{pre}{gated}/{leaf}"] = _np(t).T.copy()
        elif head == "attn":
            mod = _module_of(model, name)
            if leaf == "w_qkv":
                from ..parallel.tp import local_counts

                c = mod.cfg
                h, hkv = local_counts(c, mod.tp)
                hd = c.inferred_head_dim
                w = _np(t)
                out[f"{pre}attn/w_q"] = w[: h * hd].T.copy()
                out[f"{pre}attn/w_k"] = w[h * hd: (h + hkv) * hd].T.copy()
                out[f"{pre}attn/w_v"] = w[(h + hkv) * hd:].T.copy()
            else:  # attn_gate [h, D], w_o [D, h hd] -> transposed
                out[f"{pre}attn/{leaf}"] = _np(t).T.copy()
        elif head == "mlp" and t.dim() == 3:  # routed experts
            if leaf == "w_gate_up":
                out[f"{pre}mlp/expert_mlp/w_gate_up"] = _np(to_reference_gate_up(t.float()))
            else:  # w_down [E, D, I] -> [E, I, D]
                out[f"{pre}mlp/expert_mlp/w_down"] = np.ascontiguousarray(_np(t).transpose(0, 2, 1))
        elif head == "mlp" and leaf in ("router",):
            out[f"{pre}mlp/router"] = _np(t).T.copy()
        elif head == "mlp" and leaf in ("router_bias", "router_threshold"):
            out[f"{pre}mlp/{leaf}"] = _np(t)
        elif head in ("shared", "mlp"):  # dense SwiGLU / activation MLP
            mod = _module_of(model, name)
            if leaf == "w_gate_up" and getattr(mod, "glu", True):
                g, u = blocked_rows_to_gate_up(t.float())
                out[f"{pre}{head}/w_gate"] = _np(g).T.copy()
                out[f"{pre}{head}/w_up"] = _np(u).T.copy()
            elif leaf == "w_gate_up":
                out[f"{pre}{head}/w_up"] = _np(t).T.copy()
            else:
                out[f"{pre}{head}/w_down"] = _np(t).T.copy()
        elif leaf in ("token_embed",):
            out["token_embed"] = _np(t)
        elif leaf in ("embed_up", "head_down", "output_proj"):
            out[leaf] = _np(t).T.copy()
        else:  # parameters without a counterpart in the reference tree keep their own path
            out["/".join(parts)] = _np(t)
    return out


def from_reference_tree(model, leaves: dict[str, np.ndarray], names: list[str]) -> dict[str, torch.Tensor]:
    """The reference's leaves -> our parameters ``names`` (fp32 tensors in this framework's layout).
    Raises ``KeyError`` naming the first missing leaf."""
    out: dict[str, torch.Tensor] = {}

    def get(path):
        if path not in leaves:
            raise KeyError(f"checkpoint has no leaf {path!r}")
        return torch.from_numpy(np.asarray(leaves[path], dtype=np.float32))

    for name in names:
        parts = name.split(".")
        if parts[0] == "blocks":
            pre, rest = f"blocks/{parts[1]}/", parts[2:]
        else:
            pre, rest = "", parts
        head, leaf = rest[0], rest[-1]
        if head in ("attn_norm", "mlp_norm", "embed_norm", "final_norm"):
            rms, gated = _norm_path(head)
            out[name] = get(f"{pre}{rms}/weight") if rest[1] == "rms" else get(f"{pre}{gated}/{leaf}").t().contiguous()
        elif head == "attn":
            if leaf == "w_qkv":
                out[name] = torch.cat([get(f"{pre}attn/w_q").t(), get(f"{pre}attn/w_k").t(),
                                       get(f"{pre}attn/w_v").t()], 0).contiguous()
            else:
                out[name] = get(f"{pre}attn/{leaf}").t().contiguous()
        elif head == "mlp" and leaf in ("w_gate_up", "w_down") and f"{pre}mlp/expert_mlp/{leaf}" in leaves:
            w = get(f"{pre}mlp/expert_mlp/{leaf}")
            out[name] = from_reference_gate_up(w) if leaf == "w_gate_up" else w.transpose(1, 2).contiguous()
        elif head == "mlp" and leaf == "router":
            out[name] = get(f"{pre}mlp/router").t().contiguous()
        elif head == "mlp" and leaf in ("router_bias", "router_threshold"):
            out[name] = get(f"{pre}mlp/{leaf}")
        elif head in ("shared", "mlp"):
            if leaf == "w_gate_up" and f"{pre}{head}/w_gate" in leaves:
                out[name] = gate_up_to_blocked_rows(get(f"{pre}{head}/w_gate").t(), get(f"{pre}{head}/w_up").t())
            elif leaf == "w_gate_up":
                out[name] = get(f"{pre}{head}/w_up").t().contiguous()
            else:
                out[name] = get(f"{pre}{head}/w_down").t().contiguous()
        elif leaf == "token_embed":
            out[name] = get("token_embed")
        elif leaf in ("embed_up", "head_down", "output_proj"):
            out[name] = get(leaf).t().contiguous()
        else:
            out[name] = get("/".join(parts))
    return out


def _store_values(trainer, flat: torch.Tensor) -> dict[str, torch.Tensor]:
    st = trainer.store
    return {i.name: flat[i.offset: i.offset + i.numel].view(i.shape) for i in st.infos}


def save_levanter(trainer, path: str, *, step: int | None = None, zstd: bool = True) -> str:
    """Write ``step``, ``params``, ``ema_params`` (when the trainer keeps an EMA) and
    ``pending_qb_betas`` as zarr arrays under ``path``, then ``metadata.json``."""
    if trainer.dist is not None and getattr(trainer.dist, "ep_size", 1) > 1:
        raise ValueError("export from a process that holds every expert (restore the sharded checkpoint "
                         "into one process first)")
    step = trainer.step if step is None else step
    os.makedirs(path, exist_ok=True)
    trees = {"params": trainer.store.master}
    if trainer.ema is not None:
        trees["ema_params"] = trainer.ema
    for root, flat in trees.items():
        leaves = to_reference_tree(trainer.model, _store_values(trainer, flat))
        for p, a in leaves.items():
            zarr_io.write_array(os.path.join(path, root, *p.split("/")), a.astype(np.float32), zstd=zstd)
    zarr_io.write_array(os.path.join(path, "step"), np.array(step, dtype=np.int32), zstd=False)
    if trainer.pending_qb is not None:
        zarr_io.write_array(os.path.join(path, "pending_qb_betas"), _np(trainer.pending_qb), zstd=False)
    meta = {"step": int(step), "timestamp": time.strftime("%Y-%m-%dT%H:%M:%S"), "is_temporary": False}
    with open(os.path.join(path, "metadata.json"), "w") as f:
        json.dump(meta, f)
    return path


def _read_tree(root: str) -> dict[str, np.ndarray]:
    leaves = {}
    for dirpath, dirnames, _ in os.walk(root):
        if zarr_io.is_array(dirpath):
            leaves[os.path.relpath(dirpath, root).replace(os.sep, "/")] = zarr_io.read_array(dirpath)
            dirnames[:] = []
    return leaves


def load_levanter(trainer, path: str, *, params_only: bool = False) -> int:
    """Load a reference-layout checkpoint into ``trainer`` (masters, bf16 copies, EMA, QB betas and
    the step unless ``params_only``). Returns the checkpoint's step."""
    if not os.path.exists(os.path.join(path, "metadata.json")):
        raise FileNotFoundError(f"{path}: no metadata.json (not a complete checkpoint)")
    st = trainer.store
    names = [i.name for i in st.infos]
    trees = [("params", st.master)]
    if trainer.ema is not None and os.path.isdir(os.path.join(path, "ema_params")) and not params_only:
        trees.append(("ema_params", trainer.ema))
    with torch.no_grad():
        for root, flat in trees:
            vals = from_reference_tree(trainer.model, _read_tree(os.path.join(path, root)), names)
            for info in st.infos:
                flat[info.offset: info.offset + info.numel].copy_(vals[info.name].reshape(-1).to(flat.device))
        st.sync_compute()
    step = int(zarr_io.read_array(os.path.join(path, "step")))
    if not params_only:
        trainer.step = step
        qb = os.path.join(path, "pending_qb_betas")
        if trainer.pending_qb is not None and zarr_io.is_array(qb):
            trainer.pending_qb.copy_(torch.from_numpy(zarr_io.read_array(qb)).to(trainer.pending_qb.device))
    return step
