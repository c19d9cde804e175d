"""Flat parameter store.

Every trainable parameter of a model lives in four flat fp32 device buffers -- ``master``,
``grad`` (the ``main_grad`` the kernels accumulate into), and the optimizer moments -- at the same
offsets, plus a flat bf16 ``compute`` buffer the model reads on the GPU. After ``attach`` each
module parameter is replaced by a view:

* >= 2-D parameters on CUDA: a view of the bf16 compute buffer (the optimizer writes it);
* 1-D parameters and every parameter on CPU: a view of the fp32 master buffer.

Each parameter's ``main_grad`` attribute is a view of ``grad``. Offsets are 64-element aligned,
and ``w_qkv`` is immediately followed by ``attn_gate`` so the attention block can run one GEMM over
``[q | k | v | gate]`` rows (``w_qkv._qkvg_view`` / ``_qkvg_grad``).

The store also records, per parameter, the AdamH *matrices* it contains (contiguous or
row-block-interleaved flat ranges whose Frobenius norms the scale-invariant update uses), so the
optimizer reproduces the reference's per-leaf / per-expert semantics
(megagpt-speedrun/adamh.py:52-67) on the fused layouts.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
from torch import nn

ALIGN = 64


@dataclass
class ParamInfo:
    name: str
    shape: tuple[int, ...]
    offset: int
    numel: int
    trainable: bool
    # AdamH matrices: list of lists of (start, length) flat ranges (relative to the buffer start)
    matrices: list[list[tuple[int, int]]] = field(default_factory=list)
    sharded_over: str | None = None  # "expert" for expert-parallel shards
    tp_sharded: bool = False  # a tensor-parallel shard (different on every rank of the TP group)

    @property
    def ndim(self) -> int:
        return len(self.shape)


def _row_block_ranges(offset: int, rows: int, cols: int, block: int, which: int, nblk: int = 2):
    """Flat ranges of the rows belonging to interleaved sub-matrix ``which`` (blocks of ``block``
    rows cycling through ``nblk`` sub-matrices)."""
    out = []
    for r0 in range(which * block, rows, nblk * block):
        out.append((offset + r0 * cols, block * cols))
    return out


def default_matrices(name: str, shape: tuple[int, ...], offset: int, module: nn.Module | None) -> list:
    """The AdamH matrices of one parameter.

    * ``w_qkv``: three matrices (q rows, k rows, v rows), matching the reference's separate
      ``w_q``/``w_k``/``w_v`` leaves (megagpt-speedrun/model.py:235-238).
    * dense / shared-expert ``w_gate_up`` (block-interleaved): gate rows and up rows are two
      matrices, matching ``DenseMLP.w_gate``/``w_up`` (megagpt-speedrun/model.py:331-342).
    * routed expert weights ``[E, ...]``: one matrix per expert (the reference vmaps AdamH over the
      leading axis, megagpt-speedrun/adamh.py:60-64); the fused per-expert ``w_gate_up`` is a
      single leaf there and stays one matrix here.
    * any other >= 2-D parameter: one matrix.
    """
    numel = 1
    for s in shape:
        numel *= s
    leaf = name.rsplit(".", 1)[-1]
    if len(shape) < 2:
        return [[(offset, numel)]]
    if leaf == "w_qkv" and module is not None and hasattr(module, "cfg"):
        from ..parallel.tp import local_counts

        c = module.cfg
        hd = c.inferred_head_dim
        d = shape[1]
        nh, nkv = local_counts(c, getattr(module, "tp", None))
        nq, nk = nh * hd, nkv * hd
        return [[(offset, nq * d)], [(offset + nq * d, nk * d)], [(offset + (nq + nk) * d, nk * d)]]
    if len(shape) == 3:
        per = shape[1] * shape[2]
        return [[(offset + e * per, per)] for e in range(shape[0])]
    if leaf == "w_gate_up" and module is not None and getattr(module, "glu", False):
        rows, cols = shape
        return [_row_block_ranges(offset, rows, cols, 128, 0), _row_block_ranges(offset, rows, cols, 128, 1)]
    return [[(offset, numel)]]


def _is_expert(module, leaf: str, p) -> bool:
    return getattr(module, "expert_range", None) is not None and leaf in ("w_gate_up", "w_down") and p.dim() == 3


class ParamStore:
    """``alloc(numel) -> (master, grad)`` places the two fp32 buffers (default: ordinary device
    tensors). ``expert_last``: lay out every routed-expert weight after all other parameters, with the
    expert region starting at ``expert_start`` (a multiple of ``pad_multiple``), so the replicated
    parameters form one prefix that can be sharded over data-parallel ranks while each
    expert-parallel rank keeps its own experts' range (ZeRO with expert parallelism)."""

    def __init__(self, model: nn.Module, device: torch.device | str, *, compute_dtype=torch.bfloat16,
                 moments: int = 2, pad_multiple: int = ALIGN, expert_last: bool = False, alloc=None):
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        self.compute_dtype = compute_dtype if self.cuda else torch.float32
        modules = dict(model.named_modules())
        self.infos: list[ParamInfo] = []
        self._params: dict[str, nn.Parameter] = {}
        off = 0
        named = list(model.named_parameters())
        self.expert_start = None
        if expert_last:
            def expert(item):
                name, p = item
                return _is_expert(modules.get(name.rsplit(".", 1)[0] if "." in name else ""), name.rsplit(".", 1)[-1], p)

            named = [x for x in named if not expert(x)] + [x for x in named if expert(x)]
            n_rep = sum(1 for x in named if not expert(x))
        for idx, (name, p) in enumerate(named):
            if expert_last and idx == n_rep:  # start of the expert region
                off = (off + pad_multiple - 1) // pad_multiple * pad_multiple
                self.expert_start = off
            mod_name = name.rsplit(".", 1)[0] if "." in name else ""
            module = modules.get(mod_name)
            leaf = name.rsplit(".", 1)[-1]
            # attn_gate directly after w_qkv (no padding) so the fused [q|k|v|gate] view exists
            if not (leaf == "attn_gate" and self.infos and self.infos[-1].name.endswith("w_qkv")):
                off = (off + ALIGN - 1) // ALIGN * ALIGN
            info = ParamInfo(name, tuple(p.shape), off, p.numel(), p.requires_grad)
            info.matrices = default_matrices(name, tuple(p.shape), off, module)
            if _is_expert(module, leaf, p):
                info.sharded_over = "expert"
            tp = getattr(module, "tp", None)
            if tp is not None and tp.size > 1 and leaf in getattr(module, "tp_sharded_params", ()):
                info.tp_sharded = True
            self.infos.append(info)
            self._params[name] = p
            off += p.numel()
        self.numel = (off + pad_multiple - 1) // pad_multiple * pad_multiple
        if expert_last and self.expert_start is None:  # no experts: the region is empty
            self.expert_start = self.numel
        dev = self.device
        if alloc is not None:  # e.g. buffers other GPUs read directly (a symmetric heap)
            self.master, self.grad = alloc(self.numel)
            self.master.zero_()
            self.grad.zero_()
        else:
            self.master = torch.zeros(self.numel, dtype=torch.float32, device=dev)
            self.grad = torch.zeros(self.numel, dtype=torch.float32, device=dev)
        self.compute = torch.zeros(self.numel, dtype=torch.bfloat16, device=dev) if self.cuda else None
        with torch.no_grad():
            for info in self.infos:
                src = self._params[info.name].detach()
                if src.is_meta:  # built on the meta device: values come from an init pass later
                    continue
                self.master[info.offset: info.offset + info.numel].copy_(src.reshape(-1).to(dev, torch.float32))
        self.sync_compute()
        self._attach(model, modules)
        self.by_name = {i.name: i for i in self.infos}

    # -------------------------------------------------------------------------------- views
    def master_view(self, info: ParamInfo) -> torch.Tensor:
        return self.master[info.offset: info.offset + info.numel].view(info.shape)

    def grad_view(self, info: ParamInfo) -> torch.Tensor:
        return self.grad[info.offset: info.offset + info.numel].view(info.shape)

    def compute_view(self, info: ParamInfo) -> torch.Tensor:
        if self.cuda and info.ndim >= 2:
            return self.compute[info.offset: info.offset + info.numel].view(info.shape)
        return self.master_view(info)

    def _attach(self, model: nn.Module, modules: dict[str, nn.Module]) -> None:
        self.params: dict[str, nn.Parameter] = {}
        for info in self.infos:
            mod_name, leaf = info.name.rsplit(".", 1) if "." in info.name else ("", info.name)
            mod = modules[mod_name]
            p = nn.Parameter(self.compute_view(info), requires_grad=info.trainable)
            p.main_grad = self.grad_view(info)
            if not self.cuda and info.trainable:
                p.register_post_accumulate_grad_hook(_accumulate_into_main_grad)
            setattr(mod, leaf, p)
            self.params[info.name] = p
        # fused [q | k | v | gate] views
        for i, info in enumerate(self.infos):
            if info.name.endswith("attn_gate") and i > 0 and self.infos[i - 1].name.endswith("w_qkv"):
                q = self.infos[i - 1]
                assert q.offset + q.numel == info.offset
                rows = q.shape[0] + info.shape[0]
                n = q.numel + info.numel
                wq = self.params[q.name]
                wq._qkvg_grad = self.grad[q.offset: q.offset + n].view(rows, q.shape[1])
                if self.cuda:
                    wq._qkvg_view = self.compute[q.offset: q.offset + n].view(rows, q.shape[1])
                else:
                    wq._qkvg_view = None

    # -------------------------------------------------------------------------------- ops
    def sync_compute(self) -> None:
        """Refresh the bf16 compute copy from the fp32 masters."""
        if self.cuda:
            from ..ops._ext import ext

            ext().cast_bf16(self.master, self.compute)

    def zero_grad(self) -> None:
        self.grad.zero_()

    def named_infos(self):
        return [(i.name, i) for i in self.infos]

    def state_dict(self) -> dict[str, torch.Tensor]:
        return {i.name: self.master_view(i).detach().cpu().clone() for i in self.infos}

    def load_state_dict(self, sd: dict[str, torch.Tensor], strict: bool = True) -> None:
        with torch.no_grad():
            for info in self.infos:
                if info.name not in sd:
                    if strict:
                        raise KeyError(f"missing parameter {info.name}")
                    continue
                t = sd[info.name]
                if tuple(t.shape) != info.shape:
                    raise ValueError(f"{info.name}: shape {tuple(t.shape)} != {info.shape}")
                self.master_view(info).copy_(t.to(self.device, torch.float32))
        self.sync_compute()


def _accumulate_into_main_grad(p: torch.Tensor) -> None:
    if p.grad is not None:
        p.main_grad.add_(p.grad.to(p.main_grad.dtype))
        p.grad = None
