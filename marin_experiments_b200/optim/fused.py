"""Fused optimizer over a ``ParamStore``.

One step = (1) per-group squared gradient norms, (2) moments + Adam update / AdamH matrix sums,
(3) AdamH scale-invariant apply, all as multi-tensor kernels over a chunk table built once
(``csrc/optim.cu``); the bf16 compute copy is written in the same passes. Per-step
hyper-parameters (learning rates, bias corrections) live in a small device tensor filled from
pinned host memory, so the step can be captured in a CUDA graph. The CPU path runs the same math
with torch ops and is the oracle of the kernels.

Global-norm clipping is per group, as in the reference (each ``multi_transform`` branch chains its
own ``clip_by_global_norm``, megagpt-speedrun/optimizer.py:38-58). ``norm_hook`` lets a
distributed caller all-reduce the per-group squared norms of sharded groups before use.
"""

from __future__ import annotations

import math
import os

import numpy as np
import torch

CHUNK = 32768
HP = 9
# (flat start, length, matrix id, group, unused, moment shift: element k's moments at m[k - moff])
_CHUNK_DTYPE = np.dtype([("start", "<i8"), ("len", "<i4"), ("mat", "<i4"), ("group", "<i4"), ("pad", "<i4"),
                         ("moff", "<i8")])


def _ns_quintic(g: torch.Tensor, steps: int) -> torch.Tensor:
    """Newton-Schulz orthogonalisation with the quintic iteration of Muon
    (a, b, c) = (3.4445, -4.7750, 2.0315) (Jordan et al., "Muon", 2024); the iteration of
    megagpt-speedrun/async_pipeline.py:379-388 and, per expert, grug-moe-pp/pipeline_zb.py:68-106.
    On CUDA, a single matrix whose sides are multiples of 64 runs the iterations in bf16 on the
    tcgen05 GEMM (``_ns_quintic_sm100``), and a stack of matrices (the per-expert weights) whose
    short side is a multiple of 128 and long side a multiple of 64 runs them as grouped tcgen05
    GEMMs, one launch per product for the whole stack (``_ns_quintic_sm100_grouped``). Other shapes,
    and everything with ``MXK_NS_FP32=1``, run batched fp32 products."""
    single = g.dim() == 2 or math.prod(g.shape[:-2]) == 1
    fp32 = os.environ.get("MXK_NS_FP32", "0") == "1"
    if g.is_cuda and not fp32 and single and g.shape[-2] % 64 == 0 and g.shape[-1] % 64 == 0:
        return _ns_quintic_sm100(g, steps)
    short, long_ = min(g.shape[-2:]), max(g.shape[-2:])
    if g.is_cuda and not fp32 and not single and short % 128 == 0 and long_ % 64 == 0:
        return _ns_quintic_sm100_grouped(g, steps)
    a, b, c = 3.4445, -4.7750, 2.0315
    x = g.float()
    transpose = x.shape[-2] > x.shape[-1]
    if transpose:
        x = x.transpose(-1, -2)
    x = x / (x.norm(dim=(-2, -1), keepdim=True) + 1e-7)
    for _ in range(steps):
        A = x @ x.transpose(-1, -2)
        B = b * A + c * (A @ A)
        x = a * x + B @ x
    if transpose:
        x = x.transpose(-1, -2)
    return x


def _ns_quintic_sm100(g: torch.Tensor, steps: int) -> torch.Tensor:
    """The quintic Newton-Schulz iteration in bf16 on the tcgen05 GEMM, per matrix of ``g``
    ``[..., r, c]`` (sides multiples of 64): the Frobenius normalisation in fp32, then per step
    ``A = X X^T``, ``A A`` (A is symmetric), ``X <- a X + (b A + c A A) X`` with X the wide
    orientation. Returns fp32."""
    from ..ops import gemm as G

    a, b, c = 3.4445, -4.7750, 2.0315
    r, cdim = g.shape[-2], g.shape[-1]
    flat = g.reshape(-1, r, cdim).float()
    transpose = r > cdim
    out = torch.empty_like(flat)
    for i in range(flat.shape[0]):
        xf = flat[i].t() if transpose else flat[i]
        x = (xf / (xf.norm() + 1e-7)).to(torch.bfloat16).contiguous()
        for _ in range(steps):
            A = G.linear(x, x)  # x x^T  [m, m]
            AA = G.linear(A, A)  # A A^T = A A
            B = (b * A.float() + c * AA.float()).to(torch.bfloat16)
            x = (a * x.float() + G.linear_dx(B, x).float()).to(torch.bfloat16)  # B [m, m] @ x [m, n]
        out[i] = x.float().t() if transpose else x.float()
    return out.reshape(g.shape)


def _ns_quintic_sm100_grouped(g: torch.Tensor, steps: int) -> torch.Tensor:
    """The quintic iteration for a stack ``[..., r, c]`` of E matrices in bf16 on grouped tcgen05
    GEMMs (group e = matrix e): per step ``A = X X^T`` and ``A A`` as grouped K-major products and
    ``(b A + c A A) X`` with X as the MN-major operand, each one launch for the whole stack; the
    Frobenius normalisation and the ``a X + ...`` combination in fp32. Returns fp32."""
    from ..ops import gemm as G

    a, b, c = 3.4445, -4.7750, 2.0315
    r, cdim = g.shape[-2], g.shape[-1]
    flat = g.reshape(-1, r, cdim).float()
    e = flat.shape[0]
    transpose = r > cdim
    xf = flat.transpose(-1, -2) if transpose else flat
    m, n = xf.shape[-2], xf.shape[-1]  # wide orientation: m <= n, m a multiple of 128
    x = (xf / (xf.norm(dim=(-2, -1), keepdim=True) + 1e-7)).to(torch.bfloat16).reshape(e * m, n).contiguous()
    A = torch.empty(e * m, m, dtype=torch.bfloat16, device=g.device)
    AA = torch.empty_like(A)
    Y = torch.empty(e * m, n, dtype=torch.bfloat16, device=g.device)
    for _ in range(steps):
        G.gemm(x, x, A, G=e, M=m, N=m, K=n, a_grp=m, b_grp=m, c_grp=m)  # A_e = X_e X_e^T
        G.gemm(A, A, AA, G=e, M=m, N=m, K=m, a_grp=m, b_grp=m, c_grp=m)  # A_e A_e^T = A_e A_e
        B = (b * A.float() + c * AA.float()).to(torch.bfloat16)
        G.gemm(B, x, Y, b_mn=True, G=e, M=m, N=n, K=m, a_grp=m, b_grp=m, c_grp=m)  # B_e X_e
        x = (a * x.float() + Y.float()).to(torch.bfloat16)
    out = x.float().reshape(e, m, n)
    if transpose:
        out = out.transpose(-1, -2)
    return out.reshape(g.shape)


class FusedOptimizer:
    def __init__(self, store, cfg, num_train_steps: int):
        self.store = store
        self.cfg = cfg
        self.num_train_steps = num_train_steps
        self.groups = cfg.groups(store)
        self.names = list(self.groups)
        self.step_count = 0
        dev = store.device
        self.m = torch.zeros_like(store.master)
        self.v = torch.zeros_like(store.master)
        self.lr_fns = {n: cfg.lr_scheduler(num_train_steps, override_lr=g["lr"]) for n, g in self.groups.items()}
        self.norm_hook = None
        self.last_grad_norms: dict[str, float] = {}
        self.mat_hook = None
        self.shard: tuple[int, int] | None = None
        self.muon_infos = [i for g in self.groups.values() if g["kind"] == "muon" for i in g["infos"]]
        self.muon_owned = list(self.muon_infos)  # the Muon matrices whose update this rank computes
        self.has_adamh = any(g["kind"] == "adamh" for g in self.groups.values())
        self._build_chunks()
        if store.cuda:
            self.hp_host = torch.zeros(len(self.names), HP, dtype=torch.float32).pin_memory()
            self.hp = torch.zeros(len(self.names), HP, dtype=torch.float32, device=dev)
            self.gnorm2 = torch.zeros(len(self.names), dtype=torch.float64, device=dev)
            self.mat_sums = torch.zeros(self.mat_count, 3, dtype=torch.float64, device=dev)

    def _shard_ranges(self) -> list[tuple[int, int, int]]:
        """(lo, hi, moment shift) of every flat range this optimizer keeps state for: the whole
        buffer, or the sharded ranges with their moments packed back to back."""
        if self.shard is None:
            return [(0, 1 << 62, 0)]
        out, pos = [], 0
        for lo, hi in self.shard:
            out.append((lo, hi, lo - pos))
            pos += hi - lo
        return out

    def _build_chunks(self) -> None:
        """Chunk table over the adam / adamh groups: (flat start, length, matrix id, group, moment
        shift), each at most CHUNK elements, restricted to the shard ranges when the optimizer state
        is sharded."""
        shards = self._shard_ranges()
        rows = []
        mat = 0
        for gi, name in enumerate(self.names):
            g = self.groups[name]
            if g["kind"] == "muon":
                continue
            for info in g["infos"]:
                mats = info.matrices if g["kind"] == "adamh" else [[(info.offset, info.numel)]]
                for ranges in mats:
                    for start, length in ranges:
                        for lo, hi, moff in shards:
                            a, b = max(start, lo), min(start + length, hi)
                            for c0 in range(a, b, CHUNK):
                                rows.append((c0, min(CHUNK, b - c0), mat, gi, 0, moff))
                    mat += 1
        self.mat_count = max(mat, 1)
        arr = np.array(rows, dtype=_CHUNK_DTYPE) if rows else np.zeros(0, dtype=_CHUNK_DTYPE)
        self.nchunks = len(rows)
        if self.store.cuda:
            self.chunks = torch.from_numpy(arr.view(np.uint8).copy()).to(self.store.device)
        self._rows = rows

    def matrix_ids(self, pred) -> list[int]:
        """AdamH / Adam matrix ids (the chunk table's numbering) of the parameters where ``pred(info)``."""
        out, mat = [], 0
        for name in self.names:
            g = self.groups[name]
            if g["kind"] == "muon":
                continue
            for info in g["infos"]:
                mats = info.matrices if g["kind"] == "adamh" else [[(info.offset, info.numel)]]
                for _ in mats:
                    if pred(info):
                        out.append(mat)
                    mat += 1
        return out

    def set_shard(self, lo: int, hi: int, *more: tuple[int, int]) -> None:
        """Keep optimizer state only for the flat range [lo, hi) and any ``more`` ranges (ZeRO; with
        expert parallelism the rank's expert region is a second range): the moments shrink to the
        ranges (packed back to back), the chunk table covers them, and ``norm_hook`` / ``mat_hook``
        must sum the per-group squared norms and the AdamH matrix sums over the ranks holding the
        other shards. Range bounds are multiples of 4 (vector access of the moments)."""
        ranges = [(int(lo), int(hi))] + [(int(a), int(b)) for a, b in more]
        if any(a % 4 or b % 4 or b < a for a, b in ranges):
            raise ValueError(f"shard ranges must be ordered multiples of 4: {ranges}")
        # Muon orthogonalises whole matrices: each one must lie inside a range (this rank runs its
        # Newton-Schulz step) or outside all of them (another rank does)
        owned = []
        for info in self.muon_infos:
            s, e = info.offset, info.offset + info.numel
            if any(a <= s and e <= b for a, b in ranges):
                owned.append(info)
            elif any(a < e and s < b for a, b in ranges):
                raise ValueError(f"Muon matrix {info.name} [{s}, {e}) straddles a shard boundary {ranges}")
        self.muon_owned = owned
        self.shard = ranges
        n = sum(b - a for a, b in ranges)
        self.m = torch.zeros(n, dtype=torch.float32, device=self.store.device)
        self.v = torch.zeros_like(self.m)
        self._build_chunks()

    # --------------------------------------------------------------------------------- state
    def state_dict(self) -> dict:
        return {"step": self.step_count, "m": self.m.detach().cpu(), "v": self.v.detach().cpu()}

    def load_state_dict(self, sd: dict) -> None:
        self.step_count = int(sd["step"])
        self.m.copy_(sd["m"].to(self.m.device))
        self.v.copy_(sd["v"].to(self.v.device))

    def current_lrs(self) -> dict[str, float]:
        return {n: self.lr_fns[n](self.step_count) for n in self.names}

    # ---------------------------------------------------------------------------------- step
    def _fill_hp(self, t: int) -> None:
        cfg = self.cfg
        b1, b2 = cfg.beta1, cfg.beta2
        for gi, name in enumerate(self.names):
            g = self.groups[name]
            kind = {"adam": 0.0, "adamh": 1.0, "muon": 2.0}[g["kind"]]
            mx = cfg.max_grad_norm if cfg.max_grad_norm else 0.0
            self.hp_host[gi] = torch.tensor([kind, self.lr_fns[name](self.step_count), b1, b2, cfg.epsilon,
                                             g["wd"], 1 - b1 ** t, 1 - b2 ** t, mx])
        self.hp.copy_(self.hp_host, non_blocking=True)

    @torch.no_grad()
    def step(self, grad_scale: float = 1.0, zero_grad: bool = True) -> None:
        self.step_count += 1
        t = self.step_count
        st = self.store
        if st.cuda:
            from ..ops._ext import ext

            self._fill_hp(t)
            self.gnorm2.zero_()
            ext().opt_sqnorm(self.chunks, self.nchunks, st.grad, grad_scale, self.gnorm2)
            if self.norm_hook is not None:
                self.norm_hook(self.gnorm2, self.names)
            self.mat_sums.zero_()
            off = 0  # the chunks carry their moment shifts
            if self.shard is None and self.mat_hook is None:
                ext().opt_step(self.chunks, self.nchunks, self.hp, self.gnorm2, grad_scale, st.grad, self.m, self.v,
                               st.master, st.compute, self.mat_sums, self.has_adamh, 0, 0)
            else:
                ext().opt_step(self.chunks, self.nchunks, self.hp, self.gnorm2, grad_scale, st.grad, self.m, self.v,
                               st.master, st.compute, self.mat_sums, self.has_adamh, off, 1)
                if self.mat_hook is not None:
                    self.mat_hook(self.mat_sums)
                ext().opt_step(self.chunks, self.nchunks, self.hp, self.gnorm2, grad_scale, st.grad, self.m, self.v,
                               st.master, st.compute, self.mat_sums, self.has_adamh, off, 2)
        elif self.shard is not None or self.mat_hook is not None:
            self._step_cpu_chunks(t, grad_scale)
        else:
            self._step_cpu(t, grad_scale)
        if self.muon_infos:
            self._step_muon(t, grad_scale)
        if zero_grad:
            st.zero_grad()

    def _group_norm2(self, name: str, grad_scale: float) -> float:
        st = self.store
        acc = 0.0
        for info in self.groups[name]["infos"]:
            g = st.grad[info.offset: info.offset + info.numel] * grad_scale
            acc += float((g.double() ** 2).sum())
        return acc

    def _step_cpu(self, t: int, grad_scale: float) -> None:
        cfg = self.cfg
        st = self.store
        b1, b2, eps = cfg.beta1, cfg.beta2, cfg.epsilon
        bc1, bc2 = 1 - b1 ** t, 1 - b2 ** t
        norms = {}
        for name in self.names:
            if self.groups[name]["kind"] != "muon":
                norms[name] = self._group_norm2(name, grad_scale)
        if self.norm_hook is not None:
            vec = torch.tensor([norms.get(n, 0.0) for n in self.names], dtype=torch.float64)
            self.norm_hook(vec, self.names)
            norms = {n: float(vec[i]) for i, n in enumerate(self.names) if n in norms}
        for name in self.names:
            g = self.groups[name]
            if g["kind"] == "muon":
                continue
            lr = self.lr_fns[name](self.step_count)
            n = math.sqrt(norms[name])
            self.last_grad_norms[name] = n
            s = grad_scale
            if cfg.max_grad_norm and n >= cfg.max_grad_norm:
                s = grad_scale * cfg.max_grad_norm / n
            for info in g["infos"]:
                sl = slice(info.offset, info.offset + info.numel)
                gr = st.grad[sl] * s
                m = self.m[sl]
                v = self.v[sl]
                m.mul_(b1).add_(gr, alpha=1 - b1)
                v.mul_(b2).addcmul_(gr, gr, value=1 - b2)
                if g["kind"] == "adam":
                    u = (m / bc1) / ((v / bc2).sqrt() + eps)
                    p = st.master[sl]
                    p.sub_(lr * (u + g["wd"] * p))
                else:
                    for ranges in info.matrices:
                        idx = torch.cat([torch.arange(a, a + b) for a, b in ranges])
                        mm, vv, pp = self.m[idx], self.v[idx], st.master[idx]
                        u = (mm / bc1) / ((vv / bc2).sqrt() + eps)
                        pn = pp.norm()
                        un = u.norm().clamp_min(1e-10)
                        new = pp - lr * u * pn / un
                        nn_ = new.norm()
                        if nn_ > 0:
                            new = new / nn_ * pn
                        st.master[idx] = new

    def _step_cpu_chunks(self, t: int, grad_scale: float) -> None:
        """Chunk-table form of the step (the sharded path): per-group squared norms and AdamH
        matrix sums are partial over this shard and completed by ``norm_hook`` / ``mat_hook``; AdamH
        then uses ``||p - a u||^2 = S_pp - 2 a S_pu + a^2 S_uu`` with ``a = lr ||p|| / ||u||``."""
        cfg = self.cfg
        st = self.store
        b1, b2, eps = cfg.beta1, cfg.beta2, cfg.epsilon
        bc1, bc2 = 1 - b1 ** t, 1 - b2 ** t
        gn = torch.zeros(len(self.names), dtype=torch.float64)
        for start, ln, _, gi, _, _ in self._rows:
            gn[gi] += float((st.grad[start:start + ln].double() * grad_scale).pow(2).sum())
        if self.norm_hook is not None:
            self.norm_hook(gn, self.names)
        scale = []
        for gi, name in enumerate(self.names):
            n = math.sqrt(float(gn[gi]))
            self.last_grad_norms[name] = n
            s_ = grad_scale
            if cfg.max_grad_norm and n >= cfg.max_grad_norm:
                s_ = grad_scale * cfg.max_grad_norm / n
            scale.append(s_)
        sums = torch.zeros(self.mat_count, 3, dtype=torch.float64)
        upd = {}
        for start, ln, mat, gi, _, moff in self._rows:
            g = self.groups[self.names[gi]]
            sl = slice(start, start + ln)
            ml = slice(start - moff, start - moff + ln)
            gr = st.grad[sl] * scale[gi]
            self.m[ml].mul_(b1).add_(gr, alpha=1 - b1)
            self.v[ml].mul_(b2).addcmul_(gr, gr, value=1 - b2)
            u = (self.m[ml] / bc1) / ((self.v[ml] / bc2).sqrt() + eps)
            p = st.master[sl]
            lr = self.lr_fns[self.names[gi]](self.step_count)
            if g["kind"] == "adam":
                p.sub_(lr * (u + g["wd"] * p))
            else:
                sums[mat, 0] += float((p.double() ** 2).sum())
                sums[mat, 1] += float((p.double() * u.double()).sum())
                sums[mat, 2] += float((u.double() ** 2).sum())
                upd[start] = u
        if self.mat_hook is not None:
            self.mat_hook(sums)
        for start, ln, mat, gi, _, _ in self._rows:
            if start not in upd:
                continue
            lr = self.lr_fns[self.names[gi]](self.step_count)
            spp, spu, suu = (float(x) for x in sums[mat])
            pn = math.sqrt(spp)
            un = max(math.sqrt(suu), 1e-10)
            a = lr * pn / un
            nn2 = spp - 2 * a * spu + a * a * suu
            p = st.master[start:start + ln]
            new = p - a * upd[start]
            if nn2 > 0:
                new = new * (pn / math.sqrt(nn2))
            p.copy_(new)

    def _moment_shift(self, k: int) -> int:
        for lo, hi, moff in self._shard_ranges():
            if lo <= k < hi:
                return moff
        raise IndexError(f"flat index {k} outside the optimizer's ranges")

    def _step_muon(self, t: int, grad_scale: float) -> None:
        """Muon update on the matrices of the muon group (momentum, Newton-Schulz, shape scale);
        with sharded state, on the matrices this rank owns."""
        cfg = self.cfg
        st = self.store
        lr = self.lr_fns["muon"](self.step_count)
        wd = self.groups["muon"]["wd"]
        mu = getattr(cfg, "momentum", 0.95)
        for info in self.muon_owned:
            sl = slice(info.offset, info.offset + info.numel)
            g = (st.grad[sl] * grad_scale).view(info.shape)
            mo = info.offset - self._moment_shift(info.offset)
            m = self.m[mo: mo + info.numel].view(info.shape)
            m.mul_(mu).add_(g)
            upd = g + mu * m if getattr(cfg, "nesterov", True) else m
            if info.ndim < 2:
                continue
            mat = upd.reshape(-1, info.shape[-2], info.shape[-1])
            o = _ns_quintic(mat, getattr(cfg, "ns_steps", 5)).reshape(info.shape)
            scale = max(1.0, info.shape[-2] / info.shape[-1]) ** 0.5
            p = st.master[sl].view(info.shape)
            p.sub_(lr * (scale * o + wd * p))
            if st.cuda and self.shard is not None:
                from ..ops._ext import ext

                ext().cast_bf16(st.master[sl], st.compute[sl])
        if st.cuda and self.shard is None:
            st.sync_compute()
