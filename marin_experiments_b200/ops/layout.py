"""Weight layouts shared by the kernels and the CPU path.

Gate/up weights of every SwiGLU MLP (routed experts, shared expert, dense GLU MLP) are stored
*block-interleaved*: rows ``[256*j, 256*j+128)`` hold gate rows ``[128*j, 128*j+128)`` and rows
``[256*j+128, 256*j+256)`` the matching up rows. One 256-column GEMM tile then carries the gate
and up pre-activations of the same 128 hidden units, so the SwiGLU is applied in the GEMM
epilogue. The reference stores ``w_gate_up [D, 2I]`` with all gate columns first
(megagpt-speedrun/_diag_ragged.py:47-56); ``to_reference_gate_up``/``from_reference_gate_up``
convert for checkpoint import/export.
"""

from __future__ import annotations

import torch

GLU_BLOCK = 128


def split_gate_up(h: torch.Tensor, inter: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Split a ``[..., 2I]`` blocked pre-activation into (gate, up), each ``[..., I]``."""
    lead = h.shape[:-1]
    hb = h.reshape(*lead, inter // GLU_BLOCK, 2, GLU_BLOCK)
    return hb[..., 0, :].reshape(*lead, inter), hb[..., 1, :].reshape(*lead, inter)


def merge_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    lead = gate.shape[:-1]
    inter = gate.shape[-1]
    g = gate.reshape(*lead, inter // GLU_BLOCK, 1, GLU_BLOCK)
    u = up.reshape(*lead, inter // GLU_BLOCK, 1, GLU_BLOCK)
    return torch.cat([g, u], dim=-2).reshape(*lead, 2 * inter)


def blocked_rows_to_gate_up(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """``w [..., 2I, D]`` (blocked rows) -> (gate ``[..., I, D]``, up ``[..., I, D]``)."""
    wt = w.transpose(-1, -2)
    g, u = split_gate_up(wt, w.shape[-2] // 2)
    return g.transpose(-1, -2), u.transpose(-1, -2)


def gate_up_to_blocked_rows(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    return merge_gate_up(gate.transpose(-1, -2), up.transpose(-1, -2)).transpose(-1, -2).contiguous()


def to_reference_gate_up(w: torch.Tensor) -> torch.Tensor:
    """Blocked ``[..., 2I, D]`` -> reference ``[..., D, 2I]`` (all gate columns, then all up)."""
    g, u = blocked_rows_to_gate_up(w)
    return torch.cat([g, u], dim=-2).transpose(-1, -2).contiguous()


def from_reference_gate_up(w_ref: torch.Tensor) -> torch.Tensor:
    inter = w_ref.shape[-1] // 2
    wt = w_ref.transpose(-1, -2)
    return gate_up_to_blocked_rows(wt[..., :inter, :], wt[..., inter:, :])
