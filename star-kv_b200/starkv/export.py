"""Ragged-rank export of trained STAR-KV projections into the kernel layout.

The reference folds the soft-thresholded singular values into V and prunes dead
ranks per head (``export_kproj_for_triton``, model.py:284-325), then truncates
every head to the smallest kept rank (model.py:319-321) so that a uniform
``[H, 128, min_r]`` tensor feeds its kernels.  The B200 kernels take ragged
per-head ranks, so this export keeps every head's own kept rank, padded with
zero rows (VS) / zero columns (U) to a multiple of 16 — zeros that contribute
exactly nothing to the keys.  The V export (``export_vproj_for_triton``,
model.py:328-358) is the one-block case of the block-V export here, with the
rank padded to a multiple of 32 (the V group size).

Inputs are the decomposed modules' state dicts as saved by the reference
(``U.weight``, ``V.weight``, ``Sigma_blocks.{h}.diag`` /
``Sigma.diag`` and ``...soft_thres_layer.alpha``), so ``.pt`` checkpoints load
unchanged.
"""

from __future__ import annotations

from typing import List, Mapping, Sequence, Tuple

import torch
import torch.nn as nn


def _kept(diag: torch.Tensor, alpha: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """Indices of the ranks above the threshold and their folded values
    (model.py:306-310; an all-dead head keeps rank 0)."""
    keep = (diag > alpha).nonzero(as_tuple=False).view(-1)
    if keep.numel() == 0:
        keep = torch.zeros(1, dtype=torch.long, device=diag.device)
    return keep, (diag[keep] - alpha).clamp_min(0)


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


class RaggedKProj(nn.Module):
    """K projection with per-head ranks: ``VS`` (``Linear[in, sum r_h]``, heads
    concatenated) and ``U_{h}`` buffers of shape ``[head_dim, r_h]``."""

    def __init__(self, vs_weight: torch.Tensor, u_heads: Sequence[torch.Tensor]):
        super().__init__()
        self.ranks: List[int] = [int(u.shape[1]) for u in u_heads]
        self.VS = nn.Linear(vs_weight.shape[1], vs_weight.shape[0], bias=False)
        self.VS.weight = nn.Parameter(vs_weight, requires_grad=False)
        for h, u in enumerate(u_heads):
            self.register_buffer(f"U_{h}", u)

    def u_heads(self) -> List[torch.Tensor]:
        return [getattr(self, f"U_{h}") for h in range(len(self.ranks))]


class BlockVProj(nn.Module):
    """V projection in the reference's interface (``VS`` and ``U`` linears); ``U`` is
    block-diagonal over V blocks, ``ranks`` / ``kv_per_block`` describe the blocks."""

    def __init__(self, vs_weight: torch.Tensor, u_weight: torch.Tensor, ranks: Sequence[int],
                 kv_per_block: Sequence[int]):
        super().__init__()
        self.ranks = [int(r) for r in ranks]
        self.kv_per_block = [int(k) for k in kv_per_block]
        self.VS = nn.Linear(vs_weight.shape[1], vs_weight.shape[0], bias=False)
        self.VS.weight = nn.Parameter(vs_weight, requires_grad=False)
        self.U = nn.Linear(u_weight.shape[1], u_weight.shape[0], bias=False)
        self.U.weight = nn.Parameter(u_weight, requires_grad=False)


def _alpha(state: Mapping[str, torch.Tensor], prefix: str) -> float:
    return float(state[prefix + "soft_thres_layer.alpha"].reshape(-1)[0])


@torch.no_grad()
def export_kproj_ragged(state: Mapping[str, torch.Tensor], head_dim: int = 128, multiple: int = 16,
                        dtype: torch.dtype = torch.float16) -> RaggedKProj:
    """Per-head export of a ``DecomposeLinear_headwise`` state dict (model.py:284-325
    without the ``min_r`` truncation): head h keeps its ranks above its threshold,
    ``VS_h = V[cols] * (s - alpha)``, ``U_h = U[h*hd:(h+1)*hd, cols]``, padded to a
    multiple of ``multiple``."""
    U_w = state["U.weight"].float()
    V_w = state["V.weight"].float()
    H = 0
    while f"Sigma_blocks.{H}.diag" in state:
        H += 1
    if H == 0:
        raise ValueError("not a head-wise K decomposition (no Sigma_blocks)")
    vs_rows, u_heads = [], []
    col_off = 0
    for h in range(H):
        diag = state[f"Sigma_blocks.{h}.diag"].float()
        keep, s_vals = _kept(diag, _alpha(state, f"Sigma_blocks.{h}."))
        cols = col_off + keep
        vs = V_w[cols] * s_vals[:, None]
        u = U_w[h * head_dim:(h + 1) * head_dim][:, cols]
        rp = _round_up(vs.shape[0], multiple)
        vs_rows.append(torch.cat([vs, vs.new_zeros(rp - vs.shape[0], vs.shape[1])], 0))
        u_heads.append(torch.cat([u, u.new_zeros(u.shape[0], rp - u.shape[1])], 1).to(dtype).contiguous())
        col_off += diag.numel()
    return RaggedKProj(torch.cat(vs_rows, 0).to(dtype), u_heads)


@torch.no_grad()
def export_vproj_blocks(states: Sequence[Mapping[str, torch.Tensor]], kv_per_block: Sequence[int],
                        head_dim: int = 128, multiple: int = 32,
                        dtype: torch.dtype = torch.float16) -> BlockVProj:
    """Export of ``DecomposeLinear`` state dicts, one per V block (model.py:328-358;
    the reference's global V is a single block covering every KV head): block j keeps
    its ranks above its threshold, ``VS_j = V[keep] * (s - alpha)``, ``U_j = U[:, keep]``
    (rows = its KV heads' outputs), padded to a multiple of ``multiple``; ``U`` is
    assembled block-diagonal ``[Hkv*hd, sum r_j]``."""
    if len(states) != len(kv_per_block):
        raise ValueError("one state dict per V block")
    vs_rows, u_blocks, ranks = [], [], []
    for st, nkv in zip(states, kv_per_block):
        U_w = st["U.weight"].float()
        V_w = st["V.weight"].float()
        if U_w.shape[0] != nkv * head_dim:
            raise ValueError("U rows of a V block must be its KV heads' outputs")
        keep, s_vals = _kept(st["Sigma.diag"].float(), _alpha(st, "Sigma."))
        vs = V_w[keep] * s_vals[:, None]
        u = U_w[:, keep]
        rp = _round_up(vs.shape[0], multiple)
        vs_rows.append(torch.cat([vs, vs.new_zeros(rp - vs.shape[0], vs.shape[1])], 0))
        u_blocks.append(torch.cat([u, u.new_zeros(u.shape[0], rp - u.shape[1])], 1))
        ranks.append(rp)
    rows = sum(u.shape[0] for u in u_blocks)
    U = u_blocks[0].new_zeros(rows, sum(ranks))
    r0 = c0 = 0
    for u in u_blocks:
        U[r0:r0 + u.shape[0], c0:c0 + u.shape[1]] = u
        r0 += u.shape[0]
        c0 += u.shape[1]
    return BlockVProj(torch.cat(vs_rows, 0).to(dtype), U.to(dtype), ranks, kv_per_block)
