"""Prompt (prefill) attention of the compressed-KV layer on the B200.

The reference's prefill (model.py:429-449) rebuilds full keys and values from
the latents and runs causal SDPA over them.  Here the rebuild is two plain GEMMs
per layer (``X_k U_k^T`` per KV head, ``X_v U_v^T`` once; cuBLAS) plus RoPE of
the keys, and the attention is the library's own tcgen05 flash-attention kernel
(``starkv_prefill_attention``): GQA by head index (no repeated K / V), the
values read in place from the (B, T, Hkv*128) product, the output written in
the (B, T, Hq, 128) order ``o_proj`` reads.
"""

from __future__ import annotations

from typing import Optional, Sequence

import torch

from . import ops


def rebuild_keys(k_lat: torch.Tensor, k_u_heads: Sequence[torch.Tensor], k_ranks: Sequence[int],
                 cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """RoPE(X_k U_k^T) per KV head (model.py:431-432): k_lat (B, T, sum r_h) ->
    (B, Hkv, T, 128).  cos / sin: (B or 1, T, 128) tables of positions 0..T-1."""
    B, T, _ = k_lat.shape
    out = torch.empty(B, len(k_ranks), T, 128, dtype=k_lat.dtype, device=k_lat.device)
    c0 = 0
    for h, (r, u) in enumerate(zip(k_ranks, k_u_heads)):
        out[:, h] = torch.matmul(k_lat[..., c0:c0 + r], u.to(k_lat.dtype).T)
        c0 += r
    half = 64
    rot = torch.cat([-out[..., half:], out[..., :half]], dim=-1)
    return out * cos[:, None] + rot * sin[:, None]


def rebuild_values(v_lat: torch.Tensor, v_u_weight: torch.Tensor, num_kv_heads: int) -> torch.Tensor:
    """X_v U_v^T split into heads (model.py:437-441): (B, T, R) -> a (B, Hkv, T, 128)
    strided view of the (B, T, Hkv*128) product."""
    B, T, _ = v_lat.shape
    full = torch.matmul(v_lat, v_u_weight.to(v_lat.dtype).T)
    return full.view(B, T, num_kv_heads, 128).transpose(1, 2)


def prompt_attention(q_rot: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, scaling: float,
                     out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """Causal attention of q_rot (B, Hq, T, 128) over keys / values (B, Hkv, T, 128)
    on the tensor cores; returns (B, Hq, T, 128) (a view of a (B, T, Hq, 128)
    tensor, so ``out.transpose(1, 2).reshape(B, T, -1)`` costs no copy)."""
    B, Hq, T, _ = q_rot.shape
    out = torch.empty(B, T, Hq, 128, dtype=out_dtype or q_rot.dtype, device=q_rot.device).transpose(1, 2)
    return ops.prefill_attention(q_rot, keys, values, scaling, out=out)
