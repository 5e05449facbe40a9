"""Drive one synthetic decode step through the GPU path (tests, smoke, bench).

``build_step`` turns a ``LayerData`` (numpy, from ``starkv.synthetic``) or a
device-generated layer into a prefilled ``DecodeLayer`` plus the step's inputs
(rotated query, the appended token's latents, optional mask).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import numpy as np
import torch

from . import ops
from .layer import DecodeLayer, pack_k_u


@dataclass
class StepInputs:
    layer: DecodeLayer
    q: torch.Tensor          # (B, Hq, 128)
    k_new: torch.Tensor      # (B, 1, sum r_h)
    v_new: torch.Tensor      # (B, 1, R)
    mask: Optional[torch.Tensor]
    k_lat: Optional[torch.Tensor] = None   # full (B, T, sum r_h) latents when kept
    v_lat: Optional[torch.Tensor] = None


def build_step(data, device="cuda", keep_latents: bool = False) -> StepInputs:
    spec = data.spec
    dt = getattr(torch, spec.dtype)
    dev = torch.device(device)
    layout = ops.layout_from_spec(spec)
    k_u = pack_k_u([torch.from_numpy(u) for u in data.k_u]).to(dtype=dt, device=dev)
    v_u = torch.from_numpy(data.v_u).to(dtype=dt, device=dev)
    layer = DecodeLayer(layout, k_u, v_u, spec.theta, device=dev)
    k_lat = torch.from_numpy(np.concatenate(data.xk, axis=-1)).to(dtype=dt, device=dev)
    v_lat = torch.from_numpy(data.xv).to(dtype=dt, device=dev)
    L = spec.context
    layer.prefill(k_lat[:, :L].contiguous(), v_lat[:, :L].contiguous())
    q = torch.from_numpy(data.q).to(dtype=dt, device=dev)
    mask = None if data.mask is None else torch.from_numpy(data.mask).to(dev)
    return StepInputs(layer, q, k_lat[:, L:].contiguous(), v_lat[:, L:].contiguous(), mask,
                      k_lat if keep_latents else None, v_lat if keep_latents else None)


def device_layer(spec, device="cuda", seed: int = 0):
    """Full-size synthetic layer generated on the device (same distributions as
    ``starkv.synthetic.make_layer``; values differ from the numpy generator).

    Returns (StepInputs, host copies needed by a CPU check of sequence 0)."""
    dt = getattr(torch, spec.dtype)
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    B, T, D = spec.batch, spec.tokens, spec.head_dim
    K, R = spec.k_rank_total, spec.v_rank_total

    def lat(n_cols, groups: List[int]):
        x = torch.randn(B, T, n_cols, generator=g, device=dev, dtype=torch.float32)
        if spec.quantized:
            col = 0
            for r in groups:
                n = max(1, int(round(0.01 * r)))
                ch = torch.randperm(r, generator=g, device=dev)[:n] + col
                x[:, :, ch] *= 8.0
                col += r
        return x.to(dt)

    k_lat = lat(K, spec.k_ranks)
    v_lat = lat(R, [R])
    k_u_heads = [(torch.randn(D, r, generator=g, device=dev) / r ** 0.5).to(dt) for r in spec.k_ranks]
    v_u = torch.zeros(spec.num_kv_heads * D, R, device=dev, dtype=dt)
    vb = spec.v_block_of_kv()
    vcol = np.concatenate([[0], np.cumsum(spec.v_ranks)])
    for kv in range(spec.num_kv_heads):
        j = vb[kv]
        r = spec.v_ranks[j]
        v_u[kv * D:(kv + 1) * D, vcol[j]:vcol[j + 1]] = (torch.randn(D, r, generator=g, device=dev) / r ** 0.5).to(dt)
    q = torch.randn(B, spec.num_q_heads, D, generator=g, device=dev).to(dt)
    layout = ops.layout_from_spec(spec)
    layer = DecodeLayer(layout, pack_k_u(k_u_heads), v_u, spec.theta, device=dev)
    L = spec.context
    layer.prefill(k_lat[:, :L].contiguous(), v_lat[:, :L].contiguous())
    step = StepInputs(layer, q, k_lat[:, L:].contiguous(), v_lat[:, L:].contiguous(), None, k_lat, v_lat)
    return step, k_u_heads, v_u


def shard_layer(step: StepInputs, k_u_heads: List[torch.Tensor], v_u: torch.Tensor, spec, sub, rank: int,
                world: int) -> StepInputs:
    """The decode state of the heads ``rank`` owns, cut out of a full layer built
    by ``device_layer`` (same latents, up-projections and query as the full
    layer, so the gathered sharded outputs can be compared with the full step)."""
    from .dist import shard_range
    b0, b1, kv0, kv1 = shard_range(spec, rank, world)
    qpk = spec.num_q_heads // spec.num_kv_heads
    kcol = np.concatenate([[0], np.cumsum(spec.k_ranks)]).astype(int)
    vcol = np.concatenate([[0], np.cumsum(spec.v_ranks)]).astype(int)
    k_lat = step.k_lat[:, :, kcol[kv0]:kcol[kv1]].contiguous()
    v_lat = step.v_lat[:, :, vcol[b0]:vcol[b1]].contiguous()
    dev = step.q.device
    layout = ops.layout_from_spec(sub)
    layer = DecodeLayer(layout, pack_k_u(k_u_heads[kv0:kv1]),
                        v_u[kv0 * 128:kv1 * 128, vcol[b0]:vcol[b1]].contiguous(), sub.theta, device=dev)
    L = spec.context
    layer.prefill(k_lat[:, :L].contiguous(), v_lat[:, :L].contiguous())
    q = step.q[:, kv0 * qpk:kv1 * qpk].contiguous()
    return StepInputs(layer, q, k_lat[:, L:].contiguous(), v_lat[:, L:].contiguous(), None)
