"""``torch.library`` registrations of the decode-path ops (CUDA only).

    torch.ops.starkv.decode_attn   fused decode attention  (starkv_decode_attention)
    torch.ops.starkv.k_attn        K logits, abx's contract (starkv_k_logits)
    torch.ops.starkv.v_attn        P . X_v in latent space, bx's contract (starkv_v_latent)
    torch.ops.starkv.quant_append  quantise + in-place cache append (starkv_append)

They replace the reference's kernel entry points (abx_rope_batched.abx,
bx_quant.bx, the quantiser + ``Cache.update``) for code that dispatches
through the torch operator registry.  A layer's ``starkv_layout`` travels as
its raw bytes in a CPU uint8 tensor (``layout_tensor``).  No CPU kernel is
registered: calling an op with CPU tensors raises.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import ops
from ._lib import Layout

_LIB = "starkv"


def layout_tensor(layout: Layout) -> torch.Tensor:
    """The layout's bytes as a CPU uint8 tensor (the ops' layout argument)."""
    return torch.frombuffer(bytearray(bytes(layout)), dtype=torch.uint8).clone()


def _layout(t: torch.Tensor) -> Layout:
    if t.device.type != "cpu" or t.dtype != torch.uint8:
        raise ValueError("layout must be a CPU uint8 tensor (starkv.torch_ops.layout_tensor)")
    return Layout.from_buffer_copy(t.numpy().tobytes())


class _CacheView:
    """The cache tensors of one call in the shape ops.* expects."""

    def __init__(self, layout, k_cache, k_scales, v_cache, v_params, length):
        self.layout, self.k_cache, self.k_scales = layout, k_cache, k_scales
        self.v_cache, self.v_params, self.length = v_cache, v_params, length


@torch.library.custom_op(f"{_LIB}::decode_attn", mutates_args=(), device_types="cuda")
def decode_attn(layout: torch.Tensor, q: torch.Tensor, k_u: torch.Tensor, v_u: torch.Tensor,
                inv_freq: torch.Tensor, k_cache: torch.Tensor, k_scales: Optional[torch.Tensor],
                v_cache: torch.Tensor, v_params: Optional[torch.Tensor], scaling: float, num_tokens: int,
                mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    lay = _layout(layout)
    cache = _CacheView(lay, k_cache, k_scales, v_cache, v_params, num_tokens)
    return ops.decode_attention(lay, cache, q, k_u, v_u, inv_freq, scaling, num_tokens, mask=mask)


@decode_attn.register_fake
def _(layout, q, k_u, v_u, inv_freq, k_cache, k_scales, v_cache, v_params, scaling, num_tokens, mask=None):
    return q.new_empty(q.shape)


@torch.library.custom_op(f"{_LIB}::k_attn", mutates_args=(), device_types="cuda")
def k_attn(layout: torch.Tensor, q: torch.Tensor, k_u: torch.Tensor, inv_freq: torch.Tensor,
           k_cache: torch.Tensor, k_scales: Optional[torch.Tensor], num_tokens: int) -> torch.Tensor:
    lay = _layout(layout)
    cache = _CacheView(lay, k_cache, k_scales, None, None, num_tokens)
    return ops.k_logits(lay, cache, q, k_u, inv_freq, num_tokens)


@k_attn.register_fake
def _(layout, q, k_u, inv_freq, k_cache, k_scales, num_tokens):
    return q.new_empty((q.shape[0], q.shape[1], num_tokens), dtype=torch.float32)


@torch.library.custom_op(f"{_LIB}::v_attn", mutates_args=(), device_types="cuda")
def v_attn(layout: torch.Tensor, probs: torch.Tensor, v_cache: torch.Tensor, v_params: Optional[torch.Tensor],
           num_tokens: int) -> torch.Tensor:
    lay = _layout(layout)
    cache = _CacheView(lay, None, None, v_cache, v_params, num_tokens)
    return ops.v_latent(lay, cache, probs, num_tokens)


@v_attn.register_fake
def _(layout, probs, v_cache, v_params, num_tokens):
    lay = _layout(layout)
    return probs.new_empty((probs.shape[0], probs.shape[1], lay.v_rank_total), dtype=torch.float32)


@torch.library.custom_op(f"{_LIB}::quant_append", mutates_args=("k_cache", "v_cache", "v_params"),
                         device_types="cuda")
def quant_append(layout: torch.Tensor, k_lat: torch.Tensor, v_lat: torch.Tensor, start_slot: int,
                 k_cache: torch.Tensor, k_scales: Optional[torch.Tensor], v_cache: torch.Tensor,
                 v_params: Optional[torch.Tensor]) -> None:
    lay = _layout(layout)
    c = ops.LatentCache.__new__(ops.LatentCache)
    c.layout, c.k_cache, c.k_scales, c.v_cache, c.v_params, c.length = lay, k_cache, k_scales, v_cache, v_params, start_slot
    c.append(k_lat.contiguous(), v_lat.contiguous())


@quant_append.register_fake
def _(layout, k_lat, v_lat, start_slot, k_cache, k_scales, v_cache, v_params):
    return None
