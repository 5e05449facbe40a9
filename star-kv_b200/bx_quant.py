"""Drop-in for the reference kernel module ``bx_quant``: ``bx(b, x1, x2,
scale_v_upper, scale_v_lower, original_rank, upper_rank)`` (bx_quant.py:117-166)
computed by the B200 V kernel (``starkv_v_latent``).

Inputs in the reference kernel's format (bx_quant.py:38-114): b (B, H, L)
softmax weights; x1 (B, L, upper_rank/2) and x2 (B, L, lower_rank/2) packed
int4 nibbles, even rank in the low nibble, dequantised as (nib - 8) * scale with
one fp16 scale per token and block, scale_v_upper / scale_v_lower (B, L, 1).
Returns out[b, h, r] = sum_l b[b, h, l] * dequant(x)[b, l, r], (B, H, original_rank)
in b's dtype.

The per-token (nib - 8) * s dequantisation is the library's int4 V format with
one (scale, zero) = (s, -8 s) pair per 32-rank group (exact in fp16), so the
shim joins the two code blocks into one row per token, writes those pairs and
runs the fused V kernel.  Both block ranks must be multiples of 32.
"""

import os as _os
import sys as _sys

_sys.path.insert(0, _os.path.dirname(_os.path.abspath(__file__)))

import torch  # noqa: E402

from starkv import ops  # noqa: E402


def bx(b: torch.Tensor, x1: torch.Tensor, x2: torch.Tensor, scale_v_upper, scale_v_lower, original_rank,
       upper_rank=256) -> torch.Tensor:
    assert b.dim() == 3 and x1.dim() == 3 and x2.dim() == 3
    B, H, L = b.shape
    R, up = int(original_rank), int(upper_rank)
    lo = R - up
    if up % 32 or lo % 32 or x1.shape[-1] * 2 < up or x2.shape[-1] * 2 < lo:
        raise ValueError("bx: upper and lower ranks must be multiples of 32 and match x1 / x2")
    codes = torch.cat([x1[..., :up // 2], x2[..., :lo // 2]], dim=-1).contiguous()        # (B, L, R/2)
    su = scale_v_upper.reshape(B, L, 1).to(torch.float16)
    sl = scale_v_lower.reshape(B, L, 1).to(torch.float16)
    s = torch.cat([su.expand(B, L, up // 32), sl.expand(B, L, lo // 32)], dim=-1)
    params = torch.stack([s, s * -8.0], dim=-1).contiguous()                                 # (B, L, R/32, 2)
    lay = ops.make_layout(B, H, H, [16] * H, [R], [H], L, True, torch.float16,
                          k_offsets=[0] * H, k_batch_strides=[L * 16] * H)
    cache = ops.LatentCache.__new__(ops.LatentCache)
    cache.layout, cache.k_cache, cache.k_scales = lay, None, None
    cache.v_cache, cache.v_params, cache.length = codes, params, L
    out = ops.v_latent(lay, cache, b.to(torch.float32).contiguous(), L)
    return out.to(b.dtype)
