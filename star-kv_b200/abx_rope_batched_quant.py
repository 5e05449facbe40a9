"""Drop-in for the reference kernel module ``abx_rope_batched_quant`` (imported at
LlamaLoRaAttention_headwise_quant.py:12, absent from the reference tree):
``abx(A, B, X1, X2, scale_upper, scale_lower, r4)`` -> q . RoPE_l(k_l) for every
slot, the K logits of the split int8 / int4 latent format, on the B200 K kernel.

A: (B, Hq, 1, 128) rotated query; B: (Hkv, r, 128) = U^T; X1 (B, H, L, split_r)
int8 and X2 (B, H, L, ceil(r4 / 2)) packed int4 (``quant_utils``), H the KV heads
or their query-head repeats (quant.py:146-147); scales (B, Hkv, L, 1) fp16.  The
latents are dequantised as quant.py's eager branch does (quant.py:137-140:
``cat(X1 * s_up, unpack(X2) * s_lo)``) into the query dtype and the logits come
from ``starkv_k_logits`` (``abx_rope_batched.abx``).  Returns (B, Hq, 1, L).
"""

import os as _os
import sys as _sys

_sys.path.insert(0, _os.path.dirname(_os.path.abspath(__file__)))

import torch  # noqa: E402

import abx_rope_batched  # noqa: E402
from quant_utils import unpack_uint8_to_int4_signed  # noqa: E402


def abx(A: torch.Tensor, B: torch.Tensor, X1: torch.Tensor, X2: torch.Tensor, scale_upper: torch.Tensor,
        scale_lower: torch.Tensor, r4: int, dtype=None) -> torch.Tensor:
    Hkv = B.shape[0]
    if X1.shape[1] != Hkv:                      # query-head repeats of the KV heads: take one copy each
        step = X1.shape[1] // Hkv
        X1, X2 = X1[:, ::step], X2[:, ::step]
    dt = dtype or A.dtype
    up = X1.to(torch.float32) * scale_upper.to(torch.float32)
    lo = unpack_uint8_to_int4_signed(X2, int(r4)).to(torch.float32) * scale_lower.to(torch.float32)
    x = torch.cat([up, lo], dim=-1).to(dt).contiguous()
    return abx_rope_batched.abx(A, B, x, dt)
