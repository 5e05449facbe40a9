"""Drop-in for the module the reference's quantised path imports and does not
ship (``from quant_utils import quantize_r_split_int8_int4_packed,
unpack_uint8_to_int4_signed``; LlamaLoRaAttention_headwise_quant.py:14,
bx_quant.py:18).  The format follows the reference's call sites:

* ``quantize_r_split_int8_int4_packed(x, split_r)`` -> ``(up_q, s_up, lo_q, s_lo, r4)``
  for x (..., r): the top ``split_r`` ranks as int8 with one symmetric fp16
  scale per row, ``s_up = fp16(absmax / 127)``, ``up_q = clamp(rint(x / s_up),
  -127, 127)``; the remaining ``r4 = r - split_r`` ranks as signed int4 with one
  symmetric fp16 scale per row, ``s_lo = fp16(absmax / 7)``, ``q = clamp(rint(x /
  s_lo), -8, 7)``, stored as the nibble ``q + 8``, two per byte, even rank in the
  low nibble (the order bx_quant.py:75-85 reads and dequantises as
  ``(nib - 8) * scale``).  A zero row gets scale 1.  Scales have shape (..., 1)
  (bx_quant.py:128-129).
* ``unpack_uint8_to_int4_signed(q, r)`` -> int8 (..., r) of ``nib - 8``.

Quantisation runs in the CUDA kernel ``starkv_quantize_split`` (IEEE fp32,
round-half-even); the unpacking is a view-level bit operation.
"""

import os as _os
import sys as _sys

_sys.path.insert(0, _os.path.dirname(_os.path.abspath(__file__)))

import torch  # noqa: E402

from starkv import ops  # noqa: E402


def quantize_r_split_int8_int4_packed(x: torch.Tensor, split_r: int):
    return ops.quantize_split(x, split_r)


def unpack_uint8_to_int4_signed(q: torch.Tensor, r: int) -> torch.Tensor:
    lo = (q & 0x0F).to(torch.int8) - 8
    hi = ((q >> 4) & 0x0F).to(torch.int8) - 8
    out = torch.stack([lo, hi], dim=-1).reshape(*q.shape[:-1], 2 * q.shape[-1])
    return out[..., :r]
