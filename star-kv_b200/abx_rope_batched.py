"""Drop-in for the reference kernel module ``abx_rope_batched``: ``abx(a, b, x, dtype)``
(abx_rope_batched.py:135-186) computed by ``starkv_k_logits`` on the tensor cores.

a: (B, Hq, 1, 128) rotated query; b: (Hkv, r, 128) = U^T of the K projection;
x: (B, Hkv, L, r) latent K cache.  Returns q . RoPE_l(x_l @ b) for every slot l,
(B, Hq, 1, L) in x's dtype, with RoPE theta 1e4 like the reference kernel
(abx_rope_batched.py:184).
"""

import os as _os
import sys as _sys

_sys.path.insert(0, _os.path.dirname(_os.path.abspath(__file__)))

import torch  # noqa: E402

from starkv import ops  # noqa: E402
from starkv.layer import rope_inv_freq  # noqa: E402

_INV = {}


def abx(a: torch.Tensor, b: torch.Tensor, x: torch.Tensor, dtype=torch.float16, theta: float = 10000.0) -> torch.Tensor:
    assert a.dim() == 4 and b.dim() == 3 and x.dim() == 4
    B, Hq, _, D = a.shape
    Hkv, r, _ = b.shape
    _, G, L, _ = x.shape
    assert G == Hkv and D == 128
    x = x.contiguous()
    lay = ops.make_layout(B, Hq, Hkv, [r] * Hkv, [32], [Hkv], L, False, x.dtype,
                          k_offsets=[h * L * r for h in range(Hkv)], k_batch_strides=[Hkv * L * r] * Hkv)
    cache = ops.LatentCache.__new__(ops.LatentCache)
    cache.layout, cache.k_cache, cache.k_scales, cache.v_cache, cache.v_params, cache.length = (
        lay, x.reshape(-1), None, None, None, L)
    key = (x.device, float(theta))
    if key not in _INV:
        _INV[key] = rope_inv_freq(theta, 128, x.device)
    k_u = b.transpose(-1, -2).to(x.dtype).contiguous().reshape(-1)
    lg = ops.k_logits(lay, cache, a[:, :, 0, :].contiguous(), k_u, _INV[key], L)
    return lg.view(B, Hq, 1, L).to(x.dtype)
