"""Drop-in for the reference module ``LlamaLoRaAttention_headwise_quant``: the
quantised ``LlamaCustomAttention`` (int8 per-channel K codes, int4 per-token-group
V codes in a ``StarKVCache(quantized=True)``), decoded by ``libstarkv``.
"""

import os as _os
import sys as _sys

_sys.path.insert(0, _os.path.dirname(_os.path.abspath(__file__)))

from starkv.attention import LlamaCustomAttentionQuant as LlamaCustomAttention  # noqa: E402,F401
from starkv.attention import StarKVCache, apply_rotary_pos_emb_custom  # noqa: E402,F401

reorder = True
triton_kernel_k = True
triton_kernel_v = True
