"""Drop-in for the reference module ``LlamaLoRaAttention_headwise``: the same
``LlamaCustomAttention`` class and ``apply_rotary_pos_emb_custom`` helper, decoded
by the B200 kernels of ``libstarkv`` (see ``starkv.attention``).

``reorder`` and ``triton_kernel`` exist because the reference's scripts set them
(model.py:588-599); the decode path does not branch on them.
"""

import os as _os
import sys as _sys

_sys.path.insert(0, _os.path.dirname(_os.path.abspath(__file__)))

from starkv.attention import LlamaCustomAttention, StarKVCache, apply_rotary_pos_emb_custom  # noqa: E402,F401

reorder = True
triton_kernel = True
