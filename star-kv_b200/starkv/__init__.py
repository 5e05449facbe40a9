"""starkv — B200 (sm_100a) compressed-KV decode attention for STAR-KV.

Host layer over ``libstarkv.so`` (C ABI, ``include/starkv.h``): latent cache,
quantise/append, fused decode attention, and drop-in attention modules that
keep the reference's ``LlamaCustomAttention`` interface.
"""

from ._lib import StarKVError, load  # noqa: F401

__all__ = ["StarKVError", "load"]
