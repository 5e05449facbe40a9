"""Drop-in ``LlamaCustomAttention`` modules backed by libstarkv.

Same constructor, attributes and forward signatures as the reference's
``LlamaLoRaAttention_headwise.LlamaCustomAttention`` (headwise.py:32-148) and
``LlamaLoRaAttention_headwise_quant.LlamaCustomAttention`` (quant.py:38-202):
``q_proj``/``o_proj`` linears, ``k_proj.VS`` / ``k_proj.U`` (``[Hkv, 128, r]``) and
``v_proj.VS`` / ``v_proj.U`` (``Linear[Hkv*128, rv]``) as produced by the reference's
export (model.py:286-380), ``forward(hidden_states, position_embeddings,
attention_mask, position_ids, past_key_values, cache_position)`` returning
``(attn_output, None)``.

Decode steps (one query token) run the fused B200 path: the new token's latents
are appended to the cache and ``starkv_decode_attention`` computes the per-head
outputs, which go through ``o_proj``.  Two caches are accepted as
``past_key_values``:

* ``StarKVCache`` — the preallocated latent cache of this package (in-place
  append; int8/int4 codes for the quantised module);
* an HF ``Cache`` (e.g. ``DynamicCache``) — its ``update`` is called exactly as
  the reference does (headwise.py:99) and the decode kernels run directly on the
  returned ``(B, Hkv, L, r)`` / ``(B, L, rv)`` latent tensors (unquantised).

Prompt steps (more than one query token) store the latents in the cache and
compute the prompt's attention on the GPU with torch SDPA on the reconstructed
keys/values, as the reference's own prefill branch does (model.py:429-449).

RoPE: the query is rotated with the supplied ``position_embeddings`` exactly as
``apply_rotary_pos_emb_custom`` (headwise.py:22-29); cached keys are rotated by
their slot positions inside the kernel, with ``inv_freq`` from the config's
``rope_theta`` (the reference's HF default rope).
"""

from __future__ import annotations

from typing import Dict, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops, prefill
from .layer import DecodeLayer, rope_inv_freq


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def apply_rotary_pos_emb_custom(x, cos, sin, unsqueeze_dim=1):
    """The reference's RoPE helper (headwise.py:22-29): when the tables do not
    match the sequence length, the last table row is used."""
    cos = cos.unsqueeze(unsqueeze_dim)
    sin = sin.unsqueeze(unsqueeze_dim)
    if x.shape[-2] != cos.shape[-2]:
        cos = cos[:, :, -1, :].unsqueeze(2)
        sin = sin[:, :, -1, :].unsqueeze(2)
    return (x * cos) + (rotate_half(x) * sin)


try:                                                    # transformers' cache base class (the model code's type)
    from transformers.cache_utils import Cache as _HFCache
except Exception:                                       # pragma: no cover - transformers absent
    _HFCache = object


class StarKVCache(_HFCache):
    """Preallocated per-layer latent caches (the static replacement of the
    reference's ``DynamicCache`` for the drop-in modules).  A transformers
    ``Cache``: pass it as ``past_key_values`` to ``LlamaModel`` /
    ``LlamaForCausalLM.forward`` (as the reference's latency harness does with
    its caches, latency.py:69-99) and the drop-in modules append each step's
    latents in place.

    capacity: token slots per sequence; quantized: int8 K / int4 V codes."""

    def __init__(self, capacity: int, quantized: bool = False):
        if _HFCache is not object:
            super().__init__(layers=[])
        self.capacity = int(capacity)
        self.quantized = bool(quantized)
        self.states: Dict[int, DecodeLayer] = {}

    # ---- the Cache interface the transformers model code uses
    def get_seq_length(self, layer_idx: int = 0) -> int:
        st = self.states.get(layer_idx)
        if st is None and self.states:
            st = next(iter(self.states.values()))
        return 0 if st is None else st.length

    def get_mask_sizes(self, query_length: int, layer_idx: int = 0):
        return self.get_seq_length(layer_idx) + query_length, 0

    def get_max_cache_shape(self, layer_idx: int = 0) -> int:
        return self.capacity

    @property
    def is_compileable(self) -> bool:
        return False

    @property
    def is_initialized(self) -> bool:
        return bool(self.states)

    @property
    def is_sliding(self):
        return [False] * max(1, len(self.states))

    def __len__(self):
        return len(self.states)

    def update(self, key_states, value_states, layer_idx, *args, **kwargs):
        raise NotImplementedError("StarKVCache is written by the STAR-KV attention modules themselves "
                                  "(latents appended in place by the decode kernels)")

    def layer(self, layer_idx: int, module: "LlamaCustomAttention", batch: int, dtype: torch.dtype) -> DecodeLayer:
        st = self.states.get(layer_idx)
        if st is None:
            v_ranks, v_kv = module.v_blocks()
            lay = ops.make_layout(batch, module.num_heads, module.num_key_value_heads, module.k_ranks(),
                                  v_ranks, v_kv, self.capacity, self.quantized, dtype)
            st = DecodeLayer(lay, module.packed_k_u(dtype), module.v_proj.U.weight.to(dtype).contiguous(),
                             module.rope_theta)
            self.states[layer_idx] = st
        return st


class LlamaCustomAttention(nn.Module):
    """Llama attention with low-rank (SVD-factored) K/V projections whose latent
    cache is decoded by the B200 kernels.  ``quantized`` selects the int8 K /
    int4 V cache of the quantised module."""

    quantized = False

    def __init__(self, config, layer_idx: Optional[int] = None, decomp_goup_num: Optional[int] = 1):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.attention_dropout = config.attention_dropout
        self.hidden_size = config.hidden_size
        self.num_heads = config.num_attention_heads
        self.head_dim = self.hidden_size // self.num_heads
        self.num_key_value_heads = config.num_key_value_heads
        self.num_key_value_groups = self.num_heads // self.num_key_value_heads
        self.max_position_embeddings = config.max_position_embeddings
        rp = getattr(config, "rope_parameters", None) or {}
        self.rope_theta = float(getattr(config, "rope_theta", None) or rp.get("rope_theta", 10000.0))
        self.is_causal = True
        self.scaling = self.head_dim ** -0.5
        bias = config.attention_bias
        self.q_proj = nn.Linear(self.hidden_size, self.num_heads * self.head_dim, bias=bias)
        self.k_proj = nn.Linear(self.hidden_size, self.num_key_value_heads * self.head_dim, bias=bias)
        self.v_proj = nn.Linear(self.hidden_size, self.num_key_value_heads * self.head_dim, bias=bias)
        self.o_proj = nn.Linear(self.num_heads * self.head_dim, self.hidden_size, bias=bias)
        self.decomp_goup_num = decomp_goup_num
        self.decomp_goup_num_kv = decomp_goup_num // self.num_key_value_groups
        self._u_cache = None

    # ---- weight views in the layouts the kernels consume
    def k_ranks(self):
        """Per-KV-head K ranks: the reference's uniform ``k_proj.U`` ``[Hkv, 128, r]``
        or the per-head ranks of a ``RaggedKProj`` (``starkv.export``)."""
        ranks = getattr(self.k_proj, "ranks", None)
        if ranks is not None:
            return list(ranks)
        r = int(self.k_proj.U.shape[-1])
        return [r] * self.num_key_value_heads

    def k_uniform(self) -> bool:
        return len(set(self.k_ranks())) == 1

    def k_u_heads(self):
        """Per-head K up-projections ``[128, r_h]``."""
        if hasattr(self.k_proj, "u_heads"):
            return self.k_proj.u_heads()
        return list(self.k_proj.U.unbind(0))

    def v_rank(self) -> int:
        return int(self.v_proj.U.weight.shape[1])

    def v_blocks(self):
        """V block ranks and KV heads per block (one global block in the reference)."""
        if hasattr(self.v_proj, "kv_per_block"):
            return list(self.v_proj.ranks), list(self.v_proj.kv_per_block)
        return [self.v_rank()], [self.num_key_value_heads]

    def packed_k_u(self, dtype) -> torch.Tensor:
        """The per-head K up-projections in the packed layout (head after head)."""
        heads = self.k_u_heads()
        key = (tuple(u.data_ptr() for u in heads), dtype)
        if self._u_cache is None or self._u_cache[0] != key:
            self._u_cache = (key, torch.cat([u.to(dtype).contiguous().reshape(-1) for u in heads]))
        return self._u_cache[1]

    # ---- forward
    def forward(self, hidden_states, position_embeddings, attention_mask, position_ids=None, past_key_values=None,
                cache_position=None, **kwargs):
        B, q_len, _ = hidden_states.shape
        dt = hidden_states.dtype
        Hq, Hkv, D = self.num_heads, self.num_key_value_heads, self.head_dim
        q = self.q_proj(hidden_states).view(B, q_len, Hq, D).transpose(1, 2)
        cos, sin = position_embeddings
        q = apply_rotary_pos_emb_custom(q, cos, sin)
        fused_decode = isinstance(past_key_values, StarKVCache) and q_len == 1
        if not fused_decode:
            k_lat = torch.matmul(hidden_states, self.k_proj.VS.weight.T)      # (B, q, Hkv*r)
            v_lat = torch.matmul(hidden_states, self.v_proj.VS.weight.T)      # (B, q, rv)
        r = self.k_ranks()[0]
        uniform = self.k_uniform()

        def key_view(lat):                     # (B, Hkv, L, r) for uniform ranks, else the (B, L, sum r_h) latents
            return lat.view(B, lat.shape[1], Hkv, r).transpose(1, 2) if uniform else lat

        if isinstance(past_key_values, StarKVCache):
            st = past_key_values.layer(self.layer_idx, self, B, dt)
            if q_len == 1:
                mask = self._decode_mask(attention_mask, B, st.length + 1)
                # fused k_proj.VS / v_proj.VS projection + quantise-append (one kernel)
                out = st.step_from_hidden(q[:, :, 0, :], hidden_states, self.k_proj.VS.weight.to(dt),
                                          self.v_proj.VS.weight.to(dt), mask=mask)
                return self.o_proj(out.reshape(B, 1, Hq * D)), None
            if st.length != 0:
                raise NotImplementedError("multi-token steps after the prompt are not supported by the decode path")
            st.prefill(k_lat.contiguous(), v_lat.contiguous())
            keys, values = key_view(k_lat), v_lat
        elif past_key_values is not None:
            if not uniform:
                raise ValueError("ragged K ranks need a StarKVCache (an HF Cache stores (B, Hkv, L, r) tensors)")
            keys, values = past_key_values.update(k_lat.view(B, q_len, Hkv, r).transpose(1, 2), v_lat,
                                                  self.layer_idx)
            if q_len == 1:
                out = self._decode_on_tensors(q[:, :, 0, :], keys, values, attention_mask)
                return self.o_proj(out.reshape(B, 1, Hq * D)), None
        else:
            keys, values = key_view(k_lat), v_lat
            if q_len == 1:
                if not uniform:
                    raise ValueError("ragged K ranks need a StarKVCache for decode steps")
                out = self._decode_on_tensors(q[:, :, 0, :], keys, values, attention_mask)
                return self.o_proj(out.reshape(B, 1, Hq * D)), None
        out = self._prompt_attention(q, keys, values, cos, sin, attention_mask)
        return self.o_proj(out.transpose(1, 2).reshape(B, q_len, Hq * D)), None

    # ---- helpers
    @staticmethod
    def _decode_mask(attention_mask, B, L):
        if attention_mask is None:
            return None
        m = attention_mask[:, 0, -1, :L] if attention_mask.dim() == 4 else attention_mask[:, :L]
        return m.to(torch.float32).expand(B, L).contiguous()

    def _decode_on_tensors(self, q_rot, keys, values, attention_mask):
        """Decode over an HF cache's latent tensors (B, Hkv, L, r) / (B, L, rv) in place."""
        B, Hkv, L, r = keys.shape
        keys = keys.contiguous()
        values = values.contiguous()
        dt = keys.dtype
        v_ranks, v_kv = self.v_blocks()
        lay = ops.make_layout(B, self.num_heads, Hkv, [r] * Hkv, v_ranks, v_kv, L, False, dt,
                              k_offsets=[h * L * r for h in range(Hkv)], k_batch_strides=[Hkv * L * r] * Hkv)
        cache = ops.LatentCache.__new__(ops.LatentCache)
        cache.layout, cache.k_cache, cache.k_scales = lay, keys.reshape(-1), None
        cache.v_cache, cache.v_params, cache.length = values, None, L
        inv = getattr(self, "_inv_freq", None)
        if inv is None or inv.device != keys.device:
            inv = self._inv_freq = rope_inv_freq(self.rope_theta, 128, keys.device)
        return ops.decode_attention(lay, cache, q_rot.contiguous(), self.packed_k_u(dt),
                                    self.v_proj.U.weight.to(dt).contiguous(), inv, self.scaling, L,
                                    mask=self._decode_mask(attention_mask, B, L))

    def _prompt_attention(self, q, keys, values, cos, sin, attention_mask):
        """Prompt (q_len > 1) attention on K/V reconstructed from the latents
        (model.py:429-449).  A causal prompt from position 0 (no explicit mask) runs
        the library's tcgen05 flash-attention kernel (``starkv.prefill``); an explicit
        additive mask, or queries that continue an earlier prompt, go to torch SDPA
        with that mask, as the reference does."""
        B, Hq, Lq, D = q.shape
        Hkv = self.num_key_value_heads
        if (attention_mask is None and keys.shape[-2] == Lq and q.is_cuda
                and q.dtype in (torch.float16, torch.bfloat16)):
            lat = keys if keys.dim() == 3 else keys.transpose(1, 2).reshape(B, Lq, -1)
            k_full = prefill.rebuild_keys(lat, self.k_u_heads(), self.k_ranks(), cos, sin)
            v_full = prefill.rebuild_values(values, self.v_proj.U.weight, Hkv)
            return prefill.prompt_attention(q, k_full, v_full, self.scaling)
        if keys.dim() == 4:                                                    # (B, Hkv, L, r)
            u = torch.stack(self.k_u_heads()).to(keys.dtype)                   # (Hkv, D, r)
            k_full = torch.matmul(keys, u.transpose(-2, -1))                   # (B, Hkv, L, D)
        else:                                                                  # ragged (B, L, sum r_h)
            cols = [0]
            for rh in self.k_ranks():
                cols.append(cols[-1] + rh)
            k_full = torch.stack([torch.matmul(keys[..., cols[h]:cols[h + 1]], u.to(keys.dtype).T)
                                  for h, u in enumerate(self.k_u_heads())], dim=1)
        k_full = apply_rotary_pos_emb_custom(k_full, cos, sin)
        v_full = torch.matmul(values, self.v_proj.U.weight.T.to(values.dtype))
        v_full = v_full.view(B, -1, Hkv, D).transpose(1, 2)
        grp = self.num_key_value_groups
        k_full = k_full.repeat_interleave(grp, dim=1)
        v_full = v_full.repeat_interleave(grp, dim=1)
        mask = None if attention_mask is None else attention_mask[:, :, :, :k_full.shape[-2]]
        return F.scaled_dot_product_attention(q, k_full, v_full, attn_mask=mask, scale=self.scaling,
                                              is_causal=mask is None and Lq > 1)


class LlamaCustomAttentionQuant(LlamaCustomAttention):
    """The quantised module (quant.py:38-202): int8 per-channel K codes and int4
    per-token-group V codes in a ``StarKVCache(quantized=True)``.  The four cache
    arguments of the reference forward are accepted; ``past_key_values_upper``
    carries the ``StarKVCache`` (the others are unused: codes and scales live in
    the one cache object)."""

    quantized = True

    def forward(self, hidden_states, position_embeddings, attention_mask, position_ids=None,
                past_key_values_upper=None, past_key_values_lower=None, scales_upper=None, scales_lower=None,
                cache_position=None, **kwargs):
        cache = past_key_values_upper
        if cache is None:                                # called by transformers' decoder layer
            cache = kwargs.pop("past_key_values", None)
        if cache is not None and not isinstance(cache, StarKVCache):
            raise TypeError("the quantised module takes a StarKVCache(quantized=True) as past_key_values_upper")
        if cache is not None and not cache.quantized:
            raise ValueError("StarKVCache must be created with quantized=True for the quantised module")
        return super().forward(hidden_states, position_embeddings, attention_mask, position_ids,
                               past_key_values=cache, cache_position=cache_position)
