"""One compressed-KV attention layer's decode state on the GPU.

``DecodeLayer`` owns the latent cache, the packed K/V up-projections, the RoPE
table and the workspace of one layer, and runs the step the reference runs in
``LlamaCustomAttention.forward`` between the latent projections and ``o_proj``
(LlamaLoRaAttention_headwise.py:98-133, LlamaLoRaAttention_headwise_quant.py:107-186):

    append(new K/V latents)  ->  decode_attention(q_rot)  ->  (B, Hq, 128)
"""

from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence

import torch

from . import _lib, ops


def rope_inv_freq(theta: float, head_dim: int = 128, device=None) -> torch.Tensor:
    """HF default-rope inverse frequencies, computed with the same torch ops as
    ``LlamaRotaryEmbedding`` so the fp32 values are identical."""
    base = float(theta)
    inv = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.int64).to(dtype=torch.float) / head_dim))
    return inv.to(device=device, dtype=torch.float32).contiguous()


class DecodeLayer:
    FUSED_PROJECTION_MAX_BATCH = 8
    def __init__(self, layout, k_u: torch.Tensor, v_u: torch.Tensor, theta: float,
                 device=None):
        """k_u: packed K up-projections (sum_h 128*r_h elements, head h = (128, r_h));
        v_u: v_proj.U.weight (Hkv*128, R)."""
        self.layout = layout
        self.device = torch.device(device or k_u.device)
        self.cache = ops.LatentCache(layout, self.device)
        self.k_u = k_u.contiguous()
        self.v_u = v_u.contiguous()
        self.scaling = 128 ** -0.5
        self.inv_freq = rope_inv_freq(theta, 128, self.device)
        self.num_splits = 0

    @property
    def length(self) -> int:
        return self.cache.length

    def prefill(self, k_lat: torch.Tensor, v_lat: torch.Tensor):
        self.cache.prefill(k_lat.contiguous(), v_lat.contiguous())

    def append(self, k_lat: torch.Tensor, v_lat: torch.Tensor):
        self.cache.append(k_lat.contiguous(), v_lat.contiguous())

    def attend(self, q_rot: torch.Tensor, mask: Optional[torch.Tensor] = None,
               out: Optional[torch.Tensor] = None, events=None) -> torch.Tensor:
        """Attention of the (B, Hq, 128) rotated query over every filled slot."""
        T = self.cache.length
        return ops.decode_attention(self.layout, self.cache, q_rot.contiguous(), self.k_u, self.v_u,
                                    self.inv_freq, self.scaling, T, mask=None if mask is None else mask.contiguous(), out=out,
                                    num_splits=self.num_splits, events=events)

    def step_from_hidden(self, q_rot: torch.Tensor, hidden: torch.Tensor, vs_k: torch.Tensor, vs_v: torch.Tensor,
                         mask: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                         events=None) -> torch.Tensor:
        """Decode step from the token's hidden state, then attend.  Small batches use
        the fused latent projection + quantise-append kernel (``starkv_project_append``,
        VS rows read once); from ``FUSED_PROJECTION_MAX_BATCH + 1`` sequences on, the
        projection is two tensor-core GEMMs (cuBLAS) followed by ``starkv_append``, which
        is faster there (B=16 on c1 shapes: 36 us against 54 us for the CUDA-core kernel)."""
        if self.layout.batch <= self.FUSED_PROJECTION_MAX_BATCH:
            self.cache.project_append(hidden.contiguous(), vs_k.contiguous(), vs_v.contiguous())
        else:
            h = hidden.reshape(self.layout.batch, 1, -1)
            self.cache.append(torch.matmul(h, vs_k.T).contiguous(), torch.matmul(h, vs_v.T).contiguous())
        return self.attend(q_rot, mask=mask, out=out, events=events)

    def prepared_step(self, q_rot: torch.Tensor, hidden: torch.Tensor, vs_k: torch.Tensor, vs_v: torch.Tensor,
                      out: torch.Tensor):
        """``step_from_hidden`` bound once to fixed buffers, for loops that reuse
        the same tensors every step (e.g. between CUDA-graph replays): the C
        argument blocks, the stream and the workspace are built here, and the
        returned ``run()`` only sets the slot / token count and makes the two C
        calls (``starkv_project_append``, ``starkv_decode_attention``) on the
        stream current now.  Batches above ``FUSED_PROJECTION_MAX_BATCH`` use
        ``step_from_hidden`` as is."""
        if self.layout.batch > self.FUSED_PROJECTION_MAX_BATCH:
            return lambda: self.step_from_hidden(q_rot, hidden, vs_k, vs_v, out=out)
        L, c = self.layout, self.cache
        dt = c.latent_dtype
        H = hidden.shape[-1]
        ops._require(hidden, "hidden", dt, L.batch * H)
        ops._require(vs_k, "vs_k", dt, L.k_rank_total * H)
        ops._require(vs_v, "vs_v", dt, L.v_rank_total * H)
        ops._require(q_rot, "q", None, L.batch * L.num_q_heads * 128, align=4)
        ops._require(out, "out", None, L.batch * L.num_q_heads * 128, align=4)
        lib = _lib.load()
        stream = ops._stream()
        lay = C.byref(L)
        pa_head = (lay, ops._ptr(hidden), H, ops._ptr(vs_k), ops._ptr(vs_v))
        pa_tail = (ops._ptr(c.k_cache), ops._ptr(c.k_scales), ops._ptr(c.v_cache), ops._ptr(c.v_params), None, None,
                   stream)
        state = {}

        def bind(T):
            ws = ops.workspace(max(ops.workspace_size(L, min(L.capacity, T + 4096), self.num_splits),
                                   ops.workspace_size(L, T, self.num_splits)), q_rot.device)
            a = ops._decode_args(L, c, q_rot, self.k_u, self.v_u, self.inv_freq, self.scaling, T, None, out, ws,
                                 self.num_splits)
            state.update(ws=ws, a=a, ref=C.byref(a))

        bind(c.length + 1)

        def run():
            if c.length >= L.capacity:
                raise _lib.StarKVError("cache is full")
            _lib.check(lib.starkv_project_append(*pa_head, c.length, *pa_tail), "starkv_project_append")
            c.length += 1
            a = state["a"]
            a.num_tokens = c.length
            rc = lib.starkv_decode_attention(lay, state["ref"], stream)
            if rc == 4:                                  # workspace too small for this token count
                bind(c.length)
                rc = lib.starkv_decode_attention(lay, state["ref"], stream)
            _lib.check(rc, "starkv_decode_attention")
        return run

    def step(self, q_rot: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
             mask: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
             events=None) -> torch.Tensor:
        """Append the new token's latents (B, 1, sum r_h) / (B, 1, R), then attend."""
        self.append(k_new, v_new)
        return self.attend(q_rot, mask=mask, out=out, events=events)


def pack_k_u(k_u_heads: Sequence[torch.Tensor]) -> torch.Tensor:
    """Concatenate per-head (128, r_h) K up-projections into the packed layout."""
    return torch.cat([u.contiguous().reshape(-1) for u in k_u_heads])
