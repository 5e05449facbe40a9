"""CPU oracle for the STAR-KV compressed-KV decode-attention step.

TEST INFRASTRUCTURE ONLY.  Nothing in the product path imports this module:
only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` may use it, and only as the checker / the timed CPU baseline.

It restates, in numpy, the reference's eager decode path
(PriyanshBhatnagar/STAR-KV):

* ``LlamaLoRaAttention_headwise.py:98-146`` — latent append, K reconstruction
  ``X_k @ U^T`` (:108), RoPE of the reconstructed keys (:109), ``q.k * scaling``
  (:110), additive mask (:117-119), fp32 softmax (:121), the ``reorder`` branch
  ``P @ X_v`` then the per-head ``U_v`` up-projection (:126-133);
* ``model.py:450-487`` — the same decode branch with the GQA repeat of the
  K heads (:476) and of ``v_u`` (:485-486);
* ``LlamaLoRaAttention_headwise.py:22-29`` — ``apply_rotary_pos_emb_custom``,
  used with full-range cos/sin tables (positions ``0..L``), and the HF
  ``LlamaRotaryEmbedding`` default tables it is fed with;
* the latent quantiser that the reference imports as
  ``quant_utils.quantize_r_split_int8_int4_packed`` (call sites
  ``LlamaLoRaAttention_headwise_quant.py:107-117,138-139,164-165``,
  ``bx_quant.py:75-86`` for the nibble order).  That module is absent from the
  reference tree, so the quantiser arithmetic below is the stated specification
  (parity unpinned against reference code; pinned by the golden vectors this
  repository generates from it):

  - K: int8 symmetric, one fp16 scale per (sequence, KV head, latent channel):
    ``s = fp16(absmax / 127)`` (``s = 1`` where that is 0),
    ``q = clamp(rint(x / float(s)), -127, 127)``; the scales are computed once
    over the prefilled latents and reused for appended tokens.
  - V: int4 asymmetric, groups of 32 consecutive latent channels of one token:
    ``s = fp16((max - min) / 15)`` (``s = 1`` where that is 0),
    ``z = fp16(min)``, ``q = clamp(rint((x - float(z)) / float(s)), 0, 15)``,
    ``x_hat = q * s + z``; two codes per byte, even channel in the low nibble.
  - All arithmetic is IEEE fp32 with round-to-nearest-even.

Ragged per-head K ranks and block-wise V ranks are the generalisation the
B200 build supports; on the reference layout they are the zero-padded K
latents and a block-diagonal ``v_proj.U`` (exact: the padding contributes 0).
"""

from __future__ import annotations

import numpy as np

F32 = np.float32


# ---------------------------------------------------------------------------
# RoPE (HF LlamaRotaryEmbedding default rope + headwise.py:22-29)
# ---------------------------------------------------------------------------

def rope_inv_freq(theta: float, head_dim: int = 128) -> np.ndarray:
    """inv_freq_i = 1 / theta^(2i/d), fp32 (HF default rope initialisation)."""
    exps = (np.arange(0, head_dim, 2, dtype=np.int64).astype(F32) / F32(head_dim)).astype(F32)
    return (F32(1.0) / np.power(F32(theta), exps, dtype=F32)).astype(F32)


def rope_cos_sin(positions: np.ndarray, inv_freq: np.ndarray):
    """cos/sin tables (N, d) as HF builds them: fp32 angle = fl(pos * inv_freq),
    ``emb = cat(freqs, freqs)``, then cos/sin in fp32."""
    ang = (positions.astype(F32)[:, None] * inv_freq[None, :].astype(F32)).astype(F32)
    emb = np.concatenate([ang, ang], axis=-1)
    return np.cos(emb).astype(F32), np.sin(emb).astype(F32)


def rotate_half(x: np.ndarray) -> np.ndarray:
    h = x.shape[-1] // 2
    return np.concatenate([-x[..., h:], x[..., :h]], axis=-1)


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """headwise.py:28 — ``x * cos + rotate_half(x) * sin`` (full-range tables)."""
    return x * cos + rotate_half(x) * sin


# ---------------------------------------------------------------------------
# Quantiser (spec restated; reference module quant_utils is absent)
# ---------------------------------------------------------------------------

def quantize_k_scales(x: np.ndarray) -> np.ndarray:
    """Per-channel symmetric int8 scales over the token axis.

    x: (..., T, r) float -> (..., r) float16.
    """
    x = x.astype(F32)
    amax = np.max(np.abs(x), axis=-2).astype(F32)
    s = (amax / F32(127.0)).astype(F32).astype(np.float16)
    s[s == 0] = np.float16(1.0)
    return s


def quantize_k_codes(x: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """x: (..., T, r), scales (..., r) fp16 -> int8 codes (..., T, r)."""
    s = scales.astype(F32)[..., None, :]
    q = np.rint((x.astype(F32) / s).astype(F32))
    return np.clip(q, -127, 127).astype(np.int8)


def dequant_k(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    return codes.astype(F32) * scales.astype(F32)[..., None, :]


def quantize_v(x: np.ndarray):
    """x: (..., R) float, R % 32 == 0 -> (codes uint8 (..., R/2), scale f16 (..., R/32),
    zero f16 (..., R/32))."""
    x = x.astype(F32)
    R = x.shape[-1]
    assert R % 32 == 0
    g = x.reshape(*x.shape[:-1], R // 32, 32)
    mn = g.min(axis=-1)
    mx = g.max(axis=-1)
    s = ((mx - mn).astype(F32) / F32(15.0)).astype(F32).astype(np.float16)
    s[s == 0] = np.float16(1.0)
    z = mn.astype(np.float16)
    q = np.rint(((g - z.astype(F32)[..., None]).astype(F32) / s.astype(F32)[..., None]).astype(F32))
    q = np.clip(q, 0, 15).astype(np.uint8).reshape(*x.shape[:-1], R)
    packed = (q[..., 0::2] | (q[..., 1::2] << 4)).astype(np.uint8)
    return packed, s, z


def unpack_v_codes(packed: np.ndarray) -> np.ndarray:
    lo = packed & 0x0F
    hi = (packed >> 4) & 0x0F
    out = np.empty(packed.shape[:-1] + (packed.shape[-1] * 2,), dtype=np.uint8)
    out[..., 0::2] = lo
    out[..., 1::2] = hi
    return out


def dequant_v(packed: np.ndarray, scale: np.ndarray, zero: np.ndarray) -> np.ndarray:
    q = unpack_v_codes(packed).astype(F32)
    R = q.shape[-1]
    g = q.reshape(*q.shape[:-1], R // 32, 32)
    x = g * scale.astype(F32)[..., None] + zero.astype(F32)[..., None]
    return x.reshape(*q.shape[:-1], R).astype(F32)


# ---------------------------------------------------------------------------
# Split quantiser of the reference's quantised module (quant_utils interface,
# call sites LlamaLoRaAttention_headwise_quant.py:107-117, 137-140, 164-165;
# dequantisation (nib - 8) * scale as bx_quant.py:75-86).  Specification (the
# module is absent from the reference): per row, ranks [0, split_r) int8 with
# s = fp16(absmax / 127), the rest signed int4 with s = fp16(absmax / 7),
# q = clamp(rint(x / s)), nibble q + 8, even rank in the low nibble; zero rows
# get s = 1.
# ---------------------------------------------------------------------------

def quantize_split(x: np.ndarray, split_r: int):
    x = x.astype(F32)
    r = x.shape[-1]
    r4 = r - split_r

    def scale(part, qmax):
        s = (np.max(np.abs(part), axis=-1, keepdims=True).astype(F32) / F32(qmax)).astype(F32).astype(np.float16)
        s[s == 0] = np.float16(1.0)
        return s

    up, lo = x[..., :split_r], x[..., split_r:]
    s_up = scale(up, 127.0) if split_r else np.ones(x.shape[:-1] + (1,), np.float16)
    s_lo = scale(lo, 7.0) if r4 else np.ones(x.shape[:-1] + (1,), np.float16)
    up_q = np.clip(np.rint((up / s_up.astype(F32)).astype(F32)), -127, 127).astype(np.int8)
    q = np.clip(np.rint((lo / s_lo.astype(F32)).astype(F32)), -8, 7).astype(np.int16) + 8
    if r4 % 2:
        q = np.concatenate([q, np.zeros(q.shape[:-1] + (1,), q.dtype)], axis=-1)
    lo_q = (q[..., 0::2] | (q[..., 1::2] << 4)).astype(np.uint8)
    return up_q, s_up, lo_q, s_lo, r4


def unpack_int4_signed(q: np.ndarray, r: int) -> np.ndarray:
    out = np.empty(q.shape[:-1] + (2 * q.shape[-1],), dtype=np.int8)
    out[..., 0::2] = (q & 0x0F).astype(np.int8) - 8
    out[..., 1::2] = ((q >> 4) & 0x0F).astype(np.int8) - 8
    return out[..., :r]


# ---------------------------------------------------------------------------
# Decode attention (headwise.py:98-146 reorder branch; model.py:450-487 GQA)
# ---------------------------------------------------------------------------

def decode_attention(q_rot, xk, k_u, xv, v_u_weight, k_ranks, v_ranks, v_block_of_kv,
                     inv_freq, scaling, mask=None, dtype=np.float64):
    """One decode step of compressed-KV attention, per-head outputs before o_proj.

    q_rot:      (B, Hq, 128) rotated query (headwise.py:105).
    xk:         list over KV heads of (B, L, r_h) dequantised K latents.
    k_u:        list over KV heads of (128, r_h) — ``k_proj.U[h]`` (model.py:318-324).
    xv:         (B, L, sum r_b) dequantised V latents, blocks concatenated.
    v_u_weight: (Hkv*128, sum r_b) — ``v_proj.U.weight`` (model.py:348-356),
                block-diagonal for block-wise V.
    v_block_of_kv: block index of each KV head.
    Returns (B, Hq, 128) in ``dtype``.
    """
    B, Hq, D = q_rot.shape
    Hkv = len(xk)
    grp = Hq // Hkv
    L = xk[0].shape[1]
    cos, sin = rope_cos_sin(np.arange(L), inv_freq)
    cos = cos.astype(dtype)
    sin = sin.astype(dtype)
    vcol = np.concatenate([[0], np.cumsum(v_ranks)]).astype(np.int64)
    out = np.zeros((B, Hq, D), dtype=dtype)
    for kv in range(Hkv):
        # headwise.py:108-109: key = X_k @ U^T, then RoPE at positions 0..L-1
        keys = np.matmul(xk[kv].astype(dtype), k_u[kv].astype(dtype).T)      # (B, L, 128)
        keys = apply_rope(keys, cos[None], sin[None])
        j = v_block_of_kv[kv]
        xv_j = xv[:, :, vcol[j]:vcol[j + 1]].astype(dtype)                    # (B, L, r_b)
        u_h = v_u_weight[kv * D:(kv + 1) * D, vcol[j]:vcol[j + 1]].astype(dtype)  # (128, r_b)
        for g in range(grp):
            h = kv * grp + g
            q = q_rot[:, h, :].astype(dtype)                                  # (B, 128)
            logits = np.einsum("bld,bd->bl", keys, q) * dtype(scaling)        # :110
            if mask is not None:
                logits = logits + mask.astype(dtype)                          # :117-119
            m = logits.max(axis=-1, keepdims=True)
            p = np.exp(logits - m)
            p = p / p.sum(axis=-1, keepdims=True)                             # :121
            o_lat = np.einsum("bl,blr->br", p, xv_j)                          # :127
            out[:, h, :] = o_lat @ u_h.T                                      # :128-130
    return out

def prompt_attention(q_rot, xk, k_u, xv, v_u_weight, k_ranks, v_ranks, v_block_of_kv,
                     inv_freq, scaling, dtype=np.float64):
    """Causal prompt (prefill) attention over K / V rebuilt from unquantised latents.

    Restates the reference's prefill branch (model.py:429-449): key_full =
    RoPE(X_k @ U_k^T) at positions 0..T-1 (:431-432), GQA repeat of the K / V heads
    (:436, :442), value_full = X_v @ v_proj.U.weight^T split into heads (:437-441),
    then softmax(q k^T * scaling) v with query t attending to keys 0..t (SDPA with
    the model's causal mask, :443-449).

    q_rot: (B, Hq, T, 128) rotated queries; xk: list over KV heads of (B, T, r_h);
    k_u: list of (128, r_h); xv: (B, T, sum r_b); v_u_weight (Hkv*128, sum r_b).
    Returns (B, Hq, T, 128) in ``dtype``.
    """
    B, Hq, T, D = q_rot.shape
    Hkv = len(xk)
    grp = Hq // Hkv
    cos, sin = rope_cos_sin(np.arange(T), inv_freq)
    cos, sin = cos.astype(dtype), sin.astype(dtype)
    vcol = np.concatenate([[0], np.cumsum(v_ranks)]).astype(np.int64)
    causal = np.tril(np.ones((T, T), dtype=bool))
    out = np.zeros((B, Hq, T, D), dtype=dtype)
    for kv in range(Hkv):
        keys = apply_rope(np.matmul(xk[kv].astype(dtype), k_u[kv].astype(dtype).T), cos[None], sin[None])
        j = v_block_of_kv[kv]
        vals = np.matmul(xv[:, :, vcol[j]:vcol[j + 1]].astype(dtype),
                         v_u_weight[kv * D:(kv + 1) * D, vcol[j]:vcol[j + 1]].astype(dtype).T)   # (B, T, 128)
        for g in range(grp):
            h = kv * grp + g
            logits = np.matmul(q_rot[:, h].astype(dtype), keys.transpose(0, 2, 1)) * dtype(scaling)
            logits = np.where(causal[None], logits, -np.inf)
            logits -= logits.max(axis=-1, keepdims=True)
            p = np.exp(logits)
            p /= p.sum(axis=-1, keepdims=True)
            out[:, h] = np.matmul(p, vals)
    return out



def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


# ---------------------------------------------------------------------------
# One decode step on a quantised latent cache
# ---------------------------------------------------------------------------

def quantize_layer(xk, xv, context):
    """Quantise a layer's latents the way the cache sees them at one decode step.

    xk: list over KV heads of (B, T, r_h) float; xv: (B, T, R).  Tokens
    ``0..context-1`` are the prefill (their K latents fix the per-channel
    scales); token ``context`` is the appended one, quantised with those scales.
    Returns dict with ``k_scales`` (list of (B, r_h) f16), ``k_codes`` (list of
    (B, T, r_h) int8), ``v_codes`` (B, T, R/2), ``v_scale``/``v_zero`` (B, T, R/32)
    and the dequantised ``xk_hat`` / ``xv_hat``.
    """
    k_scales = [quantize_k_scales(x[:, :context, :]) for x in xk]
    k_codes = [quantize_k_codes(x, s) for x, s in zip(xk, k_scales)]
    v_codes, v_scale, v_zero = quantize_v(xv)
    return dict(
        k_scales=k_scales, k_codes=k_codes, v_codes=v_codes, v_scale=v_scale, v_zero=v_zero,
        xk_hat=[dequant_k(c, s) for c, s in zip(k_codes, k_scales)],
        xv_hat=dequant_v(v_codes, v_scale, v_zero))


def layer_reference(data, dtype=np.float64):
    """Per-head outputs (B, Hq, 128) of one decode step of a synthetic layer
    (``starkv.synthetic.LayerData``), on the quantised cache when the layer is
    quantised."""
    spec = data.spec
    if spec.quantized:
        qz = quantize_layer(data.xk, data.xv, spec.context)
        xk, xv = qz["xk_hat"], qz["xv_hat"]
    else:
        xk, xv = data.xk, data.xv
    return decode_attention(
        data.q, xk, data.k_u, xv, data.v_u, spec.k_ranks, spec.v_ranks,
        spec.v_block_of_kv(), rope_inv_freq(spec.theta, spec.head_dim),
        spec.head_dim ** -0.5, mask=data.mask, dtype=dtype)
