"""Inputs of the golden decode step, shared by tests/golden/make_golden.py (which
runs the reference module on them) and the drop-in module tests (which run
ours): hidden state and projection weights whose outputs are the synthetic
latents, and the prefilled cache contents the reference sees."""

import os
import sys

import numpy as np

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for _p in (os.path.join(_ROOT, "star-kv_b200"), os.path.join(_ROOT, "oracle")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import starkv_oracle as O  # noqa: E402


def build_module_inputs(spec, data, rng):
    """Hidden state and projection weights whose outputs are the synthetic latents.

    The new token's latents and the rotated query are set by choosing the
    projection weights as ``W = target * e_0^T`` with a one-hot hidden state, so
    that ``hidden @ W^T`` reproduces the synthetic values exactly."""
    B = spec.batch
    D = spec.head_dim
    hidden = spec.num_q_heads * D
    rmax = max(spec.k_ranks)
    # hidden_states[b] = e_b (one-hot over the first B coordinates)
    assert B <= hidden
    h = np.zeros((B, 1, hidden), dtype=np.float32)
    for b in range(B):
        h[b, 0, b] = 1.0
    T = spec.tokens
    # k_proj.VS rows: (Hkv*rmax, hidden), column b = new-token latent of sequence b
    vs_k = np.zeros((spec.num_kv_heads * rmax, hidden), dtype=np.float32)
    for kv, r in enumerate(spec.k_ranks):
        for b in range(B):
            vs_k[kv * rmax:kv * rmax + r, b] = data.xk[kv][b, T - 1, :]
    vs_v = np.zeros((spec.v_rank_total, hidden), dtype=np.float32)
    for b in range(B):
        vs_v[:, b] = data.xv[b, T - 1, :]
    # q_proj: rows give the *pre-RoPE* query; we want q_rot = data.q after RoPE at
    # position T-1, so feed the inverse rotation.
    inv = O.rope_inv_freq(spec.theta, D)
    cos, sin = O.rope_cos_sin(np.array([T - 1]), inv)
    q_pre = data.q * cos[0] - O.rotate_half(data.q) * sin[0]              # R^{-1} q
    wq = np.zeros((hidden, hidden), dtype=np.float32)
    for b in range(B):
        wq[:, b] = q_pre[b].reshape(-1)
    wo = (rng.standard_normal((hidden, hidden), dtype=np.float32) / np.sqrt(hidden)).astype(np.float32)
    k_u = np.zeros((spec.num_kv_heads, D, rmax), dtype=np.float32)
    for kv, r in enumerate(spec.k_ranks):
        k_u[kv, :, :r] = data.k_u[kv]
    return h, wq, vs_k, vs_v, k_u, wo



def prefill_cache(spec, data):
    """(B, Hkv, L, rmax) K latents (ragged ranks zero-padded) and (B, L, R) V latents
    of the prefilled cache; dequantised when the layer is quantised.  Also the
    (B, Hkv, rmax) fp16 K scales (None when unquantised)."""
    L, B = spec.context, spec.batch
    rmax = max(spec.k_ranks)
    if spec.quantized:
        qz = O.quantize_layer(data.xk, data.xv, L)
        xk_prev = [x[:, :L] for x in qz["xk_hat"]]
        xv_prev = qz["xv_hat"][:, :L]
        ks = np.ones((B, spec.num_kv_heads, rmax), dtype=np.float16)
        for kv, r in enumerate(spec.k_ranks):
            ks[:, kv, :r] = qz["k_scales"][kv]
    else:
        xk_prev = [x[:, :L] for x in data.xk]
        xv_prev = data.xv[:, :L]
        ks = None
    kprev = np.zeros((B, spec.num_kv_heads, L, rmax), dtype=np.float32)
    for kv, r in enumerate(spec.k_ranks):
        kprev[:, kv, :, :r] = xk_prev[kv]
    return kprev, np.ascontiguousarray(xv_prev, dtype=np.float32), ks


def module_inputs(spec, data):
    rng = np.random.default_rng(4242)
    h, wq, vs_k, vs_v, k_u, wo = build_module_inputs(spec, data, rng)
    kprev, vprev, _ = prefill_cache(spec, data)
    return h, wq, vs_k, vs_v, k_u, wo, kprev, vprev
