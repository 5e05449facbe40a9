"""The drop-in modules and kernel shims against the reference.

* ``LlamaLoRaAttention_headwise.LlamaCustomAttention`` (ours) with an HF
  ``DynamicCache``, built exactly like the golden generator builds the
  reference module, must reproduce the reference's module output (after
  ``o_proj``) stored in the golden vectors.
* The quantised module with a ``StarKVCache`` (prompt + decode through the
  module's forward) against the oracle on the quantised cache.
* ``abx_rope_batched.abx`` (ours) against the oracle logits."""

import json
import os

import numpy as np
import pytest
import torch
import torch.nn as nn

import starkv_oracle as O
from starkv.synthetic import make_layer, make_spec

from conftest import GOLDEN

pytestmark = pytest.mark.gpu
REL_L2, MAX_ABS = 2e-3, 1e-2
MANIFEST = json.load(open(os.path.join(GOLDEN, "manifest.json")))


def _config(spec):
    from transformers import LlamaConfig
    hidden = spec.num_q_heads * spec.head_dim
    return LlamaConfig(hidden_size=hidden, num_attention_heads=spec.num_q_heads, num_key_value_heads=spec.num_kv_heads,
                       intermediate_size=4 * hidden, rope_theta=spec.theta,
                       max_position_embeddings=max(4096, spec.tokens + 1), attention_bias=False, head_dim=128)


def _attach(mod, vs_k, k_u, vs_v, v_u):
    kp = nn.Module()
    kp.VS = nn.Linear(vs_k.shape[1], vs_k.shape[0], bias=False)
    kp.VS.weight = nn.Parameter(torch.from_numpy(vs_k))
    kp.register_buffer("U", torch.from_numpy(k_u))
    vp = nn.Module()
    vp.VS = nn.Linear(vs_v.shape[1], vs_v.shape[0], bias=False)
    vp.VS.weight = nn.Parameter(torch.from_numpy(vs_v))
    vp.U = nn.Linear(v_u.shape[1], v_u.shape[0], bias=False)
    vp.U.weight = nn.Parameter(torch.from_numpy(v_u))
    mod.k_proj, mod.v_proj = kp, vp


# Quantised golden cases quantise the appended token inside the reference's
# cache; a plain DynamicCache does not, so those are covered by the StarKVCache
# test below instead.
@pytest.mark.parametrize("name", sorted(n for n, m in MANIFEST.items() if m["config"] == "c0"))
def test_dropin_module_matches_reference_golden(cuda, name):
    from transformers import DynamicCache
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding

    import LlamaLoRaAttention_headwise as mine
    from golden_inputs import module_inputs

    m = MANIFEST[name]
    spec = make_spec(m["config"], seed=0, **m["overrides"])
    data = make_layer(spec, with_mask=m["with_mask"])
    h, wq, vs_k, vs_v, k_u, wo, kprev, vprev = module_inputs(spec, data)
    config = _config(spec)
    mod = mine.LlamaCustomAttention(config, layer_idx=0, decomp_goup_num=spec.num_q_heads)
    with torch.no_grad():
        mod.q_proj.weight.copy_(torch.from_numpy(wq))
        mod.o_proj.weight.copy_(torch.from_numpy(wo))
    _attach(mod, vs_k, k_u, vs_v, data.v_u)
    mod = mod.to(cuda).float().eval()
    cache = DynamicCache()
    cache.update(torch.from_numpy(kprev).to(cuda), torch.from_numpy(vprev).to(cuda), 0)
    B = spec.batch
    pos = torch.arange(spec.tokens, device=cuda).unsqueeze(0).expand(B, -1)
    x = torch.from_numpy(h).to(cuda)
    cos, sin = LlamaRotaryEmbedding(config=config).to(cuda)(x, pos)
    mask = None
    if data.mask is not None:
        mask = torch.from_numpy(data.mask).to(cuda)[:, None, None, :]
    with torch.no_grad():
        out, _ = mod(x, (cos, sin), mask, pos[:, -1:], past_key_values=cache)
    got = out.reshape(B, -1).cpu().numpy()
    gold = np.load(os.path.join(GOLDEN, f"{name}.npz"))["out"]
    assert O.rel_l2(got, gold) <= REL_L2
    assert np.abs(got - gold).max() <= MAX_ABS


def test_quantised_module_prompt_then_decode(cuda):
    """Prompt through forward (quantise-prefill into the StarKVCache), then three
    decode steps; each step against the oracle on the quantised cache."""
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding

    import LlamaLoRaAttention_headwise_quant as q_mod

    spec = make_spec("c1", seed=31, num_q_heads=8, batch=2, context=300)
    config = _config(spec)
    rng = np.random.default_rng(5)
    hidden, H, D, r, rv = config.hidden_size, spec.num_q_heads, 128, 64, 256
    mod = q_mod.LlamaCustomAttention(config, layer_idx=3, decomp_goup_num=H)
    f = lambda *s: rng.standard_normal(s, dtype=np.float32)
    with torch.no_grad():
        mod.q_proj.weight.copy_(torch.from_numpy(f(hidden, hidden) / np.sqrt(hidden)))
        mod.o_proj.weight.copy_(torch.from_numpy(f(hidden, hidden) / np.sqrt(hidden)))
    vs_k, k_u = f(H * r, hidden) / np.sqrt(hidden), f(H, D, r) / np.sqrt(r)
    vs_v, v_u = f(rv, hidden) / np.sqrt(hidden), f(H * D, rv) / np.sqrt(rv)
    _attach(mod, vs_k, k_u, vs_v, v_u)
    mod = mod.to(cuda).half().eval()
    cache = q_mod.StarKVCache(capacity=spec.context + 8, quantized=True)
    B, L = spec.batch, spec.context
    hs = torch.from_numpy(f(B, L + 3, hidden)).to(cuda).half()
    rope = LlamaRotaryEmbedding(config=config).to(cuda)
    pos = torch.arange(L + 3, device=cuda).unsqueeze(0).expand(B, -1)
    cos, sin = rope(hs, pos)
    with torch.no_grad():
        mod(hs[:, :L], (cos[:, :L], sin[:, :L]), None, pos[:, :L], past_key_values_upper=cache)
    # oracle on fp32 copies of the same latents
    with torch.no_grad():
        lat_k = (hs.float() @ mod.k_proj.VS.weight.float().T).cpu().numpy()    # (B, L+3, H*r)
        lat_v = (hs.float() @ mod.v_proj.VS.weight.float().T).cpu().numpy()
    lat_k = lat_k.astype(np.float16).astype(np.float32)
    lat_v = lat_v.astype(np.float16).astype(np.float32)
    qz_scales = [O.quantize_k_scales(lat_k[:, :L, h * r:(h + 1) * r]) for h in range(H)]
    for step in range(3):
        T = L + step + 1
        with torch.no_grad():
            out, _ = mod(hs[:, T - 1:T], (cos[:, :T], sin[:, :T]), None, pos[:, T - 1:T],
                         past_key_values_upper=cache)
        with torch.no_grad():
            qrot = mod.q_proj(hs[:, T - 1:T]).view(B, 1, H, D).transpose(1, 2).float()
            c_, s_ = cos[:, T - 1:T].float()[:, None], sin[:, T - 1:T].float()[:, None]
            qrot = (qrot * c_ + torch.cat([-qrot[..., 64:], qrot[..., :64]], -1) * s_)[:, :, 0].cpu().numpy()
        xk = [O.dequant_k(O.quantize_k_codes(lat_k[:, :T, h * r:(h + 1) * r], qz_scales[h]), qz_scales[h])
              for h in range(H)]
        c, sc, z = O.quantize_v(lat_v[:, :T])
        attn = O.decode_attention(qrot, xk, [k_u[h].astype(np.float16).astype(np.float32) for h in range(H)],
                                  O.dequant_v(c, sc, z), v_u.astype(np.float16).astype(np.float32), [r] * H, [rv],
                                  [0] * H, O.rope_inv_freq(spec.theta), 128 ** -0.5)
        ref = attn.reshape(B, 1, H * D) @ mod.o_proj.weight.detach().float().cpu().numpy().T
        got = out.float().cpu().numpy()
        assert O.rel_l2(got, ref) <= REL_L2, step
    assert cache.get_seq_length(3) == L + 3


def test_abx_shim_matches_oracle(cuda):
    import abx_rope_batched as shim
    rng = np.random.default_rng(8)
    B, Hq, Hkv, L, r = 2, 8, 4, 777, 48
    a = rng.standard_normal((B, Hq, 1, 128), dtype=np.float32)
    b = (rng.standard_normal((Hkv, r, 128), dtype=np.float32) / np.sqrt(r))
    x = rng.standard_normal((B, Hkv, L, r), dtype=np.float32)
    to = lambda t: torch.from_numpy(t).to(cuda).half()
    got = shim.abx(to(a), to(b), to(x)).float().cpu().numpy()[:, :, 0]
    a16, b16, x16 = (t.astype(np.float16).astype(np.float64) for t in (a, b, x))
    cos, sin = O.rope_cos_sin(np.arange(L), O.rope_inv_freq(1e4))
    for h in range(Hq):
        kv = h // (Hq // Hkv)
        keys = O.apply_rope(x16[:, kv] @ b16[kv], cos, sin)
        ref = np.einsum("bld,bd->bl", keys, a16[:, h, 0])
        assert O.rel_l2(got[:, h], ref) <= REL_L2
