"""Ragged-rank export (``starkv.export``) against the reference's own export.

* Equal kept ranks: identical to ``model.export_kproj_for_triton`` (golden
  vectors made by the reference, ``tests/golden/make_export_golden.py``).
* Ragged kept ranks: the reference truncates every head to the smallest kept
  rank (model.py:319-321); its result must be the per-head prefix of ours.
* Zero padding to the kernel's rank granularity, the block-V export, and the
  drop-in module's prompt path with ragged heads (equal to a uniform module whose
  extra latent rows are zero)."""

import os

import numpy as np
import pytest
import torch
import torch.nn as nn

from starkv.export import export_kproj_ragged, export_vproj_blocks

from conftest import GOLDEN

G = np.load(os.path.join(GOLDEN, "export_k.npz"))


def _kstate(case):
    st = {"U.weight": torch.from_numpy(G["U"]), "V.weight": torch.from_numpy(G["V"])}
    for h in range(2):
        st[f"Sigma_blocks.{h}.diag"] = torch.from_numpy(G[f"{case}_diag{h}"])
        st[f"Sigma_blocks.{h}.soft_thres_layer.alpha"] = torch.tensor([float(G[f"{case}_alpha{h}"])])
    return st


def test_export_equal_ranks_matches_reference():
    k = export_kproj_ragged(_kstate("equal"), dtype=torch.float32)
    assert k.ranks == [32, 32]
    np.testing.assert_array_equal(k.VS.weight.numpy(), G["equal_VS"])
    np.testing.assert_array_equal(torch.stack(k.u_heads()).numpy(), G["equal_Uref"])


def test_export_ragged_ranks_extend_reference_prefix():
    k = export_kproj_ragged(_kstate("ragged"), dtype=torch.float32)
    assert k.ranks == [32, 16]
    ref_vs, ref_u = G["ragged_VS"], G["ragged_Uref"]          # truncated to min_r = 16
    m = ref_u.shape[-1]
    off = 0
    for h, u in enumerate(k.u_heads()):
        np.testing.assert_array_equal(u.numpy()[:, :m], ref_u[h])
        np.testing.assert_array_equal(k.VS.weight.numpy()[off:off + m], ref_vs[h * m:(h + 1) * m])
        off += k.ranks[h]


def test_export_pads_with_zeros():
    st = _kstate("ragged")
    d = st["Sigma_blocks.0.diag"]
    st["Sigma_blocks.0.soft_thres_layer.alpha"] = torch.tensor([float(d.sort(descending=True).values[20])])
    k = export_kproj_ragged(st, dtype=torch.float32)
    assert k.ranks == [32, 16]                                  # 20 kept -> 32
    u0 = k.u_heads()[0].numpy()
    assert np.all(u0[:, 20:] == 0) and np.all(k.VS.weight.numpy()[20:32] == 0)
    assert np.any(u0[:, 19] != 0)


def test_export_vproj_blocks_block_diagonal():
    torch.manual_seed(3)
    states, kvs = [], [1, 2]
    for nkv, r in zip(kvs, (40, 64)):
        diag = torch.rand(r) + 0.1
        states.append({"U.weight": torch.randn(nkv * 128, r), "V.weight": torch.randn(r, 48),
                       "Sigma.diag": diag, "Sigma.soft_thres_layer.alpha": torch.tensor([0.5])})
    v = export_vproj_blocks(states, kvs, dtype=torch.float32)
    assert v.ranks == [32 * ((int((s["Sigma.diag"] > 0.5).sum()) + 31) // 32) for s in states]
    U, VS = v.U.weight.numpy(), v.VS.weight.numpy()
    assert U.shape == (3 * 128, sum(v.ranks)) and VS.shape == (sum(v.ranks), 48)
    assert np.all(U[:128, v.ranks[0]:] == 0) and np.all(U[128:, :v.ranks[0]] == 0)
    keep = (states[0]["Sigma.diag"] > 0.5).nonzero().view(-1)
    s = states[0]["Sigma.diag"][keep] - 0.5
    np.testing.assert_allclose(VS[:len(keep)], (states[0]["V.weight"][keep] * s[:, None]).numpy(), rtol=0, atol=0)
    np.testing.assert_allclose(U[:128, :len(keep)], states[0]["U.weight"][:, keep].numpy(), rtol=0, atol=0)


def test_dropin_prompt_with_ragged_heads_equals_padded_uniform():
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding

    import LlamaLoRaAttention_headwise as mine
    cfg = LlamaConfig(hidden_size=256, num_attention_heads=2, num_key_value_heads=2, intermediate_size=512,
                      max_position_embeddings=64, attention_bias=False, head_dim=128)
    torch.manual_seed(5)
    k = export_kproj_ragged(_kstate("ragged"), dtype=torch.float32)
    hidden = torch.randn(1, 6, 256)
    vs_k = torch.randn(sum(k.ranks), 256) / 16                   # a K latent projection with ragged heads
    k.VS.weight = nn.Parameter(vs_k)
    v = export_vproj_blocks([{"U.weight": torch.randn(256, 64), "V.weight": torch.randn(64, 256) / 16,
                              "Sigma.diag": torch.rand(64) + 1, "Sigma.soft_thres_layer.alpha": torch.tensor([0.])}],
                            [2], dtype=torch.float32)
    a = mine.LlamaCustomAttention(cfg, layer_idx=0, decomp_goup_num=2)
    a.k_proj, a.v_proj = k, v
    # the same projection with uniform rank 32: head 1 padded by zero latents
    b = mine.LlamaCustomAttention(cfg, layer_idx=0, decomp_goup_num=2)
    b.load_state_dict({n: t for n, t in a.state_dict().items() if n.startswith(("q_proj", "o_proj"))}, strict=False)
    kp = nn.Module()
    vs_pad = torch.zeros(64, 256)
    vs_pad[:32] = vs_k[:32]
    vs_pad[32:48] = vs_k[32:48]
    kp.VS = nn.Linear(256, 64, bias=False)
    kp.VS.weight = nn.Parameter(vs_pad)
    u1 = torch.zeros(128, 32)
    u1[:, :16] = k.u_heads()[1]
    kp.register_buffer("U", torch.stack([k.u_heads()[0], u1]))
    b.k_proj, b.v_proj = kp, v
    rope = LlamaRotaryEmbedding(cfg)
    pos = torch.arange(6)[None]
    cos, sin = rope(hidden, pos)
    with torch.no_grad():
        oa, _ = a(hidden, (cos, sin), None)
        ob, _ = b(hidden, (cos, sin), None)
    np.testing.assert_allclose(oa.numpy(), ob.numpy(), rtol=1e-5, atol=1e-5)


def _ragged_and_padded(cfg):
    import LlamaLoRaAttention_headwise as mine
    torch.manual_seed(7)
    k = export_kproj_ragged(_kstate("ragged"), dtype=torch.float32)
    vs_k = torch.randn(sum(k.ranks), 256) / 16
    k.VS.weight = nn.Parameter(vs_k)
    v = export_vproj_blocks([{"U.weight": torch.randn(256, 64), "V.weight": torch.randn(64, 256) / 16,
                              "Sigma.diag": torch.rand(64) + 1, "Sigma.soft_thres_layer.alpha": torch.tensor([0.])}],
                            [2], dtype=torch.float32)
    a = mine.LlamaCustomAttention(cfg, layer_idx=0, decomp_goup_num=2)
    a.k_proj, a.v_proj = k, v
    b = mine.LlamaCustomAttention(cfg, layer_idx=0, decomp_goup_num=2)
    b.load_state_dict({n: t for n, t in a.state_dict().items() if n.startswith(("q_proj", "o_proj"))}, strict=False)
    kp = nn.Module()
    vs_pad = torch.zeros(64, 256)
    vs_pad[:48] = vs_k
    kp.VS = nn.Linear(256, 64, bias=False)
    kp.VS.weight = nn.Parameter(vs_pad)
    u1 = torch.zeros(128, 32)
    u1[:, :16] = k.u_heads()[1]
    kp.register_buffer("U", torch.stack([k.u_heads()[0], u1]))
    b.k_proj, b.v_proj = kp, v
    return a, b


@pytest.mark.gpu
def test_dropin_decode_with_ragged_heads_equals_padded_uniform(cuda):
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding

    from starkv.attention import StarKVCache
    cfg = LlamaConfig(hidden_size=256, num_attention_heads=2, num_key_value_heads=2, intermediate_size=512,
                      max_position_embeddings=512, attention_bias=False, head_dim=128)
    a, b = _ragged_and_padded(cfg)
    a, b = a.cuda().half(), b.cuda().half()
    rope = LlamaRotaryEmbedding(cfg).cuda()
    torch.manual_seed(9)
    hidden = torch.randn(2, 200, 256, device="cuda").half()
    outs = []
    for mod in (a, b):
        cache = StarKVCache(capacity=256)
        pos = torch.arange(199, device="cuda")[None]
        cos, sin = rope(hidden[:, :199], pos)
        with torch.no_grad():
            mod(hidden[:, :199], (cos.half(), sin.half()), None, past_key_values=cache)
            cos, sin = rope(hidden[:, 199:], pos[:, -1:] + 1)
            o, _ = mod(hidden[:, 199:], (cos.half(), sin.half()), None, past_key_values=cache)
        outs.append(o.float().cpu().numpy())
    err = np.linalg.norm(outs[0] - outs[1]) / np.linalg.norm(outs[1])
    assert err <= 2e-3 and np.abs(outs[0] - outs[1]).max() <= 1e-2, err
