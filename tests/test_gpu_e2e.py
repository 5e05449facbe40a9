"""End-to-end greedy decode (``starkv.e2e``) on a tiny model: decoding with the
cache (fused projection + decode kernels per layer) must reproduce recomputing
the whole sequence through the prompt path (SDPA on the reconstructed keys and
values) at every step: same tokens, logits within rel-L2 2e-3."""

import numpy as np
import pytest
import torch

from starkv.attention import StarKVCache
from starkv.e2e import build_model, forward_tokens, generate, generate_graphed

pytestmark = pytest.mark.gpu


def test_e2e_cached_decode_matches_recompute(cuda):
    model = build_model(num_layers=2, hidden=512, heads=4, kv_heads=4, mlp=1024, vocab=1000, v_block_kv=2,
                        quantized=False, seed=3, device=cuda, max_positions=512)
    g = torch.Generator(device=cuda).manual_seed(1)
    prompt = torch.randint(0, 1000, (2, 37), generator=g, device=cuda)
    ids, _ = generate(model, prompt, 6)
    seq = prompt
    for s in range(6):
        ref = forward_tokens(model, seq, 0, StarKVCache(seq.shape[1] + 1, quantized=False))
        assert torch.equal(ref.argmax(-1), ids[:, s])
        if s == 5:
            cache = StarKVCache(seq.shape[1] + 1, quantized=False)
            forward_tokens(model, seq[:, :-1], 0, cache)
            got = forward_tokens(model, seq[:, -1:], seq.shape[1] - 1, cache).float().cpu().numpy()
            want = forward_tokens(model, seq, 0, StarKVCache(seq.shape[1] + 1, quantized=False)).float().cpu().numpy()
            assert np.linalg.norm(got - want) / np.linalg.norm(want) <= 2e-3
        seq = torch.cat([seq, ids[:, s:s + 1]], dim=1)


def test_e2e_quantized_runs_and_is_deterministic(cuda):
    model = build_model(num_layers=2, hidden=512, heads=4, kv_heads=4, mlp=1024, vocab=1000, v_block_kv=2,
                        quantized=True, seed=4, device=cuda, max_positions=512)
    g = torch.Generator(device=cuda).manual_seed(2)
    prompt = torch.randint(0, 1000, (1, 64), generator=g, device=cuda)
    a, _ = generate(model, prompt, 5)
    b, _ = generate(model, prompt, 5)
    assert torch.equal(a, b)


@pytest.mark.parametrize("quantized", [False, True])
def test_graphed_decode_matches_eager_decode(cuda, quantized):
    """The decode loop with each layer's dense work replayed from CUDA graphs
    (attention calls between the replays) generates the same tokens as the eager
    per-layer loop, over batch sizes on both sides of the fused-projection cutoff."""
    model = build_model(num_layers=3, hidden=512, heads=4, kv_heads=4, mlp=1024, vocab=1000, v_block_kv=2,
                        quantized=quantized, seed=7, device=cuda, max_positions=1024)
    g = torch.Generator(device=cuda).manual_seed(3)
    for B in (1, 9):
        prompt = torch.randint(0, 1000, (B, 150), generator=g, device=cuda)
        a, _ = generate(model, prompt, 12)
        b, _ = generate_graphed(model, prompt, 12)
        assert torch.equal(a, b)


@pytest.mark.parametrize("quantized", [False, True])
def test_transformers_forward_with_starkv_cache(cuda, quantized):
    """``LlamaForCausalLM.forward`` (transformers' own model code, as the
    reference's latency harness drives it, latency.py:69-99) with the drop-in
    modules and a ``StarKVCache`` passed as ``past_key_values``: the prompt and
    three decode steps give the same logits as the package's own per-layer loop
    (``forward_tokens``) on a separate cache, and the cache grows by one slot a step."""
    model = build_model(num_layers=2, hidden=512, heads=4, kv_heads=4, mlp=1024, vocab=1000, v_block_kv=2,
                        quantized=quantized, seed=5, device=cuda, max_positions=512)
    g = torch.Generator(device=cuda).manual_seed(3)
    prompt = torch.randint(0, 1000, (2, 29), generator=g, device=cuda)
    hf_cache = StarKVCache(64, quantized=quantized)
    own_cache = StarKVCache(64, quantized=quantized)
    with torch.no_grad():
        out = model(input_ids=prompt, past_key_values=hf_cache, use_cache=True)
        ref = forward_tokens(model, prompt, 0, own_cache)
        np.testing.assert_allclose(out.logits[:, -1].float().cpu().numpy(), ref.float().cpu().numpy(),
                                   rtol=1e-2, atol=1e-2)
        tok = ref.argmax(-1, keepdim=True)
        for s in range(3):
            out = model(input_ids=tok, past_key_values=hf_cache, use_cache=True)
            ref = forward_tokens(model, tok, prompt.shape[1] + s, own_cache)
            got, want = out.logits[:, -1].float().cpu().numpy(), ref.float().cpu().numpy()
            assert np.linalg.norm(got - want) / np.linalg.norm(want) <= 2e-3
            assert hf_cache.get_seq_length() == prompt.shape[1] + s + 1
            tok = ref.argmax(-1, keepdim=True)
