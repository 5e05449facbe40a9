"""End-to-end greedy decode with STAR-KV attention in every layer (config c3).

A Llama-2-7B-shaped model (32 layers, hidden 4096, 32 heads, MLP 11008, vocab
32000) with random-init fp16 weights whose attention modules are the drop-in
``LlamaCustomAttentionQuant`` (int8 K / int4 V latent cache) or
``LlamaCustomAttention``: per layer, K ranks per KV head and V block ranks are
drawn from a seed (default average K rank 32 of {16, 32, 48}, V blocks of 4 KV
heads with ranks in {64, 128, 192}), K heads ragged (``starkv.export``).

The prompt goes through the modules' prompt path (latents stored in the
``StarKVCache``, keys/values rebuilt from the latents as the reference's prefill
does, model.py:429-449, causal attention by the library's tcgen05 prefill kernel); every generated token goes through
the fused decode path per layer: ``starkv_project_append`` (latent projection +
quantise-append) and ``starkv_decode_attention``.  The rest of each layer (norms,
MLP, embeddings, LM head) is the transformers Llama code.

    python -m starkv.e2e --context 4096 --new 128 [--layers 32] [--unquantized]

prints one JSON line: decode tokens/s (batch 1) and ms per generated token.
"""

from __future__ import annotations

import argparse
import json
import time
from typing import List, Optional, Sequence

import numpy as np
import torch

from .attention import LlamaCustomAttention, LlamaCustomAttentionQuant, StarKVCache
from .export import BlockVProj, RaggedKProj


def build_model(num_layers: int = 32, hidden: int = 4096, heads: int = 32, kv_heads: int = 32, mlp: int = 11008,
                vocab: int = 32000, k_rank_choices: Sequence[int] = (16, 32, 48),
                v_rank_choices: Sequence[int] = (64, 128, 192), v_block_kv: int = 4, quantized: bool = True,
                seed: int = 0, device="cuda", dtype=torch.float16, max_positions: int = 131072 + 256):
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(hidden_size=hidden, num_attention_heads=heads, num_key_value_heads=kv_heads,
                      intermediate_size=mlp, vocab_size=vocab, num_hidden_layers=num_layers,
                      max_position_embeddings=max_positions, attention_bias=False, head_dim=128)
    torch.manual_seed(seed)
    with torch.device(device):
        model = LlamaForCausalLM(cfg).to(dtype).eval()
    rng = np.random.default_rng(seed)
    g = torch.Generator(device=device).manual_seed(seed)
    cls = LlamaCustomAttentionQuant if quantized else LlamaCustomAttention
    for i, layer in enumerate(model.model.layers):
        attn = cls(cfg, layer_idx=i, decomp_goup_num=heads)
        attn.q_proj, attn.o_proj = layer.self_attn.q_proj, layer.self_attn.o_proj
        ranks = [int(x) for x in rng.choice(k_rank_choices, size=kv_heads)]
        vs_k = (torch.randn(sum(ranks), hidden, generator=g, device=device) * 0.02).to(dtype)
        u_heads = [(torch.randn(128, r, generator=g, device=device) / r ** 0.5).to(dtype) for r in ranks]
        attn.k_proj = RaggedKProj(vs_k, u_heads)
        nb = kv_heads // v_block_kv
        vr = [int(x) for x in rng.choice(v_rank_choices, size=nb)]
        vs_v = (torch.randn(sum(vr), hidden, generator=g, device=device) * 0.02).to(dtype)
        U = torch.zeros(kv_heads * 128, sum(vr), device=device, dtype=dtype)
        c0 = 0
        for j, r in enumerate(vr):
            rows = slice(j * v_block_kv * 128, (j + 1) * v_block_kv * 128)
            U[rows, c0:c0 + r] = (torch.randn(v_block_kv * 128, r, generator=g, device=device) / r ** 0.5).to(dtype)
            c0 += r
        attn.v_proj = BlockVProj(vs_v, U, vr, [v_block_kv] * nb)
        layer.self_attn = attn
    model.starkv_quantized = quantized
    return model


@torch.no_grad()
def forward_tokens(model, ids: torch.Tensor, start: int, cache: StarKVCache) -> torch.Tensor:
    """Run tokens ``ids`` (B, n) at positions start..start+n-1 through every layer with
    the STAR-KV attention and ``cache``; returns the last position's logits (B, vocab)."""
    B, n = ids.shape
    h = model.model.embed_tokens(ids)
    pos = torch.arange(start, start + n, device=ids.device)[None].expand(B, n)
    cos, sin = model.model.rotary_emb(h, pos)
    quant = getattr(model, "starkv_quantized", True)
    for layer in model.model.layers:
        x = layer.input_layernorm(h)
        if quant:
            a, _ = layer.self_attn(x, (cos, sin), None, past_key_values_upper=cache)
        else:
            a, _ = layer.self_attn(x, (cos, sin), None, past_key_values=cache)
        h = h + a
        h = h + layer.mlp(layer.post_attention_layernorm(h))
    return model.lm_head(model.model.norm(h[:, -1:]))[:, 0]


@torch.no_grad()
def generate(model, prompt: torch.Tensor, new_tokens: int, capacity: int = 0, stats: Optional[dict] = None):
    """Greedy decode: returns (generated ids (B, new_tokens), decode seconds per token).
    ``stats`` (optional dict) receives ``prompt_s``: device time of the prompt pass."""
    B, P = prompt.shape
    cache = StarKVCache(capacity or P + new_tokens, quantized=getattr(model, "starkv_quantized", True))
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record()
    logits = forward_tokens(model, prompt, 0, cache)
    p1.record()
    tok = logits.argmax(-1, keepdim=True)
    out: List[torch.Tensor] = [tok]
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for s in range(new_tokens - 1):
        logits = forward_tokens(model, tok, P + s, cache)
        tok = logits.argmax(-1, keepdim=True)
        out.append(tok)
    e1.record()
    torch.cuda.synchronize()
    per_tok = e0.elapsed_time(e1) / 1e3 / max(1, new_tokens - 1)
    if stats is not None:
        stats["prompt_s"] = p0.elapsed_time(p1) / 1e3
    return torch.cat(out, dim=1), per_tok


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--context", type=int, default=4096)
    ap.add_argument("--new", type=int, default=128)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--unquantized", action="store_true")
    a = ap.parse_args()
    t0 = time.time()
    model = build_model(num_layers=a.layers, quantized=not a.unquantized, seed=a.seed)
    g = torch.Generator(device="cuda").manual_seed(a.seed + 1)
    prompt = torch.randint(0, model.config.vocab_size, (a.batch, a.context), generator=g, device="cuda")
    generate(model, prompt[:, :16], 4)                      # warm-up (kernels, workspaces)
    st = {}
    ids, per_tok = generate(model, prompt, a.new, stats=st)
    print(json.dumps({"metric": "end-to-end greedy decode (c3)", "value": a.batch / per_tok, "unit": "tokens/s",
                      "ms_per_token": per_tok * 1e3, "prompt_ms": st["prompt_s"] * 1e3, "batch": a.batch, "context": a.context, "new_tokens": a.new,
                      "layers": a.layers, "quantized": not a.unquantized, "weights": "random-init fp16",
                      "first_tokens": ids[0, :8].tolist(), "wall_s": time.time() - t0}))


if __name__ == "__main__":
    main()
