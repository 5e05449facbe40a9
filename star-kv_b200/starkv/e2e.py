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

from .attention import LlamaCustomAttention, LlamaCustomAttentionQuant, StarKVCache, apply_rotary_pos_emb_custom
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


@torch.no_grad()
def generate_graphed(model, prompt: torch.Tensor, new_tokens: int, capacity: int = 0,
                     stats: Optional[dict] = None):
    """``generate`` with each decode step's dense work replayed from CUDA graphs.

    The attention call of a step takes its token count from the host (the kernels'
    grids and split partitions depend on it), so it stays outside the graphs; the
    rest of a layer is captured once: graph A_i (input norm, q_proj, RoPE of the
    query) and graph B_i (o_proj, residual, post-attention norm, MLP, residual),
    plus one graph for the token embedding and RoPE tables and one for the LM
    head and argmax.  A step is then 2 + 2L graph launches and 2L C-ABI calls
    (``starkv_project_append`` + ``starkv_decode_attention`` per layer) on the
    current stream, all on static buffers.  Returns what ``generate`` returns,
    with the same tokens."""
    B, P = prompt.shape
    quant = getattr(model, "starkv_quantized", True)
    cache = StarKVCache(capacity or P + new_tokens, quantized=quant)
    dev = prompt.device
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record()
    logits = forward_tokens(model, prompt, 0, cache)
    p1.record()
    tok = logits.argmax(-1, keepdim=True)
    out: List[torch.Tensor] = [tok]
    layers = model.model.layers
    dt = model.model.embed_tokens.weight.dtype
    attn0 = layers[0].self_attn
    Hq, D = attn0.num_heads, attn0.head_dim
    tok_s = tok.clone()
    pos_s = torch.full((B, 1), P, dtype=torch.long, device=dev)
    h_s = torch.empty(B, 1, model.config.hidden_size, dtype=dt, device=dev)
    x_s = torch.empty_like(h_s)
    q_s = torch.empty(B, Hq, D, dtype=dt, device=dev)
    attn_s = torch.empty(B, Hq, D, dtype=dt, device=dev)
    cos_s = torch.empty(B, 1, D, dtype=dt, device=dev)
    sin_s = torch.empty_like(cos_s)
    vs = [(l.self_attn.k_proj.VS.weight.to(dt).contiguous(), l.self_attn.v_proj.VS.weight.to(dt).contiguous())
          for l in layers]
    states = [cache.layer(i, l.self_attn, B, dt) for i, l in enumerate(layers)]

    def embed():
        h_s.copy_(model.model.embed_tokens(tok_s))
        c, s_ = model.model.rotary_emb(h_s, pos_s)
        cos_s.copy_(c)
        sin_s.copy_(s_)

    def pre(i):
        layer = layers[i]
        x_s.copy_(layer.input_layernorm(h_s))
        q = layer.self_attn.q_proj(x_s).view(B, 1, Hq, D).transpose(1, 2)
        q_s.copy_(apply_rotary_pos_emb_custom(q, cos_s, sin_s)[:, :, 0, :])

    def post(i):
        layer = layers[i]
        h_s.add_(layer.self_attn.o_proj(attn_s.reshape(B, 1, Hq * D)))
        h_s.add_(layer.mlp(layer.post_attention_layernorm(h_s)))

    def head():
        lg = model.lm_head(model.model.norm(h_s))[:, 0]
        tok_s.copy_(lg.argmax(-1, keepdim=True))
        pos_s.add_(1)

    fns = [embed] + [(lambda i=i: pre(i)) for i in range(len(layers))] + \
          [(lambda i=i: post(i)) for i in range(len(layers))] + [head]
    # warm the captured ops on a side stream (allocator pools, cuBLAS handles), as torch requires
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    saved = (tok_s.clone(), pos_s.clone())
    with torch.cuda.stream(side):
        for f in fns:
            f()
    torch.cuda.current_stream().wait_stream(side)
    tok_s.copy_(saved[0])
    pos_s.copy_(saved[1])
    graphs = []
    pool = None
    for f in fns:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=pool):
            f()
        pool = g.pool()
        graphs.append(g)
    g_embed, g_pre, g_post, g_head = graphs[0], graphs[1:1 + len(layers)], graphs[1 + len(layers):-1], graphs[-1]
    steps = [st.prepared_step(q_s, x_s, vs[i][0], vs[i][1], attn_s) for i, st in enumerate(states)]
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for s in range(new_tokens - 1):
        g_embed.replay()
        for i in range(len(states)):
            g_pre[i].replay()
            steps[i]()
            g_post[i].replay()
        g_head.replay()
        out.append(tok_s.clone())
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
    ap.add_argument("--no-graphs", action="store_true", help="eager per-layer decode (no CUDA graphs)")
    a = ap.parse_args()
    t0 = time.time()
    model = build_model(num_layers=a.layers, quantized=not a.unquantized, seed=a.seed)
    g = torch.Generator(device="cuda").manual_seed(a.seed + 1)
    prompt = torch.randint(0, model.config.vocab_size, (a.batch, a.context), generator=g, device="cuda")
    gen = generate if a.no_graphs else generate_graphed
    gen(model, prompt[:, :16], 4)                           # warm-up (kernels, workspaces)
    st = {}
    ids, per_tok = gen(model, prompt, a.new, stats=st)
    print(json.dumps({"metric": "end-to-end greedy decode (c3)", "value": a.batch / per_tok, "unit": "tokens/s",
                      "ms_per_token": per_tok * 1e3, "prompt_ms": st["prompt_s"] * 1e3, "batch": a.batch, "context": a.context, "new_tokens": a.new,
                      "layers": a.layers, "quantized": not a.unquantized, "cuda_graphs": not a.no_graphs, "weights": "random-init fp16",
                      "first_tokens": ids[0, :8].tolist(), "wall_s": time.time() - t0}))


if __name__ == "__main__":
    main()
